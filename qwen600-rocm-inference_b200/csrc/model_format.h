// model_format.h — the Qwen3-0.6B checkpoint layout and its safetensors I/O.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

namespace qb {

struct TensorSpec {
    std::string name;
    std::vector<int64_t> shape;
    size_t offset = 0;   // byte offset in the canonical block (= safetensors data section)
    size_t bytes = 0;
};

// Canonical layout: the 311 tensors of Qwen3-0.6B (bf16) in byte-wise sorted
// name order, packed back to back from offset 0.  This is the layout of the
// reference's TENSOR_METADATA (static_loader.h:83-400) — lm_head first, layers
// in string order 0,1,10,...,19,2,20,... — derived here from the architecture
// instead of stored as a table.
const std::vector<TensorSpec>& canonical_table();
size_t canonical_total_bytes();
int canonical_index(const std::string& name);   // -1 if absent

// Index of each per-layer tensor in the canonical table.
struct LayerIndex {
    int in_ln, down, gate, up, post_ln, k_norm, k_proj, o_proj, q_norm, q_proj, v_proj;
};
LayerIndex layer_index(int layer);
int embed_index();
int lm_head_index();
int final_norm_index();

// A parsed safetensors header: for every canonical tensor, where it lies in the
// file (absolute byte offset).  Validates dtype (BF16), shape, bounds, overlap.
struct CheckpointMap {
    std::vector<size_t> file_offset;   // indexed like canonical_table()
    size_t file_bytes = 0;
    size_t data_start = 0;             // 8 + header length (0 for an ordered blob)
    bool canonical_order = false;      // data section is byte-identical in layout to the block
    bool blob = false;                 // the tensors come from an ordered weight blob
    std::string source;                // the file the tensors are read from
};
// Returns 0 or a QWEN_E_* status; err receives a message.  `path` may name a
// safetensors file or an ordered weight blob (recognised by its exact size and
// the absence of a safetensors header).  Like the reference's loader
// (static_loader.hip.h:185-202), a blob named weights_qwen600.bin beside a
// safetensors file, of the exact size, is read instead of that file once the
// file's header has been validated.
int parse_checkpoint(const std::string& path, CheckpointMap& out, std::string& err);

// The reference's ordered weight blob (export.py:80-146): raw bf16 tensors
// back to back, no header, in the order embed_tokens, lm_head, final norm, then
// per layer q, k, v, o, q_norm, k_norm, gate, up, down, input_layernorm,
// post_attention_layernorm.  Indices into canonical_table().
const std::vector<int>& blob_order();
// Writes the blob of a (BF16) safetensors checkpoint.
int write_blob(const std::string& safetensors_path, const std::string& out_path, std::string& err);

// Synthetic checkpoint (see qwen_write_synthetic_checkpoint in qwen_b200.h).
int write_synthetic(const std::string& path, uint64_t seed, std::string& err);

}  // namespace qb
