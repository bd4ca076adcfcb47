/* static_loader_b200.h — the reference's weight-loader surface (static_loader.h,
 * Ramshankar07/qwen600-ROCm-inference) on top of libqwen_b200.so.
 *
 * A program written against the reference keeps its names:
 *
 *     qwen_loader::QwenWeights w;
 *     qwen_loader::load_qwen_weights("model.safetensors", w);     // static_loader.h:402
 *     bf16* q = w.layers[3].attention.q_proj_weight;             // static_loader.h:37-78
 *     size_t off = qwen_loader::TENSOR_METADATA[7].offset;        // static_loader.h:83-400
 *
 * Same names, member names and meaning as static_loader.h:37-78 (AttentionWeights,
 * FFNWeights, TransformerBlockWeights, QwenWeights), :80-81 (TOTAL_WEIGHTS_BYTES,
 * NUM_TENSORS), :83 (TensorMetadata), :85-400 (TENSOR_METADATA) and :402-494
 * (load_qwen_weights).  Differences, all in the direction of safety:
 *   - TENSOR_METADATA is derived from the architecture by the library
 *     (qwen_tensor_info) instead of being a stored table; it indexes the same way
 *     (TENSOR_METADATA[i].name / .offset / .size_bytes) and holds the same entries;
 *   - load_qwen_weights accepts the tensors of the file in any order (the
 *     reference requires its exact byte layout) and throws std::runtime_error
 *     on every failure (the reference exit()s on CUDA errors, static_loader.h:22-30);
 *   - the device block is released with qwen_weights_free by ~QwenWeights, as the
 *     reference releases it with cudaFree.
 * bf16 is __nv_bfloat16 when <cuda_bf16.h> is reachable (as in the reference),
 * else a 16-bit storage type of the same size.  Everything is inline, so several
 * translation units may include this header.
 */
#ifndef STATIC_LOADER_B200_H
#define STATIC_LOADER_B200_H

#include <cstddef>
#include <stdexcept>
#include <string>

#include "qwen_b200.h"

#if defined(__has_include)
#if __has_include(<cuda_bf16.h>)
#include <cuda_bf16.h>
#define QWEN_B200_HAVE_CUDA_BF16 1
#endif
#endif

namespace qwen_loader {

#ifdef QWEN_B200_HAVE_CUDA_BF16
using bf16 = __nv_bfloat16;
#else
struct bf16 { unsigned short bits; };
#endif
static_assert(sizeof(bf16) == 2, "bf16 is a 16-bit type");

struct AttentionWeights {
    bf16* q_proj_weight = nullptr;
    bf16* k_proj_weight = nullptr;
    bf16* v_proj_weight = nullptr;
    bf16* o_proj_weight = nullptr;
    bf16* q_norm_weight = nullptr;
    bf16* k_norm_weight = nullptr;
};

struct FFNWeights {
    bf16* gate_proj_weight = nullptr;
    bf16* up_proj_weight = nullptr;
    bf16* down_proj_weight = nullptr;
};

struct TransformerBlockWeights {
    bf16* input_layernorm_weight = nullptr;
    bf16* post_attention_layernorm_weight = nullptr;
    AttentionWeights attention;
    FFNWeights ffn;
};

/* Number of transformer blocks (config.h N_LAYERS). */
constexpr int QWEN_B200_N_LAYERS = 28;

struct QwenWeights {
    bf16* token_embedding_table = nullptr;                  /* model.embed_tokens.weight */
    TransformerBlockWeights layers[QWEN_B200_N_LAYERS];
    bf16* final_norm_weight = nullptr;                      /* model.norm.weight */
    bf16* output_head_weight = nullptr;                     /* lm_head.weight */
    void* _gpu_mem_block = nullptr;                         /* owned block (load_qwen_weights), or nullptr */

    ~QwenWeights() {
        if (_gpu_mem_block) qwen_weights_free(_gpu_mem_block);
    }
};

/* static_loader.h:80-81 */
const size_t TOTAL_WEIGHTS_BYTES = 1503264768;
const int NUM_TENSORS = 311;

struct TensorMetadata {
    const char* name;
    size_t offset;
    size_t size_bytes;
};

/* TENSOR_METADATA[i] as in static_loader.h:83-400: entry i of the canonical
 * (byte-sorted name) layout, filled from the library on first use. */
class TensorMetadataTable {
public:
    const TensorMetadata& operator[](int i) const {
        fill();
        if (i < 0 || i >= NUM_TENSORS) throw std::out_of_range("TENSOR_METADATA index out of range");
        return entries_[i];
    }

private:
    void fill() const {
        if (filled_) return;
        if (qwen_num_tensors() != NUM_TENSORS || qwen_total_weight_bytes() != TOTAL_WEIGHTS_BYTES)
            throw std::runtime_error("libqwen_b200 was built for a different tensor layout");
        for (int i = 0; i < NUM_TENSORS; i++) {
            const char* n = nullptr;
            size_t off = 0, bytes = 0;
            if (qwen_tensor_info(i, &n, &off, &bytes) != QWEN_OK) throw std::runtime_error(qwen_last_error());
            entries_[i] = TensorMetadata{n, off, bytes};
        }
        filled_ = true;
    }
    mutable TensorMetadata entries_[NUM_TENSORS] = {};
    mutable bool filled_ = false;
};

inline const TensorMetadataTable TENSOR_METADATA{};

/* Points every member of `w` at its tensor inside the canonical device block
 * `block` (found by name, so the assignment does not depend on table order). */
inline void assign_weight_pointers(void* block, QwenWeights& w) {
    char* base = static_cast<char*>(block);
    auto at = [&](const std::string& name) -> bf16* {
        for (int i = 0; i < NUM_TENSORS; i++)
            if (name == TENSOR_METADATA[i].name) return reinterpret_cast<bf16*>(base + TENSOR_METADATA[i].offset);
        throw std::runtime_error("tensor " + name + " missing from the canonical layout");
    };
    w.token_embedding_table = at("model.embed_tokens.weight");
    w.final_norm_weight = at("model.norm.weight");
    w.output_head_weight = at("lm_head.weight");
    for (int l = 0; l < QWEN_B200_N_LAYERS; l++) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        TransformerBlockWeights& b = w.layers[l];
        b.input_layernorm_weight = at(p + "input_layernorm.weight");
        b.post_attention_layernorm_weight = at(p + "post_attention_layernorm.weight");
        b.attention.q_proj_weight = at(p + "self_attn.q_proj.weight");
        b.attention.k_proj_weight = at(p + "self_attn.k_proj.weight");
        b.attention.v_proj_weight = at(p + "self_attn.v_proj.weight");
        b.attention.o_proj_weight = at(p + "self_attn.o_proj.weight");
        b.attention.q_norm_weight = at(p + "self_attn.q_norm.weight");
        b.attention.k_norm_weight = at(p + "self_attn.k_norm.weight");
        b.ffn.gate_proj_weight = at(p + "mlp.gate_proj.weight");
        b.ffn.up_proj_weight = at(p + "mlp.up_proj.weight");
        b.ffn.down_proj_weight = at(p + "mlp.down_proj.weight");
    }
}

/* static_loader.h:402-494: the checkpoint into ONE device block (device 0, as
 * in the reference) in the canonical layout, and every pointer of `weights`. */
inline void load_qwen_weights(const std::string& filepath, QwenWeights& weights, int device = 0) {
    if (weights._gpu_mem_block) {
        qwen_weights_free(weights._gpu_mem_block);
        weights._gpu_mem_block = nullptr;
    }
    void* block = nullptr;
    if (qwen_weights_load(filepath.c_str(), device, &block) != QWEN_OK)
        throw std::runtime_error("load_qwen_weights: " + std::string(qwen_last_error()));
    weights._gpu_mem_block = block;
    assign_weight_pointers(block, weights);
}

}  // namespace qwen_loader

#endif /* STATIC_LOADER_B200_H */
