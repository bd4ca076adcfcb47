// Drives the reference-named loader surface (include/static_loader_b200.h and
// Transformer.weights in include/qwen_model_b200.h) the way code written
// against static_loader.h / qwen_model.cuh does.
//   shim_loader table            prints NUM_TENSORS, TOTAL_WEIGHTS_BYTES and
//                                every TENSOR_METADATA entry (no GPU needed)
//   shim_loader load <ckpt>      load_qwen_weights + build_transformer on device 0:
//                                checks every member pointer of both against the
//                                canonical offsets and prints an FNV-1a hash of
//                                a few tensors read back from each block
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "qwen_model_b200.h"

using namespace qwen_loader;

static uint64_t fnv(const std::vector<uint8_t>& v) {
    uint64_t h = 1469598103934665603ull;
    for (uint8_t b : v) { h ^= b; h *= 1099511628211ull; }
    return h;
}

static size_t offset_of(const std::string& name) {
    for (int i = 0; i < NUM_TENSORS; i++)
        if (name == TENSOR_METADATA[i].name) return TENSOR_METADATA[i].offset;
    throw std::runtime_error("no tensor " + name);
}

static int check_pointers(const QwenWeights& w, const void* block, const char* who) {
    const char* b = static_cast<const char*>(block);
    int bad = 0;
    auto chk = [&](const bf16* p, const std::string& name) {
        if (reinterpret_cast<const char*>(p) != b + offset_of(name)) { std::fprintf(stderr, "%s: %s misplaced\n", who, name.c_str()); bad++; }
    };
    chk(w.token_embedding_table, "model.embed_tokens.weight");
    chk(w.final_norm_weight, "model.norm.weight");
    chk(w.output_head_weight, "lm_head.weight");
    for (int l = 0; l < QWEN_B200_N_LAYERS; l++) {
        const std::string p = "model.layers." + std::to_string(l) + ".";
        const TransformerBlockWeights& L = w.layers[l];
        chk(L.input_layernorm_weight, p + "input_layernorm.weight");
        chk(L.post_attention_layernorm_weight, p + "post_attention_layernorm.weight");
        chk(L.attention.q_proj_weight, p + "self_attn.q_proj.weight");
        chk(L.attention.k_proj_weight, p + "self_attn.k_proj.weight");
        chk(L.attention.v_proj_weight, p + "self_attn.v_proj.weight");
        chk(L.attention.o_proj_weight, p + "self_attn.o_proj.weight");
        chk(L.attention.q_norm_weight, p + "self_attn.q_norm.weight");
        chk(L.attention.k_norm_weight, p + "self_attn.k_norm.weight");
        chk(L.ffn.gate_proj_weight, p + "mlp.gate_proj.weight");
        chk(L.ffn.up_proj_weight, p + "mlp.up_proj.weight");
        chk(L.ffn.down_proj_weight, p + "mlp.down_proj.weight");
    }
    return bad;
}

static uint64_t read_hash(const void* dev, size_t bytes) {
    std::vector<uint8_t> h(bytes);
    if (cudaMemcpy(h.data(), dev, bytes, cudaMemcpyDeviceToHost) != cudaSuccess) throw std::runtime_error("cudaMemcpy failed");
    return fnv(h);
}

int main(int argc, char** argv) {
    try {
        if (argc >= 2 && std::strcmp(argv[1], "table") == 0) {
            std::printf("%d %zu\n", NUM_TENSORS, TOTAL_WEIGHTS_BYTES);
            for (int i = 0; i < NUM_TENSORS; i++)
                std::printf("%s %zu %zu\n", TENSOR_METADATA[i].name, TENSOR_METADATA[i].offset, TENSOR_METADATA[i].size_bytes);
            return 0;
        }
        if (argc >= 3 && std::strcmp(argv[1], "load") == 0) {
            QwenWeights w;
            load_qwen_weights(argv[2], w);
            int bad = check_pointers(w, w._gpu_mem_block, "load_qwen_weights");
            Transformer t;
            build_transformer(&t, argv[2]);
            bad += check_pointers(t.weights, qwen_device_weights(t.handle), "Transformer.weights");
            if (t.weights._gpu_mem_block != nullptr || t.state.d_logits_fp32 != qwen_device_logits(t.handle)) bad++;
            // a few tensors read back through the members a reference caller uses
            std::printf("%016llx %016llx\n", (unsigned long long)read_hash(w.layers[5].attention.q_proj_weight, 2048 * 1024 * 2),
                        (unsigned long long)read_hash(t.weights.layers[5].attention.q_proj_weight, 2048 * 1024 * 2));
            std::printf("%016llx %016llx\n", (unsigned long long)read_hash(w.layers[27].ffn.down_proj_weight, 1024 * 3072 * 2),
                        (unsigned long long)read_hash(t.weights.layers[27].ffn.down_proj_weight, 1024 * 3072 * 2));
            std::printf("%016llx %016llx\n", (unsigned long long)read_hash(w.final_norm_weight, 1024 * 2),
                        (unsigned long long)read_hash(t.weights.final_norm_weight, 1024 * 2));
            free_transformer(&t);
            return bad == 0 ? 0 : 1;
        }
    } catch (const std::exception& e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
    std::fprintf(stderr, "usage: %s table | load <checkpoint>\n", argv[0]);
    return 2;
}
