// engine.cu — the C ABI of include/qwen_b200.h: checkpoint upload, device
// buffers, the decode launches and the isolated GEMV.
//
// Reference counterparts (Ramshankar07/qwen600-ROCm-inference):
//   qwen_create        build_transformer + malloc_run_state (qwen_model.cuh:63-92)
//                      + load_qwen_weights (static_loader.h:402-494)
//   qwen_forward       forward (qwen_model.cuh:772-851)
//   qwen_decode_step   forward + sample (main.cu:144-145, sampler.h:120-175)
//   qwen_destroy       free_transformer (qwen_model.cuh:94-111)
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <mutex>
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <chrono>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/qwen_b200.h"
#include "decode_kernel.cuh"
#include "gemv_kernel.cuh"
#include "attention_tc5.cuh"
#include "gemm_tc.cuh"
#include "prefill_kernels.cuh"
#include "model_format.h"

using namespace qb;

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------
static thread_local std::string g_err;
static int fail(int code, const std::string& msg) { g_err = msg; return code; }
#define CU(call)                                                                                        \
    do {                                                                                                \
        cudaError_t e_ = (call);                                                                        \
        if (e_ != cudaSuccess) return fail(QWEN_E_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
    } while (0)

// Kernels of the prompt pass are launched with programmatic stream
// serialization: each may start (set up barriers and tensor memory, load
// weights) while the kernel before it finishes, and waits for it with
// pdl_wait before it reads anything that kernel produced (ptx.cuh).
// QWEN_B200_PDL=0 launches them normally.
static bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("QWEN_B200_PDL");
        return !(e && strcmp(e, "0") == 0);
    }();
    return on;
}
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}

extern "C" const char* qwen_last_error(void) { return g_err.c_str(); }
// for the library's host-only files (tokenizer.cpp)
int qwen_internal_fail(int code, const std::string& msg) { return fail(code, msg); }
extern "C" int qwen_abi_version(void) { return 10000; }

// ---------------------------------------------------------------------------
// tensor table / checkpoint
// ---------------------------------------------------------------------------
extern "C" int qwen_num_tensors(void) { return (int)canonical_table().size(); }
extern "C" int qwen_vocab_size(void) { return VOCAB_SIZE; }
extern "C" size_t qwen_total_weight_bytes(void) { return canonical_total_bytes(); }
extern "C" int qwen_tensor_info(int index, const char** name, size_t* offset, size_t* bytes) {
    const auto& t = canonical_table();
    if (index < 0 || index >= (int)t.size()) return fail(QWEN_E_ARG, "tensor index out of range");
    if (name) *name = t[index].name.c_str();
    if (offset) *offset = t[index].offset;
    if (bytes) *bytes = t[index].bytes;
    return QWEN_OK;
}
extern "C" int qwen_checkpoint_validate(const char* path) {
    if (!path) return fail(QWEN_E_ARG, "path is NULL");
    CheckpointMap m; std::string err;
    const int rc = parse_checkpoint(path, m, err);
    return rc == QWEN_OK ? QWEN_OK : fail(rc, err);
}
extern "C" int qwen_write_ordered_blob(const char* safetensors_path, const char* out_path) {
    if (!safetensors_path || !out_path) return fail(QWEN_E_ARG, "NULL argument");
    std::string err;
    const int rc = write_blob(safetensors_path, out_path, err);
    return rc == QWEN_OK ? QWEN_OK : fail(rc, err);
}

extern "C" int qwen_write_synthetic_checkpoint(const char* path, uint64_t seed) {
    if (!path) return fail(QWEN_E_ARG, "path is NULL");
    std::string err;
    const int rc = write_synthetic(path, seed, err);
    return rc == QWEN_OK ? QWEN_OK : fail(rc, err);
}

// Stream the checkpoint's tensors to their canonical offsets in `dev` through
// two pinned staging buffers (read of one overlaps the copy of the other).
static int upload_checkpoint(const std::string& path, const CheckpointMap& m, uint8_t* dev, cudaStream_t st) {
    const auto& t = canonical_table();
    struct Seg { size_t f, d, n; };
    std::vector<Seg> segs;
    std::vector<int> order(t.size());
    for (size_t i = 0; i < t.size(); i++) order[i] = (int)i;
    std::sort(order.begin(), order.end(), [&](int a, int b) { return m.file_offset[a] < m.file_offset[b]; });
    for (int i : order) {
        const Seg s{m.file_offset[i], t[i].offset, t[i].bytes};
        if (!segs.empty() && segs.back().f + segs.back().n == s.f && segs.back().d + segs.back().n == s.d) segs.back().n += s.n;
        else segs.push_back(s);
    }
    (void)path;
    const int fd = open(m.source.c_str(), O_RDONLY);
    if (fd < 0) return fail(QWEN_E_IO, "cannot open checkpoint: " + m.source);
    const size_t CH = (size_t)64 << 20;
    void* stage[2] = {nullptr, nullptr};
    cudaEvent_t ev[2] = {nullptr, nullptr};
    bool used[2] = {false, false};
    int rc = QWEN_OK;
    for (int i = 0; i < 2 && rc == QWEN_OK; i++) {
        if (cudaHostAlloc(&stage[i], CH, cudaHostAllocDefault) != cudaSuccess || cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) != cudaSuccess)
            rc = fail(QWEN_E_CUDA, "pinned staging allocation failed");
    }
    int b = 0;
    for (const Seg& s : segs) {
        for (size_t off = 0; off < s.n && rc == QWEN_OK; off += CH) {
            const size_t len = std::min(CH, s.n - off);
            if (used[b] && cudaEventSynchronize(ev[b]) != cudaSuccess) { rc = fail(QWEN_E_CUDA, "staging event wait failed"); break; }
            size_t got = 0;
            while (got < len) {
                const ssize_t r = pread(fd, (char*)stage[b] + got, len - got, (off_t)(s.f + off + got));
                if (r <= 0) { rc = fail(QWEN_E_IO, "short read from checkpoint (truncated file?)"); break; }
                got += (size_t)r;
            }
            if (rc != QWEN_OK) break;
            if (cudaMemcpyAsync(dev + s.d + off, stage[b], len, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                cudaEventRecord(ev[b], st) != cudaSuccess) { rc = fail(QWEN_E_CUDA, "weight upload failed"); break; }
            used[b] = true;
            b ^= 1;
        }
        if (rc != QWEN_OK) break;
    }
    if (cudaStreamSynchronize(st) != cudaSuccess && rc == QWEN_OK) rc = fail(QWEN_E_CUDA, "weight upload sync failed");
    for (int i = 0; i < 2; i++) { if (ev[i]) cudaEventDestroy(ev[i]); if (stage[i]) cudaFreeHost(stage[i]); }
    close(fd);
    return rc;
}

extern "C" int qwen_weights_load(const char* path, int device, void** dev_block) {
    if (!path || !dev_block) return fail(QWEN_E_ARG, "NULL argument");
    *dev_block = nullptr;
    CheckpointMap m; std::string err;
    int rc = parse_checkpoint(path, m, err);
    if (rc != QWEN_OK) return fail(rc, err);
    CU(cudaSetDevice(device));
    void* blk = nullptr;
    CU(cudaMalloc(&blk, canonical_total_bytes()));
    cudaStream_t st;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) { cudaFree(blk); return fail(QWEN_E_CUDA, "stream creation failed"); }
    rc = upload_checkpoint(path, m, (uint8_t*)blk, st);
    cudaStreamDestroy(st);
    if (rc != QWEN_OK) { cudaFree(blk); return rc; }
    *dev_block = blk;
    return QWEN_OK;
}
extern "C" int qwen_weights_free(void* dev_block) {
    if (dev_block) CU(cudaFree(dev_block));
    return QWEN_OK;
}

// ---------------------------------------------------------------------------
// load-time repacking
// ---------------------------------------------------------------------------
// Wo [DIM][Q_DIM] -> [8][DIM][256]: group g's 256 input columns contiguous per row.
// One layer's Wo [1024][2048] -> [8 groups][1024 rows][kWoCols]: group g's 256
// input columns of every row contiguous, then kWoCols - 256 zero pad columns.
__global__ void pack_wo_kernel(const uint16_t* __restrict__ wo, uint16_t* __restrict__ wo_g) {
    const size_t n = (size_t)kGroups * DIM * kWoCols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int g = (int)(i / ((size_t)DIM * kWoCols)), rem = (int)(i % ((size_t)DIM * kWoCols));
        const int r = rem / kWoCols, cc = rem % kWoCols;
        wo_g[i] = cc < 256 ? wo[(size_t)r * Q_DIM + 256 * g + cc] : (uint16_t)0;
    }
}

// gate and up rows interleaved in blocks of 128 (block 2j: gate rows 128j ..,
// block 2j+1: the same up rows), so one 128 x 256 GEMM tile holds both halves
// of 128 hidden units and its epilogue can apply SwiGLU.
__global__ void pack_gu_kernel(const uint16_t* __restrict__ wg, const uint16_t* __restrict__ wu, uint16_t* __restrict__ wgu) {
    const size_t n = (size_t)2 * HIDDEN_DIM * DIM / 8;   // 16-byte units
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const size_t row = i / (DIM / 8), col = i % (DIM / 8);
        const size_t j = row / 256, k = row % 256;
        const uint16_t* src = k < 128 ? wg + (128 * j + k) * DIM : wu + (128 * j + k - 128) * DIM;
        reinterpret_cast<uint4*>(wgu)[i] = reinterpret_cast<const uint4*>(src)[col];
    }
}

// RoPE cos/sin of every position, computed the way the reference writes it
// (qwen_model.cuh:331-334): freq = 1/powf(theta, 2j/128), angle = pos*freq in
// fp32.  The libm calls go through volatile pointers so the compiler cannot
// fold them at a different precision.
static void rope_table(std::vector<float>& tab) {
    float (*volatile p_pow)(float, float) = powf;
    void (*volatile p_sincos)(float, float*, float*) = sincosf;
    tab.assign((size_t)SEQ_LEN * HEAD_DIM, 0.f);
    for (int j = 0; j < HEAD_DIM / 2; j++) {
        const float freq = 1.0f / p_pow(ROPE_THETA, (float)(j * 2) / (float)HEAD_DIM);
        for (int pos = 0; pos < SEQ_LEN; pos++) {
            const float val = (float)pos * freq;
            float s, c;
            p_sincos(val, &s, &c);
            tab[(size_t)pos * HEAD_DIM + j] = c;
            tab[(size_t)pos * HEAD_DIM + 64 + j] = s;
        }
    }
}

// ---------------------------------------------------------------------------
// context
// ---------------------------------------------------------------------------
struct qwen_ctx {
    int device = 0;
    int nsm = 0;
    cudaStream_t stream = nullptr;
    uint8_t* wblock = nullptr;
    uint16_t *wo_g = nullptr, *kc = nullptr, *vc = nullptr;
    float *rope = nullptr, *logits = nullptr;
    uint64_t* xchg = nullptr;      // all exchange words (one allocation)
    size_t xchg_words = 0;
    unsigned long long launches = 0;   // since the last reset (bounds the 32-bit sequence tag)
    cudaGraphExec_t step_exec = nullptr;   // qwen_decode_step's copy-in, launch, copy-out, replayed
    // batched decode (qwen_batch_*): one KV cache per slot, allocated by qwen_batch_init
    int b_max = 0;
    uint16_t *bkc = nullptr, *bvc = nullptr;
    int *b_tokens = nullptr, *b_pos = nullptr, *b_ci = nullptr;
    float *b_logits = nullptr, *b_cv = nullptr, *b_part = nullptr;
    uint32_t* b_tk = nullptr;              // top-k level scratch: two key and two id lists
    std::vector<int> b_cached;
    std::unordered_map<int, cudaGraphExec_t> b_graphs;   // batch step per (batch, k), replayed
    bool b_graph_off = false;
    bool step_graph_off = false;           // capture failed once: direct launches from then on
    float *cand_v = nullptr, *top_v = nullptr;
    int *cand_i = nullptr, *top_i = nullptr, *prompt = nullptr, *tokens = nullptr, *chunk_count = nullptr;
    uint32_t* ctr = nullptr;
    StepIn* d_in = nullptr;
    StepOut* d_out = nullptr;
    StepIn* h_in = nullptr;
    StepOut* h_out = nullptr;
    float* h_logits = nullptr;
    int* h_tokens = nullptr;
    DecodeParams params{};
    // prompt pass on the tensor cores (allocated on first use)
    const uint16_t* wo_raw[N_LAYERS] = {};   // o_proj in the canonical block
    float *pf_x = nullptr, *pf_y = nullptr, *pf_q = nullptr, *pf_xn = nullptr;
    uint16_t* pf_as = nullptr;
    uint16_t* pf_hs = nullptr;   // SwiGLU output in three bf16 parts (written by the fused gate|up GEMM)
    uint16_t* wgu = nullptr;     // gate|up weights interleaved per 128 rows, all layers
    int shard_pos0 = -1, shard_steps = 0;   // the sharded-head loop in progress (qwen_shard_begin .. _finish)
    int cached = 0;
    bool gemm_prefill = true;   // qwen_prefill uses prefill_pass for long prompts
    int pf_parts = 2;           // bf16 parts of the activations the pass's projections read (3: fp32-exact, 2, 1)
    int att5 = 1;               // prompt-pass attention: 1 tcgen05 (attention_tc5.cuh, the default), 0 mma.sync
    bool qkv_epi = true;        // QK-norm, RoPE and the K/V append in the q|k|v GEMM's epilogue where it applies
    uint16_t* vt = nullptr;     // the layer's V transposed ([head][dim][position]) for the tcgen05 attention
    int last_k = 0;
};

static void ctx_free(qwen_t* c) {
    if (!c) return;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->params.trace) cudaFree(c->params.trace);
    void* dev[] = {c->pf_x, c->pf_y, c->pf_q, c->pf_xn, c->pf_as, c->pf_hs, c->wgu, c->vt, c->wblock, c->wo_g, c->kc, c->vc, c->rope, c->xchg, c->logits,
                   c->cand_v, c->top_v, c->cand_i, c->top_i, c->prompt, c->tokens, c->ctr, c->d_in, c->d_out, c->chunk_count};
    for (void* p : dev) if (p) cudaFree(p);
    void* host[] = {c->h_in, c->h_out, c->h_logits, c->h_tokens};
    for (void* p : host) if (p) cudaFreeHost(p);
    if (c->step_exec) cudaGraphExecDestroy(c->step_exec);
    for (auto& kv : c->b_graphs) cudaGraphExecDestroy(kv.second);
    void* bdev[] = {c->bkc, c->bvc, c->b_tokens, c->b_pos, c->b_ci, c->b_logits, c->b_cv, c->b_part, c->b_tk};
    for (void* p : bdev) if (p) cudaFree(p);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

static int reset_device_state(qwen_t* c) {
    CU(cudaMemsetAsync(c->ctr, 0, (size_t)kNumCtr * kCtrStride * sizeof(uint32_t), c->stream));
    CU(cudaMemsetAsync(c->xchg, 0, c->xchg_words * sizeof(uint64_t), c->stream));   // tag 0 is never current
    c->launches = 0;
    StepOut o{};
    o.seq = 1;
    *c->h_out = o;
    CU(cudaMemcpyAsync(c->d_out, c->h_out, sizeof(StepOut), cudaMemcpyHostToDevice, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    return QWEN_OK;
}

template <typename T>
static int dalloc(T** p, size_t n) {
    CU(cudaMalloc((void**)p, n * sizeof(T)));
    return QWEN_OK;
}
#define TRY(x) do { const int rc_ = (x); if (rc_ != QWEN_OK) { ctx_free(c); return rc_; } } while (0)

extern "C" int qwen_create(const char* path, int device, qwen_t** out) {
    if (!path || !out) return fail(QWEN_E_ARG, "NULL argument");
    *out = nullptr;
    CheckpointMap m; std::string err;
    int rc = parse_checkpoint(path, m, err);
    if (rc != QWEN_OK) return fail(rc, err);
    int ndev = 0;
    CU(cudaGetDeviceCount(&ndev));
    if (device < 0 || device >= ndev) return fail(QWEN_E_ARG, "device index out of range");
    CU(cudaSetDevice(device));
    qwen_t* c = new qwen_ctx();
    c->device = device;
    if (cudaDeviceGetAttribute(&c->nsm, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) { ctx_free(c); return fail(QWEN_E_CUDA, "device query failed"); }
    if (c->nsm < kGroups * kMinGS || c->nsm > kGroups * kMaxGS || (VOCAB_SIZE + c->nsm - 1) / c->nsm > kMaxLocalRows ||
        (HIDDEN_DIM + c->nsm - 1) / c->nsm > kMaxMlpRows) {
        ctx_free(c); return fail(QWEN_E_UNSUPPORTED, "unsupported SM count " + std::to_string(c->nsm));
    }
    for (auto kern : {decode_kernel<false>, decode_kernel<true>}) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kDecodeSmemBytes) != cudaSuccess) {
            ctx_free(c); return fail(QWEN_E_CUDA, "cannot reserve " + std::to_string(kDecodeSmemBytes) + " B of shared memory");
        }
        int nb = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, kern, kThreads, kDecodeSmemBytes) != cudaSuccess || nb < 1) {
            ctx_free(c); return fail(QWEN_E_CUDA, "decode kernel cannot be resident on every SM");
        }
    }
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess) { ctx_free(c); return fail(QWEN_E_CUDA, "stream creation failed"); }

    const size_t total = canonical_total_bytes();
    TRY(dalloc(&c->wblock, total));
    TRY(upload_checkpoint(path, m, c->wblock, c->stream));
    TRY(dalloc(&c->wo_g, (size_t)N_LAYERS * kGroups * DIM * kWoCols));
    TRY(dalloc(&c->wgu, (size_t)N_LAYERS * 2 * HIDDEN_DIM * DIM));
    const size_t kv = (size_t)N_LAYERS * N_KV_HEADS * SEQ_LEN * HEAD_DIM;
    TRY(dalloc(&c->kc, kv));
    TRY(dalloc(&c->vc, kv));
    TRY(dalloc(&c->rope, (size_t)SEQ_LEN * HEAD_DIM));
    const size_t n_xw = (size_t)(N_LAYERS + 1) * DIM, n_qkv = (size_t)N_LAYERS * 4096,
                 n_part = (size_t)N_LAYERS * kGroups * kMaxGS * kPartStride, n_y = (size_t)N_LAYERS * kGroups * DIM,
                 n_h = (size_t)N_LAYERS * HIDDEN_DIM;
    c->xchg_words = n_xw + n_qkv + n_part + n_y + n_h;
    TRY(dalloc(&c->xchg, c->xchg_words));
    TRY(dalloc(&c->logits, (size_t)VOCAB_SIZE));
    TRY(dalloc(&c->cand_v, (size_t)c->nsm * kMaxCand));
    TRY(dalloc(&c->cand_i, (size_t)c->nsm * kMaxCand));
    TRY(dalloc(&c->top_v, (size_t)kMaxCand));
    TRY(dalloc(&c->top_i, (size_t)kMaxCand));
    TRY(dalloc(&c->prompt, (size_t)SEQ_LEN));
    TRY(dalloc(&c->tokens, (size_t)SEQ_LEN));
    TRY(dalloc(&c->ctr, (size_t)kNumCtr * kCtrStride));
    TRY(dalloc(&c->chunk_count, (size_t)2 * c->nsm));
    TRY(dalloc(&c->d_in, 1));
    TRY(dalloc(&c->d_out, 1));
    if (cudaHostAlloc((void**)&c->h_in, sizeof(StepIn), 0) != cudaSuccess || cudaHostAlloc((void**)&c->h_out, sizeof(StepOut), 0) != cudaSuccess ||
        cudaHostAlloc((void**)&c->h_logits, (size_t)VOCAB_SIZE * sizeof(float), 0) != cudaSuccess ||
        cudaHostAlloc((void**)&c->h_tokens, (size_t)SEQ_LEN * sizeof(int), 0) != cudaSuccess) {
        ctx_free(c); return fail(QWEN_E_CUDA, "pinned host allocation failed");
    }
    if (cudaMemsetAsync(c->kc, 0, kv * 2, c->stream) != cudaSuccess || cudaMemsetAsync(c->vc, 0, kv * 2, c->stream) != cudaSuccess ||
        cudaMemsetAsync(c->prompt, 0, SEQ_LEN * sizeof(int), c->stream) != cudaSuccess) {
        ctx_free(c); return fail(QWEN_E_CUDA, "memset failed");
    }
    std::vector<float> tab;
    rope_table(tab);
    if (cudaMemcpyAsync(c->rope, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice, c->stream) != cudaSuccess) {
        ctx_free(c); return fail(QWEN_E_CUDA, "rope upload failed");
    }

    DecodeParams& P = c->params;
    auto W = [&](int idx) { return (const uint16_t*)(c->wblock + canonical_table()[idx].offset); };
    P.embed = W(embed_index());
    P.lm = W(lm_head_index());
    P.final_ln = W(final_norm_index());
    for (int l = 0; l < N_LAYERS; l++) {
        const LayerIndex li = layer_index(l);
        P.in_ln[l] = W(li.in_ln); P.post_ln[l] = W(li.post_ln);
        P.wq[l] = W(li.q_proj); P.wk[l] = W(li.k_proj); P.wv[l] = W(li.v_proj);
        P.qn[l] = W(li.q_norm); P.kn[l] = W(li.k_norm);
        P.wg[l] = W(li.gate); P.wu[l] = W(li.up); P.wd[l] = W(li.down);
        pack_wo_kernel<<<1024, 256, 0, c->stream>>>(W(li.o_proj), c->wo_g + (size_t)l * kGroups * DIM * kWoCols);
        pack_gu_kernel<<<1024, 256, 0, c->stream>>>(W(li.gate), W(li.up), c->wgu + (size_t)l * 2 * HIDDEN_DIM * DIM);
        c->wo_raw[l] = W(li.o_proj);
    }
    if (cudaGetLastError() != cudaSuccess) { ctx_free(c); return fail(QWEN_E_CUDA, "repack launch failed"); }
    P.wo_g = c->wo_g; P.kc = c->kc; P.vc = c->vc; P.rope = c->rope; P.prompt = c->prompt;
    P.xw = c->xchg; P.qkvw = P.xw + n_xw; P.partw = P.qkvw + n_qkv; P.yw = P.partw + n_part; P.hw = P.yw + n_y;
    P.logits = c->logits;
    P.cand_v = c->cand_v; P.cand_i = c->cand_i; P.top_v = c->top_v; P.top_i = c->top_i; P.ctr = c->ctr;
    P.in = c->d_in; P.out = c->d_out; P.tokens_out = c->tokens; P.tokens_cap = SEQ_LEN;
    P.lm_begin = 0; P.lm_end = VOCAB_SIZE;
    // tuning knobs (environment, read once per handle): L2 prefetch lead in
    // chunks, back-off in ns between polls of an exchange word
    P.prefetch_chunks = 0;
    P.poll_ns = 0;
    P.wait_ns = kWaitNs;
    P.debug_skip = -1;
    if (const char* e = getenv("QWEN_B200_PREFETCH")) P.prefetch_chunks = std::max(0, std::min(64, atoi(e)));
    if (const char* e = getenv("QWEN_B200_POLL_NS")) P.poll_ns = std::max(0, std::min(2000, atoi(e)));
    // prompt-pass attention: "tc5" selects the tcgen05 kernel, "mma" the mma.sync one
    if (const char* e = getenv("QWEN_B200_PREFILL_ATTN")) c->att5 = strcmp(e, "mma") == 0 ? 0 : 1;
    // "0": q|k|v GEMM with fp32 output, then qkv_post_kernel, in every prompt pass
    if (const char* e = getenv("QWEN_B200_QKV_EPILOGUE")) c->qkv_epi = strcmp(e, "0") != 0;
    P.chunk_count = c->chunk_count;
    TRY(reset_device_state(c));
    *out = c;
    return QWEN_OK;
}

extern "C" void qwen_destroy(qwen_t* c) { ctx_free(c); }
extern "C" int qwen_device(const qwen_t* c) { return c ? c->device : -1; }
extern "C" float* qwen_host_logits(qwen_t* c) { return c ? c->h_logits : nullptr; }
extern "C" const float* qwen_device_logits(qwen_t* c) { return c ? c->logits : nullptr; }
extern "C" const void* qwen_device_weights(const qwen_t* c) { return c ? c->wblock : nullptr; }
extern "C" int qwen_cached_positions(const qwen_t* c) { return c ? c->cached : -1; }

static int count_launch(qwen_t* c) {
    if (++c->launches >= 0xFFFFFF00ull) {   // the 32-bit exchange tag is about to wrap: start over
        CU(cudaStreamSynchronize(c->stream));
        const int rc = reset_device_state(c);
        if (rc != QWEN_OK) return rc;
        c->launches = 1;
    }
    return QWEN_OK;
}

static int enqueue_decode(qwen_t* c) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)c->nsm);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kDecodeSmemBytes;
    cfg.stream = c->stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (c->params.trace) CU(cudaLaunchKernelEx(&cfg, decode_kernel<true>, c->params));
    else CU(cudaLaunchKernelEx(&cfg, decode_kernel<false>, c->params));
    return QWEN_OK;
}

static int launch_decode(qwen_t* c) {
    const int rc = count_launch(c);
    return rc != QWEN_OK ? rc : enqueue_decode(c);
}

// qwen_decode_step's device work — StepIn in, one decode launch, StepOut out —
// as a CUDA graph, captured once per handle and replayed (one API call per
// token instead of three).  The launch tag lives in device memory, so the
// same graph serves every step; changes to the kernel's by-value parameters
// (vocabulary shard, tracing) drop it.  If capture or instantiation fails the
// handle keeps the direct launches.
static void drop_step_graph(qwen_t* c) {
    if (c->step_exec) cudaGraphExecDestroy(c->step_exec);
    c->step_exec = nullptr;
}

static void build_step_graph(qwen_t* c) {
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) != cudaSuccess) { c->step_graph_off = true; return; }
    bool ok = cudaMemcpyAsync(c->d_in, c->h_in, sizeof(StepIn), cudaMemcpyHostToDevice, c->stream) == cudaSuccess;
    ok = ok && enqueue_decode(c) == QWEN_OK;
    ok = ok && cudaMemcpyAsync(c->h_out, c->d_out, sizeof(StepOut), cudaMemcpyDeviceToHost, c->stream) == cudaSuccess;
    const bool ended = cudaStreamEndCapture(c->stream, &g) == cudaSuccess;
    if (ok && ended && g && cudaGraphInstantiate(&c->step_exec, g, 0) != cudaSuccess) c->step_exec = nullptr;
    if (g) cudaGraphDestroy(g);
    if (!c->step_exec) {
        c->step_graph_off = true;
        cudaGetLastError();   // clear a capture error; the direct path reports its own
    }
}

// After a synchronised launch sequence: surface a device-side wait timeout.
static int check_step(qwen_t* c) {
    if (c->h_out->err) {
        const unsigned e = c->h_out->err; const int w = c->h_out->err_where;
        reset_device_state(c);
        c->cached = 0;
        if (e & 24u)   // 8: invalid input token on device, 16: no finite logit to sample
            return fail(QWEN_E_STATE, "non-finite logits or invalid chained token (code " + std::to_string(e) +
                                          "); device state reset, KV cache invalidated");
        return fail(QWEN_E_TIMEOUT, "device wait expired (code " + std::to_string(e) + ", where " + std::to_string(w) +
                                        "); device state reset, KV cache invalidated");
    }
    return QWEN_OK;
}

static int check_sampling(const qwen_sampling_t* sp) {
    if (!sp) return QWEN_OK;
    if (!(sp->temperature >= 0.0f)) return fail(QWEN_E_ARG, "temperature must be >= 0");
    if (sp->top_k < 0) return fail(QWEN_E_ARG, "top_k must be >= 0 (0 means the full vocabulary)");
    return QWEN_OK;
}

static bool is_greedy(const qwen_sampling_t* sp) { return !sp || sp->temperature == 0.0f || sp->top_k == 1; }

// Sampling settings the device sampler reproduces token for token.  The
// reference draws over its candidates in the order its quickselect leaves them
// (sampler.h:131-134) and, with the nucleus cut on, re-sorts them by
// probability first (sampler.h:153-156).  With the cut on and at most kMaxCand
// candidates the device's descending order is that order (candidates whose
// fp32 logits are exactly equal aside); with the cut off (topp outside (0, 1))
// the order is the partition order of a quickselect over the whole
// vocabulary, which only that sequential pass reproduces, and top_k = 0 or
// > kMaxCand exceeds the device list.  Those settings sample on the host from
// the device logits (qwen_sample_host, the reference's own order).
static bool device_exact(const qwen_sampling_t* sp) {
    return is_greedy(sp) || (sp->topp > 0.0f && sp->topp < 1.0f && sp->top_k >= 1 && sp->top_k <= kMaxCand);
}

static void fill_in(qwen_t* c, int token, int pos, const qwen_sampling_t* sp, unsigned long long rng, int flags) {
    StepIn& in = *c->h_in;
    in.token = token; in.pos = pos; in.flags = flags; in.rng = rng;
    if (sp) { in.temperature = sp->temperature; in.topp = sp->topp; in.top_k = sp->top_k; }
    else { in.temperature = 0.f; in.topp = 1.f; in.top_k = 1; }
}

extern "C" int qwen_forward(qwen_t* c, int token, int pos, float* logits_host) {
    if (!c) return fail(QWEN_E_ARG, "NULL handle");
    if (token < 0 || token >= VOCAB_SIZE) return fail(QWEN_E_ARG, "token out of range");
    if (pos < 0 || pos >= SEQ_LEN) return fail(QWEN_E_ARG, "pos out of range [0, SEQ_LEN)");
    if (pos > c->cached) return fail(QWEN_E_STATE, "pos skips uncached positions");
    if (c->params.lm_begin != 0 || c->params.lm_end != VOCAB_SIZE) {
        if (logits_host) return fail(QWEN_E_STATE, "full logits requested from a vocabulary-sharded handle");
    }
    CU(cudaSetDevice(c->device));
    fill_in(c, token, pos, nullptr, 0, kFlagWriteLogits);
    CU(cudaMemcpyAsync(c->d_in, c->h_in, sizeof(StepIn), cudaMemcpyHostToDevice, c->stream));
    int rc = launch_decode(c);
    if (rc != QWEN_OK) return rc;
    if (logits_host) CU(cudaMemcpyAsync(logits_host, c->logits, (size_t)VOCAB_SIZE * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaMemcpyAsync(c->h_out, c->d_out, sizeof(StepOut), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    c->last_k = 1;
    if ((rc = check_step(c)) != QWEN_OK) return rc;
    c->cached = pos + 1;
    return QWEN_OK;
}

// n_steps chained steps whose token is drawn on the host from each step's
// device logits by qwen_sample_host (settings device_exact() rejects): one
// launch, one logits copy and one host draw per step.  *device_ms (if given)
// receives the time of the whole loop, host draws included.
static int host_sampled_steps(qwen_t* c, int token, int pos, int n_steps, const qwen_sampling_t* sp, unsigned long long* rng_state,
                              int* tokens_out, float* device_ms) {
    if (!rng_state) return fail(QWEN_E_ARG, "sampling needs rng_state");
    if (c->params.lm_begin != 0 || c->params.lm_end != VOCAB_SIZE)
        return fail(QWEN_E_UNSUPPORTED, "this sampling setting draws over the full vocabulary on the host; the handle serves a vocabulary shard");
    CU(cudaSetDevice(c->device));
    const auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < n_steps; i++) {
        fill_in(c, token, pos + i, nullptr, 0, kFlagWriteLogits);
        CU(cudaMemcpyAsync(c->d_in, c->h_in, sizeof(StepIn), cudaMemcpyHostToDevice, c->stream));
        int rc = launch_decode(c);
        if (rc != QWEN_OK) return rc;
        CU(cudaMemcpyAsync(c->h_logits, c->logits, (size_t)VOCAB_SIZE * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
        CU(cudaMemcpyAsync(c->h_out, c->d_out, sizeof(StepOut), cudaMemcpyDeviceToHost, c->stream));
        CU(cudaStreamSynchronize(c->stream));
        if ((rc = check_step(c)) != QWEN_OK) return rc;
        c->cached = pos + i + 1;
        if ((rc = qwen_sample_host(c->h_logits, VOCAB_SIZE, sp, rng_state, &token)) != QWEN_OK)
            return fail(rc, "host sampling failed");
        tokens_out[i] = token;
    }
    if (device_ms) *device_ms = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - t0).count();
    c->last_k = 1;
    return QWEN_OK;
}

extern "C" int qwen_decode_step(qwen_t* c, int token, int pos, const qwen_sampling_t* sp, unsigned long long* rng_state, int* next) {
    if (!c || !next) return fail(QWEN_E_ARG, "NULL argument");
    if (token < 0 || token >= VOCAB_SIZE) return fail(QWEN_E_ARG, "token out of range");
    if (pos < 0 || pos >= SEQ_LEN) return fail(QWEN_E_ARG, "pos out of range [0, SEQ_LEN)");
    if (pos > c->cached) return fail(QWEN_E_STATE, "pos skips uncached positions");
    int rc = check_sampling(sp);
    if (rc != QWEN_OK) return rc;
    if (!device_exact(sp)) return host_sampled_steps(c, token, pos, 1, sp, rng_state, next, nullptr);
    CU(cudaSetDevice(c->device));
    if (!c->step_exec && !c->step_graph_off && !c->params.trace) build_step_graph(c);
    fill_in(c, token, pos, sp, rng_state ? *rng_state : 0, kFlagWriteLogits);
    if (c->step_exec && !c->params.trace) {
        if ((rc = count_launch(c)) != QWEN_OK) return rc;
        CU(cudaGraphLaunch(c->step_exec, c->stream));
    } else {
        CU(cudaMemcpyAsync(c->d_in, c->h_in, sizeof(StepIn), cudaMemcpyHostToDevice, c->stream));
        if ((rc = launch_decode(c)) != QWEN_OK) return rc;
        CU(cudaMemcpyAsync(c->h_out, c->d_out, sizeof(StepOut), cudaMemcpyDeviceToHost, c->stream));
    }
    CU(cudaStreamSynchronize(c->stream));
    c->last_k = (!sp || sp->temperature == 0.0f || sp->top_k == 1) ? 1 : sp->top_k;
    if ((rc = check_step(c)) != QWEN_OK) return rc;
    *next = c->h_out->out_token;
    if (rng_state) *rng_state = c->h_out->rng;
    c->cached = pos + 1;
    return QWEN_OK;
}

extern "C" int qwen_generate(qwen_t* c, int token, int pos, int n_steps, const qwen_sampling_t* sp, unsigned long long* rng_state,
                             int* tokens_out) {
    if (!c || !tokens_out) return fail(QWEN_E_ARG, "NULL argument");
    if (n_steps <= 0) return fail(QWEN_E_ARG, "n_steps must be positive");
    if (token < 0 || token >= VOCAB_SIZE) return fail(QWEN_E_ARG, "token out of range");
    if (pos < 0 || (long long)pos + n_steps > SEQ_LEN) return fail(QWEN_E_ARG, "pos + n_steps exceeds SEQ_LEN");
    if (pos > c->cached) return fail(QWEN_E_STATE, "pos skips uncached positions");
    int rc = check_sampling(sp);
    if (rc != QWEN_OK) return rc;
    if (!device_exact(sp)) return host_sampled_steps(c, token, pos, n_steps, sp, rng_state, tokens_out, nullptr);
    CU(cudaSetDevice(c->device));
    fill_in(c, token, pos, sp, rng_state ? *rng_state : 0, kFlagWriteLogits);
    CU(cudaMemcpyAsync(c->d_in, c->h_in, sizeof(StepIn), cudaMemcpyHostToDevice, c->stream));
    CU(cudaMemsetAsync(&c->d_out->n_done, 0, sizeof(int), c->stream));
    for (int i = 0; i < n_steps; i++)
        if ((rc = launch_decode(c)) != QWEN_OK) return rc;
    CU(cudaMemcpyAsync(c->h_tokens, c->tokens, (size_t)n_steps * sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaMemcpyAsync(c->h_out, c->d_out, sizeof(StepOut), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    c->last_k = (!sp || sp->temperature == 0.0f || sp->top_k == 1) ? 1 : sp->top_k;
    if ((rc = check_step(c)) != QWEN_OK) return rc;
    memcpy(tokens_out, c->h_tokens, (size_t)n_steps * sizeof(int));
    if (rng_state) *rng_state = c->h_out->rng;
    c->cached = pos + n_steps;
    return QWEN_OK;
}

extern "C" int qwen_generate_timed(qwen_t* c, int token, int pos, int n_steps, const qwen_sampling_t* sp,
                                   unsigned long long* rng_state, int* tokens_out, float* device_ms) {
    if (!c || !tokens_out || !device_ms) return fail(QWEN_E_ARG, "NULL argument");
    if (n_steps <= 0) return fail(QWEN_E_ARG, "n_steps must be positive");
    if (token < 0 || token >= VOCAB_SIZE) return fail(QWEN_E_ARG, "token out of range");
    if (pos < 0 || (long long)pos + n_steps > SEQ_LEN) return fail(QWEN_E_ARG, "pos + n_steps exceeds SEQ_LEN");
    if (pos > c->cached) return fail(QWEN_E_STATE, "pos skips uncached positions");
    int rc = check_sampling(sp);
    if (rc != QWEN_OK) return rc;
    if (!device_exact(sp)) return host_sampled_steps(c, token, pos, n_steps, sp, rng_state, tokens_out, device_ms);
    CU(cudaSetDevice(c->device));
    cudaEvent_t e0, e1;
    CU(cudaEventCreate(&e0));
    if (cudaEventCreate(&e1) != cudaSuccess) { cudaEventDestroy(e0); return fail(QWEN_E_CUDA, "event creation failed"); }
    fill_in(c, token, pos, sp, rng_state ? *rng_state : 0, 0);
    rc = QWEN_OK;
    if (cudaMemcpyAsync(c->d_in, c->h_in, sizeof(StepIn), cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        cudaMemsetAsync(&c->d_out->n_done, 0, sizeof(int), c->stream) != cudaSuccess ||
        cudaStreamSynchronize(c->stream) != cudaSuccess || cudaEventRecord(e0, c->stream) != cudaSuccess)
        rc = fail(QWEN_E_CUDA, "timed generate setup failed");
    for (int i = 0; i < n_steps && rc == QWEN_OK; i++) rc = launch_decode(c);
    if (rc == QWEN_OK && (cudaEventRecord(e1, c->stream) != cudaSuccess || cudaEventSynchronize(e1) != cudaSuccess))
        rc = fail(QWEN_E_CUDA, "timed generate failed");
    if (rc == QWEN_OK) {
        cudaEventElapsedTime(device_ms, e0, e1);
        if (cudaMemcpyAsync(c->h_tokens, c->tokens, (size_t)n_steps * sizeof(int), cudaMemcpyDeviceToHost, c->stream) != cudaSuccess ||
            cudaMemcpyAsync(c->h_out, c->d_out, sizeof(StepOut), cudaMemcpyDeviceToHost, c->stream) != cudaSuccess ||
            cudaStreamSynchronize(c->stream) != cudaSuccess)
            rc = fail(QWEN_E_CUDA, "timed generate readback failed");
    }
    cudaEventDestroy(e0); cudaEventDestroy(e1);
    if (rc != QWEN_OK) return rc;
    c->last_k = (!sp || sp->temperature == 0.0f || sp->top_k == 1) ? 1 : sp->top_k;
    if ((rc = check_step(c)) != QWEN_OK) return rc;
    memcpy(tokens_out, c->h_tokens, (size_t)n_steps * sizeof(int));
    if (rng_state) *rng_state = c->h_out->rng;
    c->cached = pos + n_steps;
    return QWEN_OK;
}

static int gemm_check(qwen_t* c);
static int attention_tc5(qwen_t* c, const uint16_t* kc_l, const uint16_t* vc_l, int pos0, int m, int rows, int vt_n, cudaStream_t st);
static int gemm_qkv_rope(const void* A, int lda, const DecodeParams& P, int l, const qb::tc::QkvOut& qo, int M, int m_valid, cudaStream_t st,
                         int parts);
namespace {
bool pair_gemm_enabled();
}
static int gemm_swiglu(const void* A, int lda, const uint16_t* wgu, uint16_t* Hs, int ld_hs, int M, int m_valid, cudaStream_t st, int parts);
struct BSeg { const void* B; int rows; };   // one weight matrix [rows][Kb] of a grouped GEMM
static int gemm_tc(const void* A, int lda, std::initializer_list<BSeg> segs, int ldb, void* C, int ldc, int M, int K, int Kb, bool c_fp32,
                   cudaStream_t st, int split_cols = 0, int* splits_used = nullptr, int m_valid = 0);

// Prompt positions [pos0, pos0 + m) in one pass (m <= pf::kMaxRows): every
// layer's projections as tcgen05 GEMMs over all rows, attention over the KV
// cache; fills the cache, computes no logits.  Tokens are in c->prompt.
static int gemm_prepare(int dev);

// The prompt pass's scratch (kMaxRows rows), allocated on first use.
static int pf_alloc(qwen_t* c) {
    using namespace qb::pf;
    if (c->pf_x) return QWEN_OK;
    TRY(dalloc(&c->pf_x, (size_t)kMaxRows * DIM));
    TRY(dalloc(&c->pf_y, (size_t)kMaxRows * 2 * HIDDEN_DIM));
    TRY(dalloc(&c->pf_q, (size_t)kMaxRows * Q_DIM));
    TRY(dalloc(&c->pf_as, (size_t)kMaxRows * 3 * HIDDEN_DIM));
    TRY(dalloc(&c->pf_hs, (size_t)kMaxRows * 3 * HIDDEN_DIM));
    TRY(dalloc(&c->pf_xn, (size_t)DIM));
    CU(cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(AttTcSmem)));
    CU(cudaFuncSetAttribute(attention_tc5_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)A5Layout::kSmem));
    TRY(dalloc(&c->vt, (size_t)N_KV_HEADS * HEAD_DIM * SEQ_LEN));
    CU(cudaMemset(c->vt, 0, (size_t)N_KV_HEADS * HEAD_DIM * SEQ_LEN * sizeof(uint16_t)));
    return gemm_prepare(c->device);
}

// What a pass reads and writes besides the handle's scratch buffers.
struct PassIO {
    const int* tokens;      // device; prompt mode: token of position p at tokens[p]; batch mode: row r's at tokens[r]
    uint16_t* kc;           // K and V caches (layer 0) of the sequence (prompt mode) or of row 0 (batch mode)
    uint16_t* vc;
    const int* pos_rows;    // NULL: rows are positions pos0 + r of one sequence; else row r is one position of sequence r
    size_t row_stride;      // batch mode: elements between consecutive rows' caches
    float* part;            // batch mode: attention partials, room for kMaxKeySplits ranges per (row, KV head)
};
constexpr int kMaxKeySplits = 16;

// *down_splits / *down_ld: how the last down projection left its output in
// pf_y (partial sums DIM columns apart, rows down_ld apart) for the caller's
// final residual add.
static int prefill_pass(qwen_t* c, int pos0, int m, int* down_splits = nullptr, const PassIO* io = nullptr, int* down_ld = nullptr) {
    using namespace qb::pf;
    constexpr int kLdAs = 3 * HIDDEN_DIM, kLdY = 2 * HIDDEN_DIM, kLdQKV = Q_DIM + 2 * KV_DIM;
    TRY(pf_alloc(c));
    const DecodeParams& P = c->params;
    cudaStream_t st = c->stream;
    // The GEMMs run on rows rounded up to 128; rows m .. rows-1 are padding: the
    // elementwise kernels skip them, the GEMMs do not store them, and whatever
    // they hold in the input buffers only reaches padding outputs (every output
    // row depends on its own input row alone).
    const int rows = (m + tc::kBM - 1) / tc::kBM * tc::kBM;
    const bool batch = io && io->pos_rows;
    const int* tok = io ? (batch ? io->tokens : io->tokens + pos0) : c->prompt + pos0;
    uint16_t* kc0 = io ? io->kc : c->kc;
    uint16_t* vc0 = io ? io->vc : c->vc;
    CU(launch_pdl(embed_kernel, dim3(rows), dim3(256), 0, st, P.embed, tok, m, rows, c->pf_x));
    int rc, sp_o = 1, sp_d = 1;   // K splits of the O and down GEMMs: partial sums side by side in pf_y
    // with few rows pf_y also has room for split-K partials of the q|k|v and
    // gate|up GEMMs (their row strides widened to hold up to 4 / 6 of them)
    const size_t ycap = (size_t)kMaxRows * kLdY;
    const int ld_qkv = kLdQKV * (int)std::max<size_t>(1, std::min<size_t>(8, ycap / ((size_t)rows * kLdQKV)));
    const int ld_gu = kLdY * (int)std::max<size_t>(1, std::min<size_t>(6, ycap / ((size_t)rows * kLdY)));
    const int ld_od = std::max(kLdY, DIM * (int)std::min<size_t>(24, ycap / ((size_t)rows * DIM)));   // O and down partials
    // QK-norm, RoPE, the K/V append and V's transposed copy in the q|k|v GEMM's
    // epilogue when that GEMM runs on SM pairs without splitting K (its 256 x
    // 256 tiles give more than half the pairs two tiles) and attention is the
    // tcgen05 kernel (the reader of the transposed copy); else qkv_post_kernel
    const bool fuse_qkv = !batch && c->att5 && c->qkv_epi && pair_gemm_enabled() && rows % (2 * tc::kBM) == 0 &&
                          2 * (kLdQKV / 256) * (rows / (2 * tc::kBM)) > c->nsm / 2;
    for (int l = 0; l < N_LAYERS; l++) {
        uint16_t* kc_l = kc0 + (size_t)l * kGroups * SEQ_LEN * HEAD_DIM;
        uint16_t* vc_l = vc0 + (size_t)l * kGroups * SEQ_LEN * HEAD_DIM;
        CU(launch_pdl(norm_split_kernel, dim3(m), dim3(256), 0, st, c->pf_x, (const float*)(l ? c->pf_y : nullptr), ld_od, sp_d, P.in_ln[l],
                      c->pf_as, kLdAs, m, c->pf_parts));
        int sp_q = 1, sp_gu = 1;
        if (fuse_qkv) {
            const qb::tc::QkvOut qo{c->pf_q, kc_l, vc_l, c->vt, P.qn[l], P.kn[l], (const float*)P.rope, pos0};
            if ((rc = gemm_qkv_rope(c->pf_as, kLdAs, P, l, qo, rows, m, st, c->pf_parts)) != QWEN_OK) return rc;
        } else {
            if ((rc = gemm_tc(c->pf_as, kLdAs, {{P.wq[l], Q_DIM}, {P.wk[l], KV_DIM}, {P.wv[l], KV_DIM}}, DIM, c->pf_y, ld_qkv, rows, c->pf_parts * DIM,
                              DIM, true, st, kLdQKV, &sp_q, m)) != QWEN_OK)
                return rc;
            CU(launch_pdl(qkv_post_kernel, dim3(m * 4), dim3(256), 0, st, (const float*)c->pf_y, ld_qkv, sp_q, kLdQKV, m, m, pos0, P.qn[l], P.kn[l],
                          (const float*)P.rope, c->pf_q, kc_l, vc_l, (const int*)(batch ? io->pos_rows : nullptr),
                          (size_t)(batch ? io->row_stride : 0)));
        }
        if (batch) {
            // key ranges per (row, KV head): enough blocks for two per SM
            const int S = std::max(1, std::min(kMaxKeySplits, (2 * c->nsm + m * N_KV_HEADS - 1) / (m * N_KV_HEADS)));
            CU(launch_pdl(attention_rows_kernel, dim3(m * N_KV_HEADS * S), dim3(kDecAttThreads), 0, st, (const float*)c->pf_q,
                          (const int*)io->pos_rows, (const uint16_t*)kc_l, (const uint16_t*)vc_l, io->row_stride, S, c->pf_as, kLdAs, io->part));
            if (S > 1)
                CU(launch_pdl(attention_combine_kernel, dim3(m * N_KV_HEADS), dim3(kDecAttThreads), 0, st, (const float*)io->part, S, c->pf_as,
                              kLdAs));
        } else if (c->att5) {
            if ((rc = attention_tc5(c, kc_l, vc_l, pos0, m, rows, fuse_qkv ? pos0 : pos0 + m, st)) != QWEN_OK) return rc;
        } else {
            attention_tc_kernel<<<rows / kAttBlock * N_KV_HEADS, kTcThreads, sizeof(AttTcSmem), st>>>(c->pf_q, pos0, kc_l, vc_l, c->pf_as,
                                                                                                       kLdAs);
        }
        if ((rc = gemm_tc(c->pf_as, kLdAs, {{c->wo_raw[l], DIM}}, Q_DIM, c->pf_y, ld_od, rows, c->pf_parts * Q_DIM, Q_DIM, true, st, DIM, &sp_o, m)) !=
            QWEN_OK)
            return rc;
        CU(launch_pdl(norm_split_kernel, dim3(m), dim3(256), 0, st, c->pf_x, (const float*)c->pf_y, ld_od, sp_o, P.post_ln[l], c->pf_as, kLdAs, m,
                      c->pf_parts));
        // gate|up + SwiGLU: fused into the GEMM epilogue when 128 x 256 tiles fill the GPU
        // without splitting K, else GEMM (split K when rows are few) + swiglu_split
        const bool fused = (2 * HIDDEN_DIM / 256) * (rows / tc::kBM) >= c->nsm;
        uint16_t* hs = fused ? c->pf_hs : c->pf_as;
        if (fused) {
            if ((rc = gemm_swiglu(c->pf_as, kLdAs, c->wgu + (size_t)l * 2 * HIDDEN_DIM * DIM, c->pf_hs, kLdAs, rows, m, st, c->pf_parts)) != QWEN_OK)
                return rc;
        } else {
            if ((rc = gemm_tc(c->pf_as, kLdAs, {{P.wg[l], HIDDEN_DIM}, {P.wu[l], HIDDEN_DIM}}, DIM, c->pf_y, ld_gu, rows, c->pf_parts * DIM, DIM, true,
                              st, kLdY, &sp_gu, m)) != QWEN_OK)
                return rc;
            CU(launch_pdl(swiglu_split_kernel, dim3((m * (HIDDEN_DIM / 4) + 255) / 256), dim3(256), 0, st, (const float*)c->pf_y, ld_gu, sp_gu, kLdY,
                          c->pf_as, kLdAs, m, c->pf_parts));
        }
        if ((rc = gemm_tc(hs, kLdAs, {{P.wd[l], DIM}}, HIDDEN_DIM, c->pf_y, ld_od, rows, c->pf_parts * HIDDEN_DIM, HIDDEN_DIM, true, st, DIM,
                          &sp_d, m)) != QWEN_OK)
            return rc;
    }
    CU(cudaGetLastError());
    if (down_splits) *down_splits = sp_d;
    if (down_ld) *down_ld = ld_od;
    return QWEN_OK;
}

// Prompts whose first n - 1 positions number at least this go through
// prefill_pass; shorter ones through one decode launch per position.
constexpr int kGemmPrefillMin = 64;

extern "C" int qwen_prefill(qwen_t* c, const int* tokens, int n, int pos0, float* logits_host) {
    if (!c || !tokens) return fail(QWEN_E_ARG, "NULL argument");
    if (n <= 0 || pos0 < 0 || (long long)pos0 + n > SEQ_LEN) return fail(QWEN_E_ARG, "prompt does not fit [0, SEQ_LEN)");
    if (pos0 > c->cached) return fail(QWEN_E_STATE, "pos0 skips uncached positions");
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= VOCAB_SIZE) return fail(QWEN_E_ARG, "prompt token out of range");
    CU(cudaSetDevice(c->device));
    CU(cudaMemcpyAsync(c->prompt + pos0, tokens, (size_t)n * sizeof(int), cudaMemcpyHostToDevice, c->stream));
    int rc;
    const bool full_vocab = c->params.lm_begin == 0 && c->params.lm_end == VOCAB_SIZE;
    if (n - 1 >= kGemmPrefillMin && c->gemm_prefill && full_vocab) {
        // every position in tensor-core passes; the logits of the last one from
        // its final residual: RMSNorm + an fp32-input LM-head GEMV
        int s = 0, m = 0, sp = 1, ld = 0;
        for (; s < n; s += m) {
            m = std::min(qb::pf::kMaxRows, n - s);
            if ((rc = prefill_pass(c, pos0 + s, m, &sp, nullptr, &ld)) != QWEN_OK) return rc;
        }
        const int last_row = m - 1;
        CU(launch_pdl(qb::pf::final_norm_row_kernel, dim3(1), dim3(256), 0, c->stream, (const float*)c->pf_x, (const float*)c->pf_y, ld, sp,
                      c->params.final_ln, last_row, c->pf_xn));
        CU(launch_pdl(qb::pf::lm_head_f32_kernel, dim3(c->nsm * 8), dim3(256), 0, c->stream, c->params.lm, (const float*)c->pf_xn, 0, (int)VOCAB_SIZE,
                      c->logits));
        CU(cudaGetLastError());
        if (logits_host) CU(cudaMemcpyAsync(logits_host, c->logits, (size_t)VOCAB_SIZE * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
        CU(cudaStreamSynchronize(c->stream));
        if ((rc = gemm_check(c)) != QWEN_OK) return rc;
        c->last_k = 0;   // no candidate list: the decode kernel did not run
        c->cached = pos0 + n;
        return QWEN_OK;
    }
    if (n - 1 >= kGemmPrefillMin && c->gemm_prefill) {   // vocabulary shard: the last position through the decode kernel
        for (int s = 0; s < n - 1; s += qb::pf::kMaxRows)
            if ((rc = prefill_pass(c, pos0 + s, std::min(qb::pf::kMaxRows, n - 1 - s))) != QWEN_OK) return rc;
    } else if (n > 1) {
        fill_in(c, 0, pos0, nullptr, 0, kFlagPromptToken | kFlagNoHead);
        CU(cudaMemcpyAsync(c->d_in, c->h_in, sizeof(StepIn), cudaMemcpyHostToDevice, c->stream));
        for (int i = 0; i < n - 1; i++)
            if ((rc = launch_decode(c)) != QWEN_OK) return rc;
    }
    // last prompt position with the LM head (logits of the prompt's end)
    CU(cudaStreamSynchronize(c->stream));
    fill_in(c, 0, pos0 + n - 1, nullptr, 0, kFlagPromptToken | kFlagWriteLogits);
    CU(cudaMemcpyAsync(c->d_in, c->h_in, sizeof(StepIn), cudaMemcpyHostToDevice, c->stream));
    if ((rc = launch_decode(c)) != QWEN_OK) return rc;
    if (logits_host) CU(cudaMemcpyAsync(logits_host, c->logits, (size_t)VOCAB_SIZE * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaMemcpyAsync(c->h_out, c->d_out, sizeof(StepOut), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    c->last_k = 1;
    if ((rc = gemm_check(c)) != QWEN_OK) return rc;
    if ((rc = check_step(c)) != QWEN_OK) return rc;
    c->cached = pos0 + n;
    return QWEN_OK;
}

// ---------------------------------------------------------------------------
// batched decode: B sequences per step, each in its own KV cache slot
// ---------------------------------------------------------------------------
constexpr int kMaxBatch = 128;
static size_t slot_elems() { return (size_t)N_LAYERS * kGroups * SEQ_LEN * HEAD_DIM; }

// Entries per row of one top-k level list: k survivors of each 512-entry group of the first level.
static int topk_scratch_ld(int n, int k) { return (n + qb::pf::kTopkGroup - 1) / qb::pf::kTopkGroup * k; }

// The k best of each of `rows` rows of fp32 logits (n columns, ld apart) into
// v / i (k per row, in column order), by topk_level_kernel levels until one
// group is left.  scratch: 4 x E words (two key lists, two id lists), E at
// least rows x topk_scratch_ld(n, k).
static cudaError_t launch_row_topk(const float* logits, int rows, int n, int ld, int k, uint32_t* scratch, size_t E, float* v, int* i,
                                   cudaStream_t st) {
    namespace pf = qb::pf;
    const int lds = topk_scratch_ld(n, k);
    uint32_t* key[2] = {scratch, scratch + E};
    int* id[2] = {reinterpret_cast<int*>(scratch + 2 * E), reinterpret_cast<int*>(scratch + 3 * E)};
    auto grid = [&](int m) {
        const int groups = (m + pf::kTopkGroup - 1) / pf::kTopkGroup;
        return dim3((unsigned)((groups + pf::kTopkWarps - 1) / pf::kTopkWarps), (unsigned)rows);
    };
    pf::topk_level_kernel<true><<<grid(n), 32 * pf::kTopkWarps, 0, st>>>(logits, nullptr, nullptr, ld, n, k, key[0], id[0], lds, v, i, n);
    int m = n, cur = 0;
    while (m > pf::kTopkGroup) {
        m = (m + pf::kTopkGroup - 1) / pf::kTopkGroup * k;
        pf::topk_level_kernel<false><<<grid(m), 32 * pf::kTopkWarps, 0, st>>>(nullptr, key[cur], id[cur], lds, m, k, key[cur ^ 1],
                                                                                id[cur ^ 1], lds, v, i, n);
        cur ^= 1;
    }
    return cudaGetLastError();
}

extern "C" int qwen_batch_init(qwen_t* c, int max_batch) {
    if (!c) return fail(QWEN_E_ARG, "NULL handle");
    if (max_batch < 1 || max_batch > kMaxBatch) return fail(QWEN_E_ARG, "max_batch must be in [1, 128]");
    if (c->b_max) return fail(QWEN_E_STATE, "batched decode already initialised on this handle");
    CU(cudaSetDevice(c->device));
    // an earlier call that failed part-way may have left some buffers: start clean
    for (void** p : {(void**)&c->bkc, (void**)&c->bvc, (void**)&c->b_tokens, (void**)&c->b_pos, (void**)&c->b_ci, (void**)&c->b_logits,
                     (void**)&c->b_cv, (void**)&c->b_part, (void**)&c->b_tk}) {
        if (*p) cudaFree(*p);
        *p = nullptr;
    }
    const size_t cache = (size_t)max_batch * slot_elems();
    const int rows = (max_batch + 127) / 128 * 128;
    if (cudaMalloc(&c->bkc, cache * sizeof(uint16_t)) != cudaSuccess || cudaMalloc(&c->bvc, cache * sizeof(uint16_t)) != cudaSuccess) {
        cudaGetLastError();
        if (c->bkc) cudaFree(c->bkc);
        c->bkc = nullptr;
        return fail(QWEN_E_CUDA, "cannot allocate " + std::to_string(max_batch) + " KV cache slots (" +
                                     std::to_string(2 * cache * sizeof(uint16_t) >> 20) + " MiB)");
    }
    TRY(dalloc(&c->b_tokens, (size_t)max_batch));
    TRY(dalloc(&c->b_pos, (size_t)max_batch));
    TRY(dalloc(&c->b_logits, (size_t)rows * VOCAB_SIZE));
    TRY(dalloc(&c->b_cv, (size_t)max_batch * kMaxCand));
    TRY(dalloc(&c->b_ci, (size_t)max_batch * kMaxCand));
    TRY(dalloc(&c->b_tk, 4 * (size_t)max_batch * topk_scratch_ld(VOCAB_SIZE, kMaxCand)));
    TRY(dalloc(&c->b_part, (size_t)max_batch * N_KV_HEADS * kMaxKeySplits * qb::pf::kPartFloats));
    // positions past a slot's length are read (and weighted zero) by the prompt pass's tiles: keep them finite
    CU(cudaMemsetAsync(c->bkc, 0, cache * sizeof(uint16_t), c->stream));
    CU(cudaMemsetAsync(c->bvc, 0, cache * sizeof(uint16_t), c->stream));
    CU(cudaStreamSynchronize(c->stream));
    TRY(pf_alloc(c));
    c->b_cached.assign(max_batch, 0);
    c->b_max = max_batch;
    return QWEN_OK;
}

extern "C" int qwen_batch_prefill(qwen_t* c, int slot, const int* tokens, int n, float* logits_host) {
    if (!c || !tokens) return fail(QWEN_E_ARG, "NULL argument");
    if (!c->b_max) return fail(QWEN_E_STATE, "qwen_batch_init first");
    if (slot < 0 || slot >= c->b_max) return fail(QWEN_E_ARG, "slot out of range");
    if (n <= 0 || n > SEQ_LEN) return fail(QWEN_E_ARG, "prompt does not fit [0, SEQ_LEN)");
    for (int i = 0; i < n; i++)
        if (tokens[i] < 0 || tokens[i] >= VOCAB_SIZE) return fail(QWEN_E_ARG, "prompt token out of range");
    CU(cudaSetDevice(c->device));
    CU(cudaMemcpyAsync(c->prompt, tokens, (size_t)n * sizeof(int), cudaMemcpyHostToDevice, c->stream));
    const PassIO io{c->prompt, c->bkc + (size_t)slot * slot_elems(), c->bvc + (size_t)slot * slot_elems(), nullptr, 0, nullptr};
    int rc, s = 0, m = 0, sp = 1, ld = 0;
    for (; s < n; s += m) {
        m = std::min(qb::pf::kMaxRows, n - s);
        if ((rc = prefill_pass(c, s, m, &sp, &io, &ld)) != QWEN_OK) return rc;
    }
    CU(launch_pdl(qb::pf::final_norm_row_kernel, dim3(1), dim3(256), 0, c->stream, (const float*)c->pf_x, (const float*)c->pf_y, ld, sp,
                  c->params.final_ln, m - 1, c->pf_xn));
    CU(launch_pdl(qb::pf::lm_head_f32_kernel, dim3(c->nsm * 8), dim3(256), 0, c->stream, c->params.lm, (const float*)c->pf_xn, 0, (int)VOCAB_SIZE,
                  c->logits));
    CU(cudaGetLastError());
    if (logits_host) CU(cudaMemcpyAsync(logits_host, c->logits, (size_t)VOCAB_SIZE * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    if ((rc = gemm_check(c)) != QWEN_OK) { c->b_cached[slot] = 0; return rc; }
    c->b_cached[slot] = n;
    return QWEN_OK;
}

extern "C" int qwen_batch_step(qwen_t* c, int batch, const int* tokens, const int* pos, const qwen_sampling_t* sp,
                               unsigned long long* rng_states, int* next) {
    if (!c || !tokens || !pos || !next) return fail(QWEN_E_ARG, "NULL argument");
    if (!c->b_max) return fail(QWEN_E_STATE, "qwen_batch_init first");
    if (batch < 1 || batch > c->b_max) return fail(QWEN_E_ARG, "batch out of [1, max_batch]");
    int rc = check_sampling(sp);
    if (rc != QWEN_OK) return rc;
    const bool greedy = is_greedy(sp);
    if (!greedy && !rng_states) return fail(QWEN_E_ARG, "sampling needs rng_states");
    const bool host_order = !device_exact(sp);   // draw over whole logits rows on the host (the reference's order)
    for (int r = 0; r < batch; r++) {
        if (tokens[r] < 0 || tokens[r] >= VOCAB_SIZE) return fail(QWEN_E_ARG, "token out of range");
        if (pos[r] < 0 || pos[r] >= SEQ_LEN) return fail(QWEN_E_ARG, "pos out of range [0, SEQ_LEN)");
        if (pos[r] > c->b_cached[r]) return fail(QWEN_E_STATE, "pos skips uncached positions of its slot");
    }
    const int K = greedy || host_order ? 1 : sp->top_k;
    const int rows = (batch + 127) / 128 * 128;
    constexpr int kLdAs = 3 * HIDDEN_DIM;
    CU(cudaSetDevice(c->device));
    CU(cudaMemcpyAsync(c->b_tokens, tokens, (size_t)batch * sizeof(int), cudaMemcpyHostToDevice, c->stream));
    CU(cudaMemcpyAsync(c->b_pos, pos, (size_t)batch * sizeof(int), cudaMemcpyHostToDevice, c->stream));
    // the step's device work: the pass over the batch rows, the final RMSNorm of
    // every row (split into three bf16 parts), the LM head as one GEMM, top-k
    // per row; captured once per (batch, k) as a CUDA graph and replayed
    auto body = [&]() -> int {
        const PassIO io{c->b_tokens, c->bkc, c->bvc, c->b_pos, slot_elems(), c->b_part};
        int sp_d = 1, ld_d = 0, r2;
        if ((r2 = prefill_pass(c, 0, batch, &sp_d, &io, &ld_d)) != QWEN_OK) return r2;
        CU(launch_pdl(qb::pf::norm_split_kernel, dim3(batch), dim3(256), 0, c->stream, c->pf_x, (const float*)c->pf_y, ld_d, sp_d,
                      c->params.final_ln, c->pf_as, kLdAs, batch, 3));
        if ((r2 = gemm_tc(c->pf_as, kLdAs, {{c->params.lm, VOCAB_SIZE}}, DIM, c->b_logits, VOCAB_SIZE, rows, 3 * DIM, DIM, true,
                          c->stream, 0, nullptr, batch)) != QWEN_OK)
            return r2;
        const size_t E = (size_t)c->b_max * topk_scratch_ld(VOCAB_SIZE, kMaxCand);
        CU(launch_row_topk(c->b_logits, batch, VOCAB_SIZE, VOCAB_SIZE, K, c->b_tk, E, c->b_cv, c->b_ci, c->stream));
        return QWEN_OK;
    };
    const int key = (batch << 8) | K;
    auto it = c->b_graphs.find(key);
    if (it == c->b_graphs.end() && !c->b_graph_off) {
        cudaGraph_t g = nullptr;
        cudaGraphExec_t ge = nullptr;
        if (cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
            const int brc = body();
            const bool ended = cudaStreamEndCapture(c->stream, &g) == cudaSuccess;
            if (brc == QWEN_OK && ended && g && cudaGraphInstantiate(&ge, g, 0) != cudaSuccess) ge = nullptr;
            if (g) cudaGraphDestroy(g);
        }
        if (ge) it = c->b_graphs.emplace(key, ge).first;
        else { c->b_graph_off = true; cudaGetLastError(); }
    }
    if (it != c->b_graphs.end()) CU(cudaGraphLaunch(it->second, c->stream));
    else if ((rc = body()) != QWEN_OK) return rc;
    std::vector<float> cv((size_t)batch * K);
    std::vector<int> ci((size_t)batch * K);
    std::vector<float> rows_host(host_order ? (size_t)batch * VOCAB_SIZE : 0);
    if (host_order)
        CU(cudaMemcpyAsync(rows_host.data(), c->b_logits, rows_host.size() * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaMemcpyAsync(cv.data(), c->b_cv, cv.size() * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaMemcpyAsync(ci.data(), c->b_ci, ci.size() * sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    if ((rc = gemm_check(c)) != QWEN_OK) {
        std::fill(c->b_cached.begin(), c->b_cached.end(), 0);
        return rc;
    }
    for (int r = 0; r < batch; r++) {
        if (greedy) next[r] = ci[r];
        else if (host_order) {
            if ((rc = qwen_sample_host(&rows_host[(size_t)r * VOCAB_SIZE], VOCAB_SIZE, sp, &rng_states[r], &next[r])) != QWEN_OK)
                return fail(rc, "host sampling failed");
        } else if ((rc = qwen_sample_candidates(&cv[(size_t)r * K], &ci[(size_t)r * K], K, sp, &rng_states[r], &next[r])) != QWEN_OK)
            return rc;
        c->b_cached[r] = pos[r] + 1;
    }
    return QWEN_OK;
}

extern "C" int qwen_batch_read_logits(qwen_t* c, int rows, float* logits_host) {
    if (!c || !logits_host) return fail(QWEN_E_ARG, "NULL argument");
    if (!c->b_max) return fail(QWEN_E_STATE, "qwen_batch_init first");
    if (rows < 1 || rows > c->b_max) return fail(QWEN_E_ARG, "rows out of [1, max_batch]");
    CU(cudaSetDevice(c->device));
    CU(cudaMemcpyAsync(logits_host, c->b_logits, (size_t)rows * VOCAB_SIZE * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    return QWEN_OK;
}

extern "C" int qwen_set_prefill_parts(qwen_t* c, int parts) {
    if (!c) return fail(QWEN_E_ARG, "NULL handle");
    if (parts < 1 || parts > 3) return fail(QWEN_E_ARG, "parts must be 1, 2 or 3");
    c->pf_parts = parts;
    for (auto& kv : c->b_graphs) cudaGraphExecDestroy(kv.second);   // captured batch steps hold the old K
    c->b_graphs.clear();
    return QWEN_OK;
}

extern "C" int qwen_set_prefill_attention(qwen_t* c, int kind) {
    if (!c) return fail(QWEN_E_ARG, "NULL handle");
    if (kind != 0 && kind != 1) return fail(QWEN_E_ARG, "kind must be 0 (mma.sync) or 1 (tcgen05)");
    c->att5 = kind;
    return QWEN_OK;
}

extern "C" int qwen_set_prefill_mode(qwen_t* c, int gemm) {
    if (!c) return fail(QWEN_E_ARG, "NULL handle");
    c->gemm_prefill = gemm != 0;
    return QWEN_OK;
}

extern "C" int qwen_read_logits(qwen_t* c, float* logits_host) {
    if (!c || !logits_host) return fail(QWEN_E_ARG, "NULL argument");
    CU(cudaSetDevice(c->device));
    const int n = c->params.lm_end - c->params.lm_begin;
    CU(cudaMemcpyAsync(logits_host, c->logits + c->params.lm_begin, (size_t)n * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    return n;
}

extern "C" int qwen_set_vocab_shard(qwen_t* c, int row_begin, int row_end) {
    if (!c) return fail(QWEN_E_ARG, "NULL handle");
    if (row_begin < 0 || row_end > VOCAB_SIZE || row_end - row_begin < c->nsm * kMaxCand / 16 || row_begin >= row_end)
        return fail(QWEN_E_ARG, "bad vocabulary shard");
    c->params.lm_begin = row_begin;
    c->params.lm_end = row_end;
    drop_step_graph(c);
    return QWEN_OK;
}

extern "C" int qwen_shard_topk(qwen_t* c, int k, float* values_host, int* ids_host) {
    if (!c || !values_host || !ids_host) return fail(QWEN_E_ARG, "NULL argument");
    if (k < 1 || k > c->last_k) return fail(QWEN_E_ARG, "k exceeds the candidates kept by the last step");
    CU(cudaSetDevice(c->device));
    CU(cudaMemcpyAsync(values_host, c->top_v, (size_t)k * sizeof(float), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaMemcpyAsync(ids_host, c->top_i, (size_t)k * sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    return QWEN_OK;
}

// ---- vocabulary-sharded head, device-resident (no host round trip per token) ----
extern "C" void* qwen_stream(qwen_t* c) { return c ? (void*)c->stream : nullptr; }

static int shard_k(const qwen_sampling_t* sp) { return is_greedy(sp) ? 1 : sp->top_k; }

extern "C" int qwen_shard_begin(qwen_t* c, int token, int pos, const qwen_sampling_t* sp, unsigned long long rng) {
    if (!c) return fail(QWEN_E_ARG, "NULL handle");
    if (token < 0 || token >= VOCAB_SIZE) return fail(QWEN_E_ARG, "token out of range");
    if (pos < 0 || pos >= SEQ_LEN) return fail(QWEN_E_ARG, "pos out of range [0, SEQ_LEN)");
    if (pos > c->cached) return fail(QWEN_E_STATE, "pos skips uncached positions");
    int rc = check_sampling(sp);
    if (rc != QWEN_OK) return rc;
    if (!device_exact(sp))
        return fail(QWEN_E_UNSUPPORTED, "the sharded head samples on the device: argmax, or top-p in (0, 1) with 1 <= top_k <= 64");
    CU(cudaSetDevice(c->device));
    fill_in(c, token, pos, sp, rng, kFlagCandidatesOnly);
    CU(cudaMemcpyAsync(c->d_in, c->h_in, sizeof(StepIn), cudaMemcpyHostToDevice, c->stream));
    CU(cudaMemsetAsync(&c->d_out->n_done, 0, sizeof(int), c->stream));
    c->shard_pos0 = pos;
    c->shard_steps = 0;
    c->last_k = shard_k(sp);
    return c->last_k;
}

extern "C" int qwen_shard_decode(qwen_t* c) {
    if (!c) return fail(QWEN_E_ARG, "NULL handle");
    if (c->shard_pos0 < 0) return fail(QWEN_E_STATE, "qwen_shard_begin first");
    if (c->shard_pos0 + c->shard_steps >= SEQ_LEN) return fail(QWEN_E_ARG, "position reaches SEQ_LEN");
    CU(cudaSetDevice(c->device));
    return launch_decode(c);
}

extern "C" int qwen_shard_candidates(qwen_t* c, float* values_dev, int* ids_dev) {
    if (!c || !values_dev || !ids_dev) return fail(QWEN_E_ARG, "NULL argument");
    CU(cudaSetDevice(c->device));
    CU(cudaMemcpyAsync(values_dev, c->top_v, (size_t)c->last_k * sizeof(float), cudaMemcpyDeviceToDevice, c->stream));
    CU(cudaMemcpyAsync(ids_dev, c->top_i, (size_t)c->last_k * sizeof(int), cudaMemcpyDeviceToDevice, c->stream));
    return QWEN_OK;
}

extern "C" int qwen_shard_merge(qwen_t* c, const float* values_dev, const int* ids_dev, int n_ranks, int stride) {
    if (!c || !values_dev || !ids_dev) return fail(QWEN_E_ARG, "NULL argument");
    if (n_ranks < 1 || n_ranks * c->last_k > 2 * kMergeThreads) return fail(QWEN_E_ARG, "n_ranks x k exceeds 512 candidates");
    if (stride < c->last_k) return fail(QWEN_E_ARG, "stride below k");
    CU(cudaSetDevice(c->device));
    shard_merge_kernel<<<1, kMergeThreads, 0, c->stream>>>(values_dev, ids_dev, n_ranks, c->last_k, stride, c->d_in, c->d_out, c->tokens,
                                                           SEQ_LEN);
    CU(cudaGetLastError());
    c->shard_steps++;
    return QWEN_OK;
}

extern "C" int qwen_shard_finish(qwen_t* c, int* tokens_host, int n, unsigned long long* rng_state) {
    if (!c) return fail(QWEN_E_ARG, "NULL handle");
    if (c->shard_pos0 < 0) return fail(QWEN_E_STATE, "qwen_shard_begin first");
    if (n < 0 || n > c->shard_steps) return fail(QWEN_E_ARG, "more tokens requested than steps merged");
    CU(cudaSetDevice(c->device));
    if (n) CU(cudaMemcpyAsync(c->h_tokens, c->tokens, (size_t)n * sizeof(int), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaMemcpyAsync(c->h_out, c->d_out, sizeof(StepOut), cudaMemcpyDeviceToHost, c->stream));
    CU(cudaStreamSynchronize(c->stream));
    const int pos0 = c->shard_pos0, steps = c->shard_steps;
    c->shard_pos0 = -1;
    int rc = check_step(c);
    if (rc != QWEN_OK) return rc;
    if (tokens_host && n) memcpy(tokens_host, c->h_tokens, (size_t)n * sizeof(int));
    if (rng_state) *rng_state = c->h_out->rng;
    c->cached = pos0 + steps;
    return QWEN_OK;
}

extern "C" int qwen_debug_capture(qwen_t* c, int enable) {
    // the residual stream and the projections of the last launch stay in the
    // exchange buffers; nothing extra to keep
    (void)enable;
    return c ? QWEN_OK : fail(QWEN_E_ARG, "NULL handle");
}

extern "C" int qwen_debug_read(qwen_t* c, float* resid, float* qkv) {
    if (!c) return fail(QWEN_E_ARG, "NULL handle");
    CU(cudaSetDevice(c->device));
    CU(cudaStreamSynchronize(c->stream));
    auto take = [&](const uint64_t* src, size_t n, float* dst) -> int {
        std::vector<uint64_t> w(n);
        CU(cudaMemcpy(w.data(), src, n * sizeof(uint64_t), cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < n; i++) { const uint32_t u = (uint32_t)w[i]; memcpy(&dst[i], &u, 4); }
        return QWEN_OK;
    };
    int rc = QWEN_OK;
    if (resid) rc = take(c->params.xw + DIM, (size_t)N_LAYERS * DIM, resid);       // residual after layer l = x_{l+1}
    if (rc == QWEN_OK && qkv) rc = take(c->params.qkvw, (size_t)N_LAYERS * 4096, qkv);
    return rc;
}

extern "C" int qwen_debug_inject_wait(qwen_t* c, unsigned long long wait_ns, int group) {
    if (!c) return fail(QWEN_E_ARG, "NULL handle");
    if (group < -1 || group >= kGroups) return fail(QWEN_E_ARG, "group must be -1 or a KV head index");
    if (wait_ns != 0 && wait_ns < 1000000ull) return fail(QWEN_E_ARG, "wait limit below 1 ms");
    c->params.wait_ns = wait_ns ? wait_ns : kWaitNs;
    c->params.debug_skip = group;
    drop_step_graph(c);
    return QWEN_OK;
}

extern "C" int qwen_trace_enable(qwen_t* c, int enable) {
    if (!c) return fail(QWEN_E_ARG, "NULL handle");
    CU(cudaSetDevice(c->device));
    const size_t n = (size_t)c->nsm * kTraceStride;
    if (enable && !c->params.trace) {
        CU(cudaMalloc(&c->params.trace, n * sizeof(unsigned long long)));
        CU(cudaMemset(c->params.trace, 0, n * sizeof(unsigned long long)));
    }
    if (!enable && c->params.trace) { CU(cudaFree(c->params.trace)); c->params.trace = nullptr; }
    drop_step_graph(c);
    return QWEN_OK;
}

extern "C" int qwen_trace_read(qwen_t* c, unsigned long long* out, int max_entries) {
    if (!c || !out) return fail(QWEN_E_ARG, "NULL argument");
    if (!c->params.trace) return fail(QWEN_E_STATE, "tracing not enabled");
    const int n = c->nsm * kTraceStride;
    if (max_entries < n) return fail(QWEN_E_ARG, "buffer too small");
    CU(cudaSetDevice(c->device));
    CU(cudaMemcpy(out, c->params.trace, (size_t)n * sizeof(unsigned long long), cudaMemcpyDeviceToHost));
    return n;
}

extern "C" int qwen_debug_chunk_counts(qwen_t* c, int* out, int max_ctas) {
    if (!c || !out) return fail(QWEN_E_ARG, "NULL argument");
    if (max_ctas < c->nsm) return fail(QWEN_E_ARG, "buffer too small");
    CU(cudaSetDevice(c->device));
    CU(cudaMemcpy(out, c->chunk_count, (size_t)2 * c->nsm * sizeof(int), cudaMemcpyDeviceToHost));
    return c->nsm;
}

// ---------------------------------------------------------------------------
// isolated GEMV
// ---------------------------------------------------------------------------
// Matrices up to this size take the direct-load kernel, larger ones the ring
// kernel (the LM head: one CTA per SM streaming a contiguous row range).
constexpr size_t kGemvDirectMaxBytes = (size_t)64 << 20;

// y = bf16(W x) on `stream`; err = the error word the ring kernel reports into.
static int gemv_launch(const void* W, const void* x, void* y, int n, int k, cudaStream_t stream, uint32_t* err, int dev) {
    int nsm = 0;
    CU(cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev));
    if ((size_t)n * (size_t)k * 2 <= kGemvDirectMaxBytes) {
        const int rows_cta = qb::gemv_direct_rows_cta(k), segs = qb::gemv_direct_segs(k);
        const int groups = (n + rows_cta - 1) / rows_cta;
        const int grid = std::min((groups + 1) / 2, nsm * 8);
        qb::gemv_direct_kernel<<<grid, rows_cta * segs * 32, 0, stream>>>((const uint16_t*)W, (const uint16_t*)x, (uint16_t*)y, n, k);
    } else {
        const int grid = n < nsm ? n : nsm;
        gemv_bf16_kernel<<<grid, kGemvThreads, kGemvSmemBytes, stream>>>((const uint16_t*)W, (const uint16_t*)x, (uint16_t*)y, n, k, err);
    }
    CU(cudaGetLastError());
    return QWEN_OK;
}

static int gemv_check_args(const void* W, const void* x, const void* y, int n, int k) {
    if (!W || !x || !y) return fail(QWEN_E_ARG, "NULL argument");
    if (n <= 0 || k <= 0 || k % 256 != 0 || k > 4096) return fail(QWEN_E_ARG, "k must be a positive multiple of 256, <= 4096, and n > 0");
    if (((uintptr_t)W | (uintptr_t)x) & 15) return fail(QWEN_E_ARG, "W and x must be 16-byte aligned");
    return QWEN_OK;
}

// Reads and clears an error word after `stream` has synchronised.
static int gemv_read_status(uint32_t* word, cudaStream_t stream, const char* who) {
    CU(cudaStreamSynchronize(stream));
    uint32_t e = 0;
    CU(cudaMemcpy(&e, word, sizeof(e), cudaMemcpyDeviceToHost));
    if (!e) return QWEN_OK;
    CU(cudaMemset(word, 0, sizeof(e)));
    return fail(QWEN_E_TIMEOUT, std::string(who) + ": a device wait expired (code " + std::to_string(e) + "); the output of a launch since "
                                "the last status query is invalid");
}

// The allocating variant's error word, one per device, allocated and cleared
// once under a lock.
static std::atomic<uint32_t*> g_gemv_err[64];
static std::mutex g_gemv_err_mu;

static int gemv_err_word(int dev, uint32_t** out) {
    uint32_t* w = g_gemv_err[dev].load();
    if (!w) {
        std::lock_guard<std::mutex> lk(g_gemv_err_mu);
        w = g_gemv_err[dev].load();
        if (!w) {
            CU(cudaFuncSetAttribute(gemv_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvSmemBytes));
            CU(cudaMalloc(&w, sizeof(uint32_t)));
            CU(cudaMemset(w, 0, sizeof(uint32_t)));
            g_gemv_err[dev].store(w);
        }
    }
    *out = w;
    return QWEN_OK;
}

extern "C" int qwen_gemv_bf16(const void* W, const void* x, void* y, int n, int k, void* stream) {
    int rc = gemv_check_args(W, x, y, n, k);
    if (rc != QWEN_OK) return rc;
    int dev = 0;
    CU(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(QWEN_E_ARG, "device index beyond 63");
    uint32_t* err = nullptr;
    if ((rc = gemv_err_word(dev, &err)) != QWEN_OK) return rc;
    return gemv_launch(W, x, y, n, k, (cudaStream_t)stream, err, dev);
}

extern "C" int qwen_gemv_bf16_status(void* stream) {
    int dev = 0;
    CU(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(QWEN_E_ARG, "device index beyond 63");
    uint32_t* err = g_gemv_err[dev].load();
    if (!err) { CU(cudaStreamSynchronize((cudaStream_t)stream)); return QWEN_OK; }   // no launch yet on this device
    return gemv_read_status(err, (cudaStream_t)stream, "qwen_gemv_bf16");
}

// ---------------------------------------------------------------------------
// tensor-core GEMM (tcgen05)
// ---------------------------------------------------------------------------
namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

// 2-D K-major bf16 tensor map: `rows` x `cols` (cols contiguous, rows ld
// elements apart), boxes of box_rows x 64 elements with the 128-byte swizzle
// the tcgen05 descriptors expect.
bool kmajor_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
    std::call_once(g_encode_once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess && q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    if (!g_encode) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)qb::tc::kBK, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

uint32_t* g_gemm_err[64] = {nullptr};
int g_nsm[64] = {0};

// Tensor maps by (base, rows, cols, ld, box rows): the weights and the prompt
// pass's buffers keep their addresses, so each map is encoded once (a pass
// issues ~10 maps per layer; encoding them every call made short passes
// host-bound).
struct MapKey {
    const void* base;
    uint64_t rows, cols, ld;
    uint32_t box;
    bool operator==(const MapKey& o) const { return base == o.base && rows == o.rows && cols == o.cols && ld == o.ld && box == o.box; }
};
struct MapKeyHash {
    size_t operator()(const MapKey& k) const {
        size_t h = std::hash<const void*>()(k.base);
        for (uint64_t v : {k.rows, k.cols, k.ld, (uint64_t)k.box}) h = h * 1000003u ^ std::hash<uint64_t>()(v);
        return h;
    }
};
std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;

bool cached_map(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows) {
    const MapKey key{base, rows, cols, ld, box_rows};
    std::lock_guard<std::mutex> lock(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) { *m = it->second; return true; }
    if (!kmajor_map(m, base, rows, cols, ld, box_rows)) return false;
    if (g_maps.size() > 4096) g_maps.clear();   // bound the cache (freed buffers' keys never hit again)
    g_maps.emplace(key, *m);
    return true;
}

// The single-CTA form, 128 x BN tiles; A holds P = K / (kb_b 64) parts side
// by side, all P loaded in one stage.
template <int BN, bool F32, int kEpi, int P>
int gemm_launch_p(const CUtensorMap& ma, const qb::tc::BMaps& bm, void* C, int ldc, int M, int K, int kb_b, int splits, int c_split_off,
                  int m_valid, int nsm, cudaStream_t st, uint32_t* err, int epi_parts, int a_rows) {
    static thread_local int attr_dev = -1;
    int dev = 0;
    CU(cudaGetDevice(&dev));
    if (attr_dev != dev) {
        CU(cudaFuncSetAttribute(qb::tc::gemm_bf16_tc_persistent<BN, F32, kEpi, P>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                qb::tc::Layout<BN, P>::kSmem));
        attr_dev = dev;
    }
    const int items = bm.end[2] * (M / qb::tc::kBM) * splits;
    CU(launch_pdl(qb::tc::gemm_bf16_tc_persistent<BN, F32, kEpi, P>, dim3(std::min(items, nsm)), dim3(qb::tc::kThreads),
                  (size_t)qb::tc::Layout<BN, P>::kSmem, st, ma, bm, C, ldc, K, kb_b, M / qb::tc::kBM, splits, c_split_off, m_valid, err, epi_parts,
                  a_rows));
    return QWEN_OK;
}
// a_rows: the height of ma's box (qb::tc::kBM, or fewer rows when M is one
// 128-row block of which only those are valid).
template <int BN, bool F32, int kEpi = 0>
int gemm_launch(const CUtensorMap& ma, const qb::tc::BMaps& bm, void* C, int ldc, int M, int K, int kb_b, int splits, int c_split_off,
                int m_valid, int nsm, cudaStream_t st, uint32_t* err, int epi_parts = 3, int a_rows = qb::tc::kBM) {
    switch (K / (kb_b * qb::tc::kBK)) {
        case 1: return gemm_launch_p<BN, F32, kEpi, 1>(ma, bm, C, ldc, M, K, kb_b, splits, c_split_off, m_valid, nsm, st, err, epi_parts, a_rows);
        case 2: return gemm_launch_p<BN, F32, kEpi, 2>(ma, bm, C, ldc, M, K, kb_b, splits, c_split_off, m_valid, nsm, st, err, epi_parts, a_rows);
        case 3: return gemm_launch_p<BN, F32, kEpi, 3>(ma, bm, C, ldc, M, K, kb_b, splits, c_split_off, m_valid, nsm, st, err, epi_parts, a_rows);
        default: return fail(QWEN_E_ARG, "the GEMM takes one to three activation parts");
    }
}
template <int BN, bool F32, int kEpi>
cudaError_t single_smem_attrs() {
    cudaError_t e = cudaFuncSetAttribute(qb::tc::gemm_bf16_tc_persistent<BN, F32, kEpi, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         qb::tc::Layout<BN, 1>::kSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(qb::tc::gemm_bf16_tc_persistent<BN, F32, kEpi, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 qb::tc::Layout<BN, 2>::kSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(qb::tc::gemm_bf16_tc_persistent<BN, F32, kEpi, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 qb::tc::Layout<BN, 3>::kSmem);
    return e;
}

// The pair (2-SM) form: clusters of two CTAs, 256 x BN tiles; A holds P =
// K / (kb_b 64) parts side by side, all P loaded in one stage.
template <int BN, bool F32, int kEpi, int P>
int gemm_launch_pair_p(const CUtensorMap& ma, const qb::tc::BMaps& bm, void* C, int ldc, int M, int K, int kb_b, int splits, int c_split_off,
                       int m_valid, int nsm, cudaStream_t st, uint32_t* err, int epi_parts, const qb::tc::QkvOut& qo) {
    static thread_local int attr_dev = -1;
    int dev = 0;
    CU(cudaGetDevice(&dev));
    if (attr_dev != dev) {
        CU(cudaFuncSetAttribute(qb::tc::gemm_bf16_tc_pair<BN, F32, kEpi, P>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                qb::tc::PairLayout<BN, P>::kSmem));
        attr_dev = dev;
    }
    const int items = bm.end[2] * (M / (2 * qb::tc::kBM)) * splits;
    const int pairs = std::min(items, nsm / 2);
    CU(launch_pdl(qb::tc::gemm_bf16_tc_pair<BN, F32, kEpi, P>, dim3(2 * pairs), dim3(qb::tc::kPairThreads), (size_t)qb::tc::PairLayout<BN, P>::kSmem,
                  st, ma, bm, C, ldc, K, kb_b, M / (2 * qb::tc::kBM), splits, c_split_off, m_valid, err, epi_parts, qo));
    return QWEN_OK;
}
template <int BN, bool F32, int kEpi = 0>
int gemm_launch_pair(const CUtensorMap& ma, const qb::tc::BMaps& bm, void* C, int ldc, int M, int K, int kb_b, int splits, int c_split_off,
                     int m_valid, int nsm, cudaStream_t st, uint32_t* err, int epi_parts = 3, const qb::tc::QkvOut& qo = qb::tc::QkvOut{}) {
    switch (K / (kb_b * qb::tc::kBK)) {
        case 1: return gemm_launch_pair_p<BN, F32, kEpi, 1>(ma, bm, C, ldc, M, K, kb_b, splits, c_split_off, m_valid, nsm, st, err, epi_parts, qo);
        case 2: return gemm_launch_pair_p<BN, F32, kEpi, 2>(ma, bm, C, ldc, M, K, kb_b, splits, c_split_off, m_valid, nsm, st, err, epi_parts, qo);
        case 3: return gemm_launch_pair_p<BN, F32, kEpi, 3>(ma, bm, C, ldc, M, K, kb_b, splits, c_split_off, m_valid, nsm, st, err, epi_parts, qo);
        default: return fail(QWEN_E_ARG, "the pair GEMM takes one to three activation parts");
    }
}
template <int BN, bool F32, int kEpi>
cudaError_t pair_smem_attrs() {
    cudaError_t e = cudaFuncSetAttribute(qb::tc::gemm_bf16_tc_pair<BN, F32, kEpi, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         qb::tc::PairLayout<BN, 1>::kSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(qb::tc::gemm_bf16_tc_pair<BN, F32, kEpi, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 qb::tc::PairLayout<BN, 2>::kSmem);
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(qb::tc::gemm_bf16_tc_pair<BN, F32, kEpi, 3>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 qb::tc::PairLayout<BN, 3>::kSmem);
    return e;
}

// Whether 256-row GEMMs run in the pair form (QWEN_B200_GEMM_PAIR=0 keeps every
// GEMM on single-CTA tiles).
bool pair_gemm_enabled() {
    static const bool on = [] {
        const char* e = getenv("QWEN_B200_GEMM_PAIR");
        return !(e && strcmp(e, "0") == 0);
    }();
    return on;
}
}  // namespace

// Device-side set-up of the GEMM on `dev` (its error word, the kernels'
// shared-memory limits), so that later launches allocate and configure
// nothing (they can then be captured into a CUDA graph).
static int gemm_prepare(int dev) {
    if (dev < 0 || dev >= 64) return fail(QWEN_E_UNSUPPORTED, "device index >= 64");
    static std::atomic<bool> done[64];
    if (done[dev].load(std::memory_order_acquire)) return QWEN_OK;
    if (!g_gemm_err[dev]) {
        CU(cudaMalloc(&g_gemm_err[dev], sizeof(uint32_t)));
        CU(cudaMemset(g_gemm_err[dev], 0, sizeof(uint32_t)));
    }
    if (!g_nsm[dev]) CU(cudaDeviceGetAttribute(&g_nsm[dev], cudaDevAttrMultiProcessorCount, dev));
    CU((single_smem_attrs<256, true, 0>()));
    CU((single_smem_attrs<256, false, 0>()));
    CU((single_smem_attrs<128, true, 0>()));
    CU((single_smem_attrs<128, false, 0>()));
    CU((single_smem_attrs<256, false, 1>()));
    CU((pair_smem_attrs<256, true, 0>()));
    CU((pair_smem_attrs<256, false, 0>()));
    CU((pair_smem_attrs<256, false, 1>()));
    CU((pair_smem_attrs<256, true, 2>()));
    done[dev].store(true, std::memory_order_release);
    return QWEN_OK;
}

// The gate|up projection with SwiGLU in the epilogue: A [M][parts DIM] (bf16
// parts) against the interleaved gate|up weights wgu [2 HIDDEN_DIM][DIM];
// writes h = silu(gate) * up as `parts` bf16 parts into Hs (rows ld_hs apart,
// parts HIDDEN_DIM apart), the parts the down projection reads.  Rows
// m_valid .. M-1 are not written.
static int gemm_swiglu(const void* A, int lda, const uint16_t* wgu, uint16_t* Hs, int ld_hs, int M, int m_valid, cudaStream_t st, int parts) {
    int dev = 0;
    CU(cudaGetDevice(&dev));
    if (dev >= 64) return fail(QWEN_E_UNSUPPORTED, "device index >= 64");
    const int rc = gemm_prepare(dev);
    if (rc != QWEN_OK) return rc;
    CUtensorMap ma;
    qb::tc::BMaps bm;
    const bool pair = pair_gemm_enabled() && M % (2 * qb::tc::kBM) == 0;
    if (!cached_map(&ma, A, (uint64_t)M, (uint64_t)(3 * DIM), (uint64_t)lda, qb::tc::kBM) ||
        !cached_map(&bm.map[0], wgu, (uint64_t)(2 * HIDDEN_DIM), (uint64_t)DIM, (uint64_t)DIM, pair ? 128 : 256))
        return fail(QWEN_E_CUDA, "cuTensorMapEncodeTiled failed");
    bm.map[1] = bm.map[2] = bm.map[0];
    bm.end[0] = bm.end[1] = bm.end[2] = 2 * HIDDEN_DIM / 256;
    if (pair)
        return gemm_launch_pair<256, false, 1>(ma, bm, Hs, ld_hs, M, parts * DIM, DIM / qb::tc::kBK, 1, 0, m_valid > 0 ? m_valid : M, g_nsm[dev],
                                               st, g_gemm_err[dev], parts);
    return gemm_launch<256, false, 1>(ma, bm, Hs, ld_hs, M, parts * DIM, DIM / qb::tc::kBK, 1, 0, m_valid > 0 ? m_valid : M, g_nsm[dev], st,
                                      g_gemm_err[dev], parts);
}

// The q|k|v projection of the prompt rows with QK-norm, RoPE, the K/V cache
// append and the transposed copy of V in its epilogue (QkvOut): A [M][parts
// DIM] (bf16 parts) against wq | wk | wv; rows m_valid .. M-1 are padding.
// Pair form only (M a multiple of 256), K not split.
static int gemm_qkv_rope(const void* A, int lda, const DecodeParams& P, int l, const qb::tc::QkvOut& qo, int M, int m_valid, cudaStream_t st,
                         int parts) {
    int dev = 0;
    CU(cudaGetDevice(&dev));
    if (dev >= 64) return fail(QWEN_E_UNSUPPORTED, "device index >= 64");
    const int rc = gemm_prepare(dev);
    if (rc != QWEN_OK) return rc;
    if (M % (2 * qb::tc::kBM)) return fail(QWEN_E_ARG, "the q|k|v epilogue runs on 256-row blocks");
    CUtensorMap ma;
    qb::tc::BMaps bm;
    if (!cached_map(&ma, A, (uint64_t)M, (uint64_t)(parts * DIM), (uint64_t)lda, qb::tc::kBM) ||
        !cached_map(&bm.map[0], P.wq[l], (uint64_t)Q_DIM, (uint64_t)DIM, (uint64_t)DIM, 128) ||
        !cached_map(&bm.map[1], P.wk[l], (uint64_t)KV_DIM, (uint64_t)DIM, (uint64_t)DIM, 128) ||
        !cached_map(&bm.map[2], P.wv[l], (uint64_t)KV_DIM, (uint64_t)DIM, (uint64_t)DIM, 128))
        return fail(QWEN_E_CUDA, "cuTensorMapEncodeTiled failed");
    bm.end[0] = Q_DIM / 256;
    bm.end[1] = bm.end[0] + KV_DIM / 256;
    bm.end[2] = bm.end[1] + KV_DIM / 256;
    return gemm_launch_pair<256, true, 2>(ma, bm, nullptr, 0, M, parts * DIM, DIM / qb::tc::kBK, 1, 0, m_valid > 0 ? m_valid : M, g_nsm[dev], st,
                                          g_gemm_err[dev], parts, qo);
}

// The prompt pass's causal attention on tcgen05 (attention_tc5.cuh): the
// layer's V for positions [0, vt_n) transposed into c->vt (positions vt_n ..
// pos0 + m - 1 are there already: the q|k|v epilogue wrote them), then one CTA
// per (64 rows, KV head).  Its error word is the GEMMs' (checked after the pass).
static int attention_tc5(qwen_t* c, const uint16_t* kc_l, const uint16_t* vc_l, int pos0, int m, int rows, int vt_n, cudaStream_t st) {
    using namespace qb::pf;
    const int dev = c->device;
    if (vt_n > 0) CU(launch_pdl(transpose_v_kernel, dim3((vt_n + 63) / 64, 2, N_KV_HEADS), dim3(64, 8), 0, st, vc_l, c->vt, vt_n));
    CUtensorMap mk, mv;
    if (!cached_map(&mk, kc_l, (uint64_t)N_KV_HEADS * SEQ_LEN, HEAD_DIM, HEAD_DIM, kA5Keys) ||
        !cached_map(&mv, c->vt, (uint64_t)N_KV_HEADS * HEAD_DIM, SEQ_LEN, SEQ_LEN, HEAD_DIM))
        return fail(QWEN_E_CUDA, "cuTensorMapEncodeTiled failed");
    CU(launch_pdl(attention_tc5_kernel, dim3(rows / kAttBlock * N_KV_HEADS), dim3(kA5Threads), (size_t)A5Layout::kSmem, st, mk, mv,
                  (const float*)c->pf_q, pos0, c->pf_as, 3 * HIDDEN_DIM, c->pf_parts, g_gemm_err[dev]));
    return QWEN_OK;
}

// C[M][N] (rows ldc apart) = A[M][K] (rows lda apart) . (B[N][Kb] repeated
// K / Kb times along K)^T, where B is the segments stacked along N (each
// [rows][Kb], rows ldb apart; at most three) and N their total rows.  One
// persistent launch; 128 x 256 tiles when they fill every SM, else 128 x 128.
// Rows m_valid .. M-1 (when 0 < m_valid < M) are padding: their results are
// not stored.  With split_cols > 0 the caller accepts K split s ways when 128 x 256 tiles
// would leave SMs idle (s the largest divisor of the K steps that keeps the
// work items within the SM count and the partials within ldc): partial sum i
// lands at columns i * split_cols + [0, N) and *splits_used = s, for the
// caller to add in order.
static int gemm_tc(const void* A, int lda, std::initializer_list<BSeg> segs, int ldb, void* C, int ldc, int M, int K, int Kb, bool c_fp32,
                   cudaStream_t st, int split_cols, int* splits_used, int m_valid) {
    if (!A || !C || segs.size() < 1 || segs.size() > 3) return fail(QWEN_E_ARG, "NULL argument or bad segment count");
    int N = 0;
    bool all256 = true;
    uintptr_t align = (uintptr_t)A | (uintptr_t)C;
    for (const BSeg& sg : segs) {
        if (!sg.B || sg.rows <= 0 || sg.rows % 128) return fail(QWEN_E_ARG, "N must be a multiple of 128");
        N += sg.rows;
        all256 = all256 && sg.rows % 256 == 0;
        align |= (uintptr_t)sg.B;
    }
    if (M <= 0 || K <= 0 || Kb <= 0 || M % qb::tc::kBM || K % qb::tc::kBK || Kb % qb::tc::kBK || K % Kb)
        return fail(QWEN_E_ARG, "M must be a multiple of 128, N of 128, K of 64");
    if (align & 15) return fail(QWEN_E_ARG, "A, B and C must be 16-byte aligned");
    if (lda < K || ldb < Kb || ldc < N || lda % 8 || ldb % 8 || ldc % 8) return fail(QWEN_E_ARG, "bad leading dimension");
    int dev = 0;
    CU(cudaGetDevice(&dev));
    if (dev >= 64) return fail(QWEN_E_UNSUPPORTED, "device index >= 64");
    if (!g_nsm[dev]) CU(cudaDeviceGetAttribute(&g_nsm[dev], cudaDevAttrMultiProcessorCount, dev));
    const int nsm = g_nsm[dev];
    if (!g_gemm_err[dev]) {
        CU(cudaMalloc(&g_gemm_err[dev], sizeof(uint32_t)));
        CU(cudaMemset(g_gemm_err[dev], 0, sizeof(uint32_t)));
    }
    // pair form (256 x 256 tiles on two SMs) for 256-row multiples whose tiles
    // (or K splits of them) give most of the SM pairs work
    if (K / Kb > 3) return fail(QWEN_E_ARG, "K must be one to three times B's K extent");
    const bool pair = pair_gemm_enabled() && all256 && M % (2 * qb::tc::kBM) == 0;
    const int tiles256 = (N / 256) * (M / qb::tc::kBM) / (pair ? 2 : 1);
    const int slots = pair ? nsm / 2 : nsm;
    int splits = 1;
    if (split_cols >= N && all256 && 2 * tiles256 <= slots)
        for (int s = 2; s * tiles256 <= slots && (s - 1) * split_cols + N <= ldc; s++)
            if ((Kb / qb::tc::kBK) % s == 0) splits = s;   // the largest that divides the K steps (each step covers every part)
    if (splits_used) *splits_used = splits;
    const int bn = all256 && (pair || splits > 1 || tiles256 >= nsm) ? 256 : 128;
    CUtensorMap ma;
    qb::tc::BMaps bm;
    const int mv = m_valid > 0 && m_valid < M ? m_valid : M;
    // one 128-row block with few valid rows (a batched decode step): A boxes of only
    // those rows (rounded up to 8), so the padding rows do not cross from L2
    const int a_rows = !pair && M == qb::tc::kBM ? (mv + 7) / 8 * 8 : qb::tc::kBM;
    if (!cached_map(&ma, A, (uint64_t)M, (uint64_t)K, (uint64_t)lda, (uint32_t)a_rows)) return fail(QWEN_E_CUDA, "cuTensorMapEncodeTiled failed");
    int s = 0, end = 0;
    for (const BSeg& sg : segs) {
        if (!cached_map(&bm.map[s], sg.B, (uint64_t)sg.rows, (uint64_t)Kb, (uint64_t)ldb, (uint32_t)(pair ? bn / 2 : bn)))
            return fail(QWEN_E_CUDA, "cuTensorMapEncodeTiled failed");
        end += sg.rows / bn;
        bm.end[s++] = end;
    }
    for (; s < 3; s++) { bm.map[s] = bm.map[0]; bm.end[s] = end; }
    const int kb_b = Kb / qb::tc::kBK;
    const int so = splits > 1 ? split_cols : 0;
    if (pair) return c_fp32 ? gemm_launch_pair<256, true>(ma, bm, C, ldc, M, K, kb_b, splits, so, mv, nsm, st, g_gemm_err[dev])
                            : gemm_launch_pair<256, false>(ma, bm, C, ldc, M, K, kb_b, splits, so, mv, nsm, st, g_gemm_err[dev]);
    if (bn == 256) return c_fp32 ? gemm_launch<256, true>(ma, bm, C, ldc, M, K, kb_b, splits, so, mv, nsm, st, g_gemm_err[dev], 3, a_rows)
                                 : gemm_launch<256, false>(ma, bm, C, ldc, M, K, kb_b, splits, so, mv, nsm, st, g_gemm_err[dev], 3, a_rows);
    return c_fp32 ? gemm_launch<128, true>(ma, bm, C, ldc, M, K, kb_b, splits, so, mv, nsm, st, g_gemm_err[dev], 3, a_rows)
                  : gemm_launch<128, false>(ma, bm, C, ldc, M, K, kb_b, splits, so, mv, nsm, st, g_gemm_err[dev], 3, a_rows);
}

// The GEMM kernel's error word for the handle's device (a bounded wait ran out
// in some launch since the last check): reported as QWEN_E_TIMEOUT, the KV cache
// invalidated; cleared.  Call after the stream has drained.
static int gemm_check(qwen_t* c) {
    uint32_t* e = c->device < 64 ? g_gemm_err[c->device] : nullptr;
    if (!e) return QWEN_OK;
    uint32_t h = 0;
    CU(cudaMemcpy(&h, e, sizeof(h), cudaMemcpyDeviceToHost));
    if (!h) return QWEN_OK;
    CU(cudaMemset(e, 0, sizeof(uint32_t)));
    c->cached = 0;
    return fail(QWEN_E_TIMEOUT, "tensor-core GEMM wait expired (code " + std::to_string(h) + "); KV cache invalidated");
}

extern "C" int qwen_gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, int c_fp32, void* stream) {
    return gemm_tc(A, K, {{B, N}}, K, C, N, M, K, K, c_fp32 != 0, (cudaStream_t)stream);
}

extern "C" int qwen_row_topk(const float* logits, int rows, int n, int ld, int k, float* values, int* ids, void* stream) {
    if (!logits || !values || !ids) return fail(QWEN_E_ARG, "NULL argument");
    if (rows < 1 || rows > 65535 || n < 1 || ld < n || k < 1 || k > kMaxCand) return fail(QWEN_E_ARG, "rows, n, ld or k out of range");
    const size_t E = (size_t)rows * topk_scratch_ld(n, k);
    uint32_t* scratch = nullptr;
    CU(cudaMalloc(&scratch, 4 * E * sizeof(uint32_t)));
    const cudaError_t e = launch_row_topk(logits, rows, n, ld, k, scratch, E, values, ids, (cudaStream_t)stream);
    const cudaError_t e2 = cudaStreamSynchronize((cudaStream_t)stream);
    cudaFree(scratch);
    CU(e);
    CU(e2);
    return QWEN_OK;
}

// ---------------------------------------------------------------------------
// isolated GEMV without allocation
// ---------------------------------------------------------------------------
// qwen_gemv_bf16 obtains its device scratch (the ring kernel's error word)
// with cudaMalloc on its first call on each device.  Some callers cannot allow
// that: code that runs while a stream is being captured, or inside a framework
// whose caching allocator already holds the device's memory.  This variant
// keeps the scratch in a file-scope device array instead.  Host code must not
// pass the array's name to a kernel (on the host it is only a stand-in for the
// symbol); the device address comes from cudaGetSymbolAddress, once per
// device, on the first call made with that device current.  The word starts
// at zero (static initialisation) and is cleared by
// qwen_gemv_bf16_static_status, which reads it.
constexpr int kGemvStaticScratchWords = 64;   // 256 bytes per device; the GEMV uses word 0
static __device__ __align__(256) uint32_t g_gemv_static_scratch[kGemvStaticScratchWords];
static std::atomic<uint32_t*> g_gemv_static_ptr[64];
static std::mutex g_gemv_static_mu;

static int gemv_static_word(int dev, uint32_t** out) {
    uint32_t* scratch = g_gemv_static_ptr[dev].load();
    if (!scratch) {   // set-up, once per device, with that device current; allocates nothing
        std::lock_guard<std::mutex> lk(g_gemv_static_mu);
        scratch = g_gemv_static_ptr[dev].load();
        if (!scratch) {
            void* p = nullptr;
            CU(cudaGetSymbolAddress(&p, g_gemv_static_scratch));
            CU(cudaFuncSetAttribute(gemv_bf16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemvSmemBytes));
            scratch = (uint32_t*)p;
            g_gemv_static_ptr[dev].store(scratch);
        }
    }
    *out = scratch;
    return QWEN_OK;
}

extern "C" int qwen_gemv_bf16_static(const void* W, const void* x, void* y, int n, int k, void* stream) {
    int rc = gemv_check_args(W, x, y, n, k);
    if (rc != QWEN_OK) return fail(rc, std::string("qwen_gemv_bf16_static serves k a positive multiple of 256, at most 4096, and n > 0 "
                                                   "(16-byte aligned W and x): ") + qwen_last_error());
    int dev = 0;
    CU(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(QWEN_E_ARG, "device index beyond 63");
    uint32_t* scratch = nullptr;
    if ((rc = gemv_static_word(dev, &scratch)) != QWEN_OK) return rc;
    return gemv_launch(W, x, y, n, k, (cudaStream_t)stream, scratch, dev);
}

extern "C" int qwen_gemv_bf16_static_status(void* stream) {
    int dev = 0;
    CU(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(QWEN_E_ARG, "device index beyond 63");
    uint32_t* scratch = g_gemv_static_ptr[dev].load();
    if (!scratch) { CU(cudaStreamSynchronize((cudaStream_t)stream)); return QWEN_OK; }
    return gemv_read_status(scratch, (cudaStream_t)stream, "qwen_gemv_bf16_static");
}
