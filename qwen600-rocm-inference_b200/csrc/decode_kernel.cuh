// decode_kernel.cuh — one batch-1 decode position of Qwen3-0.6B as ONE
// persistent cooperative kernel (one CTA per SM).
//
// Replaces the reference's per-token chain of ~450 launches
// (qwen_model.cuh:772-851: rmsnorm_gpu, 7 cuBLAS GEMVs per layer,
// qk_norm_fused_gpu, rope_gpu_naive, attention_gpu with a device sync,
// swiglu_gpu, the LM head and the bf16->fp32 conversion) and the host sampler
// (sampler.h:120-175) for the device-sampling entry points.
//
// Structure.  Every CTA owns a fixed slice of every weight matrix.  A producer
// warp streams the CTA's slices, in consumption order, through a ring of
// kSlots x 32 KB shared-memory slots with 1-D bulk async copies (TMA engine,
// mbarrier completion, L2 evict-first).  The stream never waits on
// activations, so weights for the next stages are already on chip while a
// stage waits for its inputs.  Sixteen consumer warps compute from the slots.
// Stages hand activations to each other through small fp32 buffers in global
// memory (L2) and gpu-scope acquire/release counters:
//
//   per layer l (the 8 KV heads define 8 CTA groups of ~G/8 CTAs):
//   QKV   group g: RMSNorm(x) (input_layernorm) -> its rows of the group's
//         512 projection rows (q heads 2g,2g+1; k, v head g) -> qkv[l]
//   ATT   group g: QK-norm + RoPE of q/k, bf16 K/V append at pos (by the CTA
//         owning pos), split-K attention over its share of positions
//         (online-softmax partial m, l, acc for both q heads)
//   OPROJ group g: combine the group's partials -> o (256 values) ->
//         its rows of Wo[:, 256g:256g+256] (packed contiguous) -> ybuf[l][g]
//   MLP   all CTAs: x_mid = x + sum_g ybuf[l][g]; RMSNorm (post-attn) ->
//         its gate and up rows -> SwiGLU -> its rows of Wd^T (packed) ->
//         fp32 red.add of its 1024-wide partial into acc[l] (CTA 0 adds x_mid)
//   HEAD  all CTAs: final RMSNorm -> its LM-head rows -> fp32 logits and a
//         local top-K; the last CTA to finish merges the candidates and
//         samples (argmax, or temperature / top-k / top-p with xorshift64*).
//
// Numerics: weights and the KV cache are bf16; every activation, the residual
// stream and all accumulations are fp32.  The down-projection partial sums
// meet in fp32 atomics, so the summation order of that one reduction varies
// between runs (round-off level, ~1e-7 relative).
//
// Every wait is bounded (kWaitNs): on expiry the kernel records an error in
// StepOut.err, stops waiting on other CTAs, still drains its own copies, and
// returns; the host then resets the counters.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "../host/config.h"

namespace qb {

constexpr int kNCW = 16;                    // consumer warps
constexpr int kNCT = kNCW * 32;             // consumer threads
constexpr int kThreads = kNCT + 32;         // + one producer warp
constexpr int kSlots = 6;
constexpr int kSlotBytes = 32768;
constexpr int kGroups = N_KV_HEADS;         // one CTA group per KV head
constexpr int kMaxGS = 32;                  // max CTAs per group
constexpr int kMinGS = 8;                   // min CTAs per group (grid >= 64)
constexpr int kMaxCand = 64;                // device top-k limit
constexpr int kHeadPart = 4 + HEAD_DIM;     // m, l, pad, pad, acc[128]
constexpr int kPartStride = 2 * kHeadPart;  // both q heads of a group
constexpr int kScoreCap = SEQ_LEN / kMinGS; // positions per CTA at most
constexpr int kMaxLocalRows = 1280;         // LM-head rows per CTA at most
constexpr int kMaxMlpRows = 64;             // hidden rows per CTA at most
constexpr int kQKVRows = 2 * HEAD_DIM + 2 * HEAD_DIM;   // 512 rows per group
constexpr int kCtrStride = 16;              // counters 64 B apart
constexpr uint64_t kWaitNs = 2000000000ull; // 2 s

// counter slots
__host__ __device__ constexpr int ctr_g1(int l, int g) { return l * kGroups + g; }
__host__ __device__ constexpr int ctr_g2(int l, int g) { return N_LAYERS * kGroups + l * kGroups + g; }
__host__ __device__ constexpr int ctr_c3(int l) { return 2 * N_LAYERS * kGroups + l; }
__host__ __device__ constexpr int ctr_c5(int l) { return 2 * N_LAYERS * kGroups + N_LAYERS + l; }
__host__ __device__ constexpr int ctr_cf() { return 2 * N_LAYERS * kGroups + 2 * N_LAYERS; }
constexpr int kNumCtr = 2 * N_LAYERS * kGroups + 2 * N_LAYERS + 1;

// StepIn.flags
constexpr int kFlagWriteLogits = 1;   // store all fp32 logits
constexpr int kFlagNoHead = 2;        // skip the LM head and sampling (prompt positions)
constexpr int kFlagPromptToken = 4;   // token = prompt[pos] instead of StepIn.token

struct StepIn {          // host-written before a launch; chained steps update it on device
    int token;
    int pos;
    int top_k;
    int flags;
    float temperature;
    float topp;
    unsigned long long rng;
};
struct StepOut {         // device-maintained
    uint32_t epoch;      // launches completed + 1; counter targets are epoch * contributors
    int n_done;          // tokens appended to tokens_out
    uint32_t err;        // nonzero: a bounded wait expired
    int err_where;       // counter slot (or -1 - slot index for ring waits) that expired
    int out_token;
    int pad;
    unsigned long long rng;
};

struct DecodeParams {
    const uint16_t* embed;
    const uint16_t* lm;
    const uint16_t* final_ln;
    const uint16_t* in_ln[N_LAYERS];
    const uint16_t* post_ln[N_LAYERS];
    const uint16_t* wq[N_LAYERS];
    const uint16_t* wk[N_LAYERS];
    const uint16_t* wv[N_LAYERS];
    const uint16_t* qn[N_LAYERS];
    const uint16_t* kn[N_LAYERS];
    const uint16_t* wg[N_LAYERS];
    const uint16_t* wu[N_LAYERS];
    const uint16_t* wo_g;    // [L][8][DIM][256]  Wo columns of group g, row-major
    const uint16_t* wd_t;    // [L][HIDDEN][DIM]  Wd transposed
    uint16_t* kc;            // [L][8][SEQ][128]
    uint16_t* vc;            // [L][8][SEQ][128]
    const float* rope;       // [SEQ][128] cos[64] | sin[64]
    const int* prompt;       // [SEQ] prompt tokens (kFlagPromptToken)
    float* qkv;              // [L][4096]
    float* part;             // [L][8][kMaxGS][kPartStride]
    float* ybuf;             // [L][8][DIM]
    float* acc;              // [L][DIM]   zero between launches
    float* logits;           // [VOCAB]
    float* cand_v;           // [G][kMaxCand]
    int* cand_i;             // [G][kMaxCand]
    float* top_v;            // [kMaxCand] merged top-K of the last launch
    int* top_i;              // [kMaxCand]
    uint32_t* ctr;           // [kNumCtr * kCtrStride]
    StepIn* in;
    StepOut* out;
    int* tokens_out;         // [tokens_cap]
    int tokens_cap;
    int lm_begin, lm_end;    // LM-head rows served by this device
    int* chunk_count;        // [G][2] chunks issued (producer) / consumed (consumers)
    float* dbg_resid;        // [L][DIM] residual after each layer, or nullptr
};

struct __align__(16) DecodeSmem {
    uint64_t full[kSlots];
    uint64_t empty[kSlots];
    float xres[DIM];         // layer input, then post-attention residual
    float xs[DIM];           // normed activation
    float red[DIM];          // cross-warp scratch
    union {
        float sc[2][kScoreCap];
        float lg[kMaxLocalRows];
    } u;
    float qs[2 * HEAD_DIM];
    float kn[HEAD_DIM];
    float vn[HEAD_DIM];
    float gq[HEAD_DIM];
    float gk[HEAD_DIM];
    float rope[HEAD_DIM];
    float os[2 * HEAD_DIM];
    float gv[kMaxMlpRows];
    float uv[kMaxMlpRows];
    float hv[kMaxMlpRows];
    float bred[2][kNCW];
    int bidx[kNCW];
    int flag;
    int abort;               // set after a ring wait expired: stop waiting on the ring
};
constexpr size_t kDecodeSmemBytes = (size_t)kSlots * kSlotBytes + sizeof(DecodeSmem);

// [n*i/parts, n*(i+1)/parts)
__host__ __device__ __forceinline__ int span_lo(int n, int parts, int i) { return (int)(((long long)n * i) / parts); }

// CTA c of G -> attention group g, rank gr within it, group size gs.
__host__ __device__ __forceinline__ void group_of(int c, int G, int& g, int& gr, int& gs) {
    const int base = G / kGroups, rem = G % kGroups, big = rem * (base + 1);
    if (c < big) { g = c / (base + 1); gr = c % (base + 1); gs = base + 1; }
    else { const int c2 = c - big; g = rem + c2 / base; gr = c2 % base; gs = base; }
}

// Row r of group g's 512 QKV rows: source row pointer and destination in qkv[l].
__device__ __forceinline__ int qkv_dst(int g, int r) {
    return r < 256 ? 256 * g + r : (r < 384 ? Q_DIM + 128 * g + (r - 256) : Q_DIM + KV_DIM + 128 * g + (r - 384));
}

__device__ __forceinline__ void better(float& v, int& i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}

// ---------------------------------------------------------------------------
// Producer: one thread streams this CTA's chunks in consumption order.
// ---------------------------------------------------------------------------
struct Producer {
    uint8_t* ring;
    DecodeSmem* S;
    StepOut* out;
    uint32_t k = 0;
    uint64_t pol;
    bool dead = false;   // a slot never came free: issue nothing more
    __device__ uint8_t* begin(uint32_t bytes) {
        const uint32_t s = k % kSlots, ph = (k / kSlots) & 1u;
        if (!dead && !mbar_wait(&S->empty[s], ph ^ 1u, 2 * kWaitNs)) {
            atomicOr(&out->err, 2u);
            atomicExch(&out->err_where, -1 - (int)s);
            dead = true;
        }
        if (!dead) mbar_arrive_expect_tx(&S->full[s], bytes);
        return ring + (size_t)s * kSlotBytes;
    }
    __device__ void copy(uint8_t* dst, const void* src, uint32_t bytes) {
        if (!dead) bulk_g2s(dst, src, bytes, &S->full[k % kSlots], pol);
    }
    __device__ void end() { k++; }
    // rows [a, b) of a row-major matrix with `row_bytes` per row, chunked
    __device__ void rows(const uint16_t* base, int a, int b, int row_bytes) {
        const int per = kSlotBytes / row_bytes;
        for (int r = a; r < b; r += per) {
            const int n = min(per, b - r);
            uint8_t* d = begin((uint32_t)(n * row_bytes));
            copy(d, (const uint8_t*)base + (size_t)r * row_bytes, (uint32_t)(n * row_bytes));
            end();
        }
    }
};

__device__ __noinline__ void decode_producer(const DecodeParams& P, uint8_t* ring, DecodeSmem* S, int c, int G, int g,
                                             int gr, int gs, int pos, int flags) {
    Producer pr;
    pr.ring = ring; pr.S = S; pr.out = P.out; pr.pol = policy_evict_first();
    const int L = pos + 1;
    const int qa = span_lo(kQKVRows, gs, gr), qb = span_lo(kQKVRows, gs, gr + 1);
    const int p0 = span_lo(L, gs, gr), p1 = span_lo(L, gs, gr + 1);
    const int pe = min(p1, pos);                       // prefetched positions [p0, pe)
    const int oa = span_lo(DIM, gs, gr), ob = span_lo(DIM, gs, gr + 1);
    const int ha = span_lo(HIDDEN_DIM, G, c), hb = span_lo(HIDDEN_DIM, G, c + 1);
    for (int l = 0; l < N_LAYERS; l++) {
        {   // gains: input_layernorm | q_norm | k_norm
            uint8_t* d = pr.begin(2 * DIM + 4 * HEAD_DIM);
            pr.copy(d, P.in_ln[l], 2 * DIM);
            pr.copy(d + 2 * DIM, P.qn[l], 2 * HEAD_DIM);
            pr.copy(d + 2 * DIM + 2 * HEAD_DIM, P.kn[l], 2 * HEAD_DIM);
            pr.end();
        }
        for (int r = qa; r < qb; r += 16) {              // QKV rows (may straddle q/k/v)
            const int n = min(16, qb - r);
            uint8_t* d = pr.begin((uint32_t)(n * 2 * DIM));
            int i = 0;
            while (i < n) {
                const int rr = r + i;
                const uint16_t* src; int lim;
                if (rr < 256) { src = P.wq[l] + (size_t)(256 * g + rr) * DIM; lim = 256; }
                else if (rr < 384) { src = P.wk[l] + (size_t)(128 * g + rr - 256) * DIM; lim = 384; }
                else { src = P.wv[l] + (size_t)(128 * g + rr - 384) * DIM; lim = 512; }
                const int m = min(n - i, lim - rr);
                pr.copy(d + (size_t)i * 2 * DIM, src, (uint32_t)(m * 2 * DIM));
                i += m;
            }
            pr.end();
        }
        const size_t kvbase = ((size_t)(l * kGroups + g) * SEQ_LEN) * HEAD_DIM;
        pr.rows(P.kc + kvbase, p0, pe, 2 * HEAD_DIM);     // K of cached positions
        pr.rows(P.vc + kvbase, p0, pe, 2 * HEAD_DIM);     // V of cached positions
        pr.rows(P.wo_g + (size_t)(l * kGroups + g) * DIM * 256, oa, ob, 2 * 256);
        { uint8_t* d = pr.begin(2 * DIM); pr.copy(d, P.post_ln[l], 2 * DIM); pr.end(); }
        pr.rows(P.wg[l], ha, hb, 2 * DIM);
        pr.rows(P.wu[l], ha, hb, 2 * DIM);
        pr.rows(P.wd_t + (size_t)l * HIDDEN_DIM * DIM, ha, hb, 2 * DIM);
    }
    if (!(flags & kFlagNoHead)) {
        { uint8_t* d = pr.begin(2 * DIM); pr.copy(d, P.final_ln, 2 * DIM); pr.end(); }
        const int nrows = P.lm_end - P.lm_begin;
        const int va = P.lm_begin + span_lo(nrows, G, c), vb = P.lm_begin + span_lo(nrows, G, c + 1);
        pr.rows(P.lm, va, vb, 2 * DIM);
    }
    P.chunk_count[2 * c] = (int)pr.k;
}

// ---------------------------------------------------------------------------
// Consumers
// ---------------------------------------------------------------------------
struct Consumer {
    const DecodeParams* P;
    uint8_t* ring;
    DecodeSmem* S;
    int tid, warp, lane;
    uint32_t k = 0;
    bool err = false;   // meaningful in thread 0 only

    __device__ const uint8_t* wait_chunk() {
        const uint32_t s = k % kSlots, ph = (k / kSlots) & 1u;
        if (!*(volatile int*)&S->abort && !mbar_wait(&S->full[s], ph, 3 * kWaitNs)) {
            *(volatile int*)&S->abort = 1;
            atomicOr(&P->out->err, 4u);
            atomicExch(&P->out->err_where, -100 - (int)s);
        }
        return ring + (size_t)s * kSlotBytes;
    }
    __device__ void release_chunk() {
        __syncwarp();
        if (lane == 0) mbar_arrive(&S->empty[k % kSlots]);
        k++;
    }
    __device__ void bar() { named_bar(1, kNCT); }
    // Thread 0 waits until counter `idx` reaches `target` (wrap-safe), then all
    // consumers pass the named barrier.
    __device__ void wait_ctr(int idx, uint32_t target) {
        if (tid == 0 && !err) {
            const uint32_t* p = P->ctr + (size_t)idx * kCtrStride;
            if ((int)(ld_acquire(p) - target) < 0) {
                const uint64_t t0 = global_ns();
                uint32_t it = 0;
                while ((int)(ld_acquire(p) - target) < 0) {
                    if ((++it & 63u) == 0) {
                        if (ld_volatile(&P->out->err)) { err = true; break; }
                        if (global_ns() - t0 > kWaitNs) {
                            atomicOr(&P->out->err, 1u);
                            atomicExch(&P->out->err_where, idx);
                            err = true;
                            break;
                        }
                    }
                }
            }
        }
        bar();
    }
    __device__ void signal(int idx) {
        bar();
        if (tid == 0) {
            __threadfence();
            red_release_add(P->ctr + (size_t)idx * kCtrStride, 1u);
        }
    }
    __device__ float block_sum(float v) {
        v = warp_sum(v);
        if (lane == 0) S->bred[0][warp] = v;
        bar();
        float t = 0.f;
        #pragma unroll
        for (int i = 0; i < kNCW; i++) t += S->bred[0][i];
        bar();
        return t;
    }
    __device__ void block_max2(float& a, float& b) {
        a = warp_max(a); b = warp_max(b);
        if (lane == 0) { S->bred[0][warp] = a; S->bred[1][warp] = b; }
        bar();
        a = S->bred[0][0]; b = S->bred[1][0];
        #pragma unroll
        for (int i = 1; i < kNCW; i++) { a = fmaxf(a, S->bred[0][i]); b = fmaxf(b, S->bred[1][i]); }
        bar();
    }
    __device__ void block_sum2(float& a, float& b) {
        a = warp_sum(a); b = warp_sum(b);
        if (lane == 0) { S->bred[0][warp] = a; S->bred[1][warp] = b; }
        bar();
        a = 0.f; b = 0.f;
        #pragma unroll
        for (int i = 0; i < kNCW; i++) { a += S->bred[0][i]; b += S->bred[1][i]; }
        bar();
    }
    // argmax over the block: largest value, ties to the smallest index
    __device__ void block_argmax(float& v, int& i) {
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
            better(v, i, v2, i2);
        }
        if (lane == 0) { S->bred[0][warp] = v; S->bidx[warp] = i; }
        bar();
        v = S->bred[0][0]; i = S->bidx[0];
        #pragma unroll
        for (int w = 1; w < kNCW; w++) better(v, i, S->bred[0][w], S->bidx[w]);
        bar();
    }
    // x (fp32, DIM) staged in S->xres -> RMSNorm with the gains in the current
    // chunk at byte offset 0 -> S->xs; returns nothing; consumes no chunk.
    __device__ void norm_into_xs(const uint16_t* gain, float ss) {
        const float r = 1.0f / sqrtf(ss * (1.0f / DIM) + EPS);
        const int j = tid * 2;
        const uint32_t w = *(const uint32_t*)(gain + j);
        S->xs[j] = (S->xres[j] * r) * bf_lo(w);
        S->xs[j + 1] = (S->xres[j + 1] * r) * bf_hi(w);
    }
    // lane's 32 fp32 x values for a K=1024 row: x[256 i + 8 lane + e]
    __device__ void load_xr(float* xr) {
        #pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 a = *(const float4*)&S->xs[256 * i + 8 * lane];
            const float4 b = *(const float4*)&S->xs[256 * i + 8 * lane + 4];
            xr[8 * i + 0] = a.x; xr[8 * i + 1] = a.y; xr[8 * i + 2] = a.z; xr[8 * i + 3] = a.w;
            xr[8 * i + 4] = b.x; xr[8 * i + 5] = b.y; xr[8 * i + 6] = b.z; xr[8 * i + 7] = b.w;
        }
    }
    // dot of a 1024-wide bf16 row in shared memory with xr (full warp)
    __device__ float row_dot(const uint8_t* row, const float* xr) {
        const uint4* w = (const uint4*)row;
        float a = 0.f;
        #pragma unroll
        for (int i = 0; i < 4; i++) a = dot8(w[i * 32 + lane], &xr[8 * i], a);
        return warp_sum(a);
    }
};

__device__ __noinline__ void decode_consumer(const DecodeParams& P, uint8_t* ring, DecodeSmem* S, int c, int G, int g,
                                             int gr, int gs, int token, int pos, int flags, uint32_t epoch) {
    Consumer C;
    C.P = &P; C.ring = ring; C.S = S;
    C.tid = threadIdx.x; C.warp = C.tid >> 5; C.lane = C.tid & 31;
    const int tid = C.tid, warp = C.warp, lane = C.lane;
    const int L = pos + 1;
    const int qa = span_lo(kQKVRows, gs, gr), qb = span_lo(kQKVRows, gs, gr + 1);
    const int p0 = span_lo(L, gs, gr), p1 = span_lo(L, gs, gr + 1);
    const int pe = min(p1, pos);
    const bool owner = (gr == gs - 1);                 // its position range ends at pos
    const int oa = span_lo(DIM, gs, gr), ob = span_lo(DIM, gs, gr + 1);
    const int ha = span_lo(HIDDEN_DIM, G, c), hb = span_lo(HIDDEN_DIM, G, c + 1);
    const uint32_t tgt_all = epoch * (uint32_t)G, tgt_grp = epoch * (uint32_t)gs;
    const float sqrt_hd = sqrtf((float)HEAD_DIM);

    if (tid < HEAD_DIM) S->rope[tid] = __ldg(P.rope + (size_t)pos * HEAD_DIM + tid);

    for (int l = 0; l < N_LAYERS; l++) {
        // ---------------- QKV ----------------
        if (l > 0) C.wait_ctr(ctr_c5(l - 1), tgt_all);
        float ss;
        {
            const int j = tid * 2;
            float2 v;
            if (l == 0) {
                const uint32_t w = __ldg((const uint32_t*)(P.embed + (size_t)token * DIM + j));
                v = make_float2(bf_lo(w), bf_hi(w));
            } else {
                v = __ldcg((const float2*)(P.acc + (size_t)(l - 1) * DIM + j));
            }
            S->xres[j] = v.x; S->xres[j + 1] = v.y;
            ss = C.block_sum(v.x * v.x + v.y * v.y);
        }
        {
            const uint8_t* ch = C.wait_chunk();
            C.norm_into_xs((const uint16_t*)ch, ss);
            if (tid < HEAD_DIM) S->gq[tid] = bf2f(((const uint16_t*)(ch + 2 * DIM))[tid]);
            else if (tid < 2 * HEAD_DIM) S->gk[tid - HEAD_DIM] = bf2f(((const uint16_t*)(ch + 2 * DIM + 2 * HEAD_DIM))[tid - HEAD_DIM]);
            C.release_chunk();
        }
        C.bar();
        {
            float xr[32];
            C.load_xr(xr);
            for (int r = qa; r < qb; r += 16) {
                const int n = min(16, qb - r);
                const uint8_t* ch = C.wait_chunk();
                if (warp < n) {
                    const float a = C.row_dot(ch + (size_t)warp * 2 * DIM, xr);
                    if (lane == 0) P.qkv[(size_t)l * 4096 + qkv_dst(g, r + warp)] = a;
                }
                C.release_chunk();
            }
        }
        C.signal(ctr_g1(l, g));

        // ---------------- ATT ----------------
        C.wait_ctr(ctr_g1(l, g), tgt_grp);
        {
            const int hh = tid >> 7, d = tid & 127;       // 0: q head 2g, 1: q head 2g+1, 2: k, 3: v
            const int src = hh < 2 ? 256 * g + tid : (hh == 2 ? Q_DIM + 128 * g + d : Q_DIM + KV_DIM + 128 * g + d);
            float v = __ldcg(P.qkv + (size_t)l * 4096 + src);
            const float ssw = warp_sum(v * v);
            if (lane == 0) S->bred[0][warp] = ssw;
            C.bar();
            const float tot = (S->bred[0][4 * hh] + S->bred[0][4 * hh + 1]) + (S->bred[0][4 * hh + 2] + S->bred[0][4 * hh + 3]);
            if (hh < 3) {
                const float r = 1.0f / sqrtf(tot * (1.0f / HEAD_DIM) + EPS);
                v = (v * r) * (hh < 2 ? S->gq[d] : S->gk[d]);
            }
            S->red[tid] = v;
            C.bar();
            if (hh < 3) {
                const float p = S->red[tid ^ 64];
                const int j = d & 63;
                const float cj = S->rope[j], sj = S->rope[64 + j];
                v = d < 64 ? (v * cj - p * sj) : (p * sj + v * cj);
            }
            if (hh < 2) S->qs[tid] = v;
            else if (owner) {
                const uint16_t b = f2bf(v);
                const size_t at = (((size_t)(l * kGroups + g) * SEQ_LEN) + pos) * HEAD_DIM + d;
                if (hh == 2) { P.kc[at] = b; S->kn[d] = bf2f(b); }
                else { P.vc[at] = b; S->vn[d] = bf2f(b); }
            }
            C.bar();
        }
        float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
        {
            float q0[4], q1[4];
            #pragma unroll
            for (int e = 0; e < 4; e++) { q0[e] = S->qs[4 * lane + e]; q1[e] = S->qs[HEAD_DIM + 4 * lane + e]; }
            for (int t0 = p0; t0 < pe; t0 += 128) {
                const int cnt = min(128, pe - t0);
                const uint8_t* ch = C.wait_chunk();
                for (int i = warp; i < cnt; i += kNCW) {
                    const uint2 kw = ((const uint2*)(ch + (size_t)i * 2 * HEAD_DIM))[lane];
                    const float k0 = bf_lo(kw.x), k1 = bf_hi(kw.x), k2 = bf_lo(kw.y), k3 = bf_hi(kw.y);
                    float a0 = q0[0] * k0; a0 = fmaf(q0[1], k1, a0); a0 = fmaf(q0[2], k2, a0); a0 = fmaf(q0[3], k3, a0);
                    float a1 = q1[0] * k0; a1 = fmaf(q1[1], k1, a1); a1 = fmaf(q1[2], k2, a1); a1 = fmaf(q1[3], k3, a1);
                    a0 = warp_sum(a0); a1 = warp_sum(a1);
                    if (lane == 0) { S->u.sc[0][t0 - p0 + i] = a0 / sqrt_hd; S->u.sc[1][t0 - p0 + i] = a1 / sqrt_hd; }
                }
                C.release_chunk();
            }
            if (owner && warp == 0) {
                float a0 = 0.f, a1 = 0.f;
                #pragma unroll
                for (int e = 0; e < 4; e++) { a0 = fmaf(q0[e], S->kn[4 * lane + e], a0); a1 = fmaf(q1[e], S->kn[4 * lane + e], a1); }
                a0 = warp_sum(a0); a1 = warp_sum(a1);
                if (lane == 0) { S->u.sc[0][pos - p0] = a0 / sqrt_hd; S->u.sc[1][pos - p0] = a1 / sqrt_hd; }
            }
            C.bar();
            const int n = p1 - p0;
            for (int i = tid; i < n; i += kNCT) { m0 = fmaxf(m0, S->u.sc[0][i]); m1 = fmaxf(m1, S->u.sc[1][i]); }
            C.block_max2(m0, m1);
            for (int i = tid; i < n; i += kNCT) {
                const float e0 = expf(S->u.sc[0][i] - m0), e1 = expf(S->u.sc[1][i] - m1);
                S->u.sc[0][i] = e0; S->u.sc[1][i] = e1; l0 += e0; l1 += e1;
            }
            C.block_sum2(l0, l1);
        }
        {
            const int half = tid >> 8, hh = (tid >> 7) & 1, d = tid & 127;
            float a = 0.f;
            for (int t0 = p0; t0 < pe; t0 += 128) {
                const int cnt = min(128, pe - t0);
                const uint16_t* vv = (const uint16_t*)C.wait_chunk();
                const float* pr = &S->u.sc[hh][t0 - p0];
                for (int i = half; i < cnt; i += 2) a = fmaf(pr[i], bf2f(vv[i * HEAD_DIM + d]), a);
                C.release_chunk();
            }
            if (owner && half == 0) a = fmaf(S->u.sc[hh][pos - p0], S->vn[d], a);
            if (half == 1) S->red[tid - 256] = a;
            C.bar();
            float* base = P.part + ((size_t)(l * kGroups + g) * kMaxGS + gr) * kPartStride;
            if (half == 0) base[hh * kHeadPart + 4 + d] = a + S->red[tid];
            if (tid == 0) { base[0] = m0; base[1] = l0; base[kHeadPart] = m1; base[kHeadPart + 1] = l1; }
        }
        C.signal(ctr_g2(l, g));

        // ---------------- OPROJ ----------------
        C.wait_ctr(ctr_g2(l, g), tgt_grp);
        if (tid < 2 * HEAD_DIM) {
            const int hh = tid >> 7, d = tid & 127;
            const float* base = P.part + (size_t)(l * kGroups + g) * kMaxGS * kPartStride + hh * kHeadPart;
            float M = -INFINITY;
            for (int cc = 0; cc < gs; cc++) M = fmaxf(M, __ldcg(base + (size_t)cc * kPartStride));
            float den = 0.f, num = 0.f;
            for (int cc = 0; cc < gs; cc++) {
                const float* b = base + (size_t)cc * kPartStride;
                const float lc = __ldcg(b + 1);
                if (lc > 0.f) {
                    const float w = expf(__ldcg(b) - M);
                    den = fmaf(lc, w, den);
                    num = fmaf(__ldcg(b + 4 + d), w, num);
                }
            }
            S->os[tid] = num / den;
        }
        C.bar();
        {
            float o8[8];
            #pragma unroll
            for (int e = 0; e < 8; e++) o8[e] = S->os[8 * lane + e];
            for (int r = oa; r < ob; r += 64) {
                const int cnt = min(64, ob - r);
                const uint8_t* ch = C.wait_chunk();
                for (int i = warp; i < cnt; i += kNCW) {
                    const uint4 w = ((const uint4*)(ch + (size_t)i * 512))[lane];
                    const float a = warp_sum(dot8(w, o8, 0.f));
                    if (lane == 0) P.ybuf[(size_t)(l * kGroups + g) * DIM + r + i] = a;
                }
                C.release_chunk();
            }
        }
        C.signal(ctr_c3(l));

        // ---------------- MLP ----------------
        C.wait_ctr(ctr_c3(l), tgt_all);
        {
            const int j = tid * 2;
            float2 x = make_float2(S->xres[j], S->xres[j + 1]);
            #pragma unroll
            for (int gg = 0; gg < kGroups; gg++) {
                const float2 y = __ldcg((const float2*)(P.ybuf + (size_t)(l * kGroups + gg) * DIM + j));
                x.x += y.x; x.y += y.y;
            }
            S->xres[j] = x.x; S->xres[j + 1] = x.y;
            ss = C.block_sum(x.x * x.x + x.y * x.y);
        }
        {
            const uint8_t* ch = C.wait_chunk();
            C.norm_into_xs((const uint16_t*)ch, ss);
            C.release_chunk();
        }
        C.bar();
        {
            float xr[32];
            C.load_xr(xr);
            for (int r = ha; r < hb; r += 16) {
                const int n = min(16, hb - r);
                const uint8_t* ch = C.wait_chunk();
                if (warp < n) {
                    const float a = C.row_dot(ch + (size_t)warp * 2 * DIM, xr);
                    if (lane == 0) S->gv[r - ha + warp] = a;
                }
                C.release_chunk();
            }
            for (int r = ha; r < hb; r += 16) {
                const int n = min(16, hb - r);
                const uint8_t* ch = C.wait_chunk();
                if (warp < n) {
                    const float a = C.row_dot(ch + (size_t)warp * 2 * DIM, xr);
                    if (lane == 0) S->uv[r - ha + warp] = a;
                }
                C.release_chunk();
            }
        }
        C.bar();
        if (tid < hb - ha) {
            const float gt = S->gv[tid];
            S->hv[tid] = (gt / (1.0f + expf(-gt))) * S->uv[tid];
        }
        C.bar();
        {
            const int cb = warp & 7, par = warp >> 3, col = cb * 128 + lane * 4;
            float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
            for (int r = ha; r < hb; r += 16) {
                const int cnt = min(16, hb - r);
                const uint8_t* ch = C.wait_chunk();
                for (int i = par; i < cnt; i += 2) {
                    const float h = S->hv[r - ha + i];
                    const uint2 w = *(const uint2*)(ch + (size_t)i * 2 * DIM + (size_t)col * 2);
                    a0 = fmaf(h, bf_lo(w.x), a0); a1 = fmaf(h, bf_hi(w.x), a1);
                    a2 = fmaf(h, bf_lo(w.y), a2); a3 = fmaf(h, bf_hi(w.y), a3);
                }
                C.release_chunk();
            }
            if (par == 1) *(float4*)&S->red[col] = make_float4(a0, a1, a2, a3);
            C.bar();
            if (par == 0) {
                const float4 o = *(const float4*)&S->red[col];
                a0 += o.x; a1 += o.y; a2 += o.z; a3 += o.w;
                if (c == 0) { a0 += S->xres[col]; a1 += S->xres[col + 1]; a2 += S->xres[col + 2]; a3 += S->xres[col + 3]; }
                atomicAdd((float4*)(P.acc + (size_t)l * DIM + col), make_float4(a0, a1, a2, a3));
            }
        }
        C.signal(ctr_c5(l));
    }

    // ---------------- HEAD ----------------
    C.wait_ctr(ctr_c5(N_LAYERS - 1), tgt_all);
    {   // zero acc[0 .. L-2] for the next launch (every CTA has read them by now)
        const int tot = (N_LAYERS - 1) * DIM;
        const int lo = span_lo(tot, G, c), hi = span_lo(tot, G, c + 1);
        for (int i = lo + tid; i < hi; i += kNCT) {
            if (P.dbg_resid) P.dbg_resid[i] = __ldcg(P.acc + i);
            P.acc[i] = 0.f;
        }
    }
    const bool head = !(flags & kFlagNoHead);
    const bool greedy = (P.in->temperature == 0.0f || P.in->top_k == 1);
    const int K = greedy ? 1 : min(P.in->top_k, kMaxCand);
    if (head) {
        float ss;
        {
            const int j = tid * 2;
            const float2 v = __ldcg((const float2*)(P.acc + (size_t)(N_LAYERS - 1) * DIM + j));
            S->xres[j] = v.x; S->xres[j + 1] = v.y;
            ss = C.block_sum(v.x * v.x + v.y * v.y);
        }
        {
            const uint8_t* ch = C.wait_chunk();
            C.norm_into_xs((const uint16_t*)ch, ss);
            C.release_chunk();
        }
        C.bar();
        const int nrows = P.lm_end - P.lm_begin;
        const int va = P.lm_begin + span_lo(nrows, G, c), vb = P.lm_begin + span_lo(nrows, G, c + 1);
        const bool wl = (flags & kFlagWriteLogits) != 0;
        {
            float xr[32];
            C.load_xr(xr);
            for (int r = va; r < vb; r += 16) {
                const int n = min(16, vb - r);
                const uint8_t* ch = C.wait_chunk();
                if (warp < n) {
                    const float a = C.row_dot(ch + (size_t)warp * 2 * DIM, xr);
                    if (lane == 0) {
                        S->u.lg[r - va + warp] = a;
                        if (wl) P.logits[r + warp] = a;
                    }
                }
                C.release_chunk();
            }
        }
        C.bar();
        const int nloc = vb - va;
        for (int kk = 0; kk < K; kk++) {
            float v = -INFINITY; int i = 0x7fffffff;
            for (int t = tid; t < nloc; t += kNCT) better(v, i, S->u.lg[t], t);
            C.block_argmax(v, i);
            if (tid == 0) {
                P.cand_v[(size_t)c * kMaxCand + kk] = v;
                P.cand_i[(size_t)c * kMaxCand + kk] = (i < nloc) ? va + i : 0x7fffffff;
                if (i < nloc) S->u.lg[i] = -INFINITY;
            }
            C.bar();
        }
    }
    // last CTA to arrive merges and samples
    C.bar();
    if (tid == 0) P.chunk_count[2 * c + 1] = (int)C.k;
    if (tid == 0) {
        __threadfence();
        const uint32_t old = atom_acq_rel_add(P.ctr + (size_t)ctr_cf() * kCtrStride, 1u);
        S->flag = (old == epoch * (uint32_t)G - 1u) ? 1 : 0;
    }
    C.bar();
    if (!S->flag) return;

    int tok = -1;
    if (head) {
        // all G*K candidates into the (now idle) ring
        float* cv = (float*)ring;
        int* ci = (int*)(ring + (size_t)G * kMaxCand * sizeof(float));
        const int tot = G * K;
        for (int t = tid; t < tot; t += kNCT) {
            const int cc = t / K, kk = t % K;
            cv[t] = __ldcg(P.cand_v + (size_t)cc * kMaxCand + kk);
            ci[t] = __ldcg(P.cand_i + (size_t)cc * kMaxCand + kk);
        }
        C.bar();
        for (int kk = 0; kk < K; kk++) {
            float v = -INFINITY; int i = 0x7fffffff, at = -1;
            for (int t = tid; t < tot; t += kNCT) {
                const float v2 = cv[t]; const int i2 = ci[t];
                if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; at = t; }
            }
            // reduce (value, id) and remember where the winner sits
            #pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
                const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
                const int a2 = __shfl_xor_sync(0xffffffffu, at, o);
                if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; at = a2; }
            }
            if (lane == 0) { S->bred[0][warp] = v; S->bidx[warp] = i; S->bred[1][warp] = __int_as_float(at); }
            C.bar();
            if (tid == 0) {
                float bv = S->bred[0][0]; int bi = S->bidx[0]; int ba = __float_as_int(S->bred[1][0]);
                for (int w = 1; w < kNCW; w++) {
                    const float v2 = S->bred[0][w]; const int i2 = S->bidx[w];
                    if (v2 > bv || (v2 == bv && i2 < bi)) { bv = v2; bi = i2; ba = __float_as_int(S->bred[1][w]); }
                }
                P.top_v[kk] = bv; P.top_i[kk] = bi;
                S->gv[kk] = bv; S->hv[kk] = __int_as_float(bi);
                if (ba >= 0) cv[ba] = -INFINITY, ci[ba] = 0x7fffffff;
            }
            C.bar();
        }
        if (tid == 0) {
            unsigned long long rng = P.in->rng;
            if (greedy) {
                tok = __float_as_int(S->hv[0]);
            } else {
                // sampler.h:137-174 over the K candidates, scanned in descending order
                const float T = P.in->temperature, topp = P.in->topp;
                int nc = K;
                const float mx = S->gv[0];
                float sum = 0.f;
                for (int i = 0; i < nc; i++) { const float e = expf((S->gv[i] - mx) / T); S->uv[i] = e; sum += e; }
                for (int i = 0; i < nc; i++) S->uv[i] /= sum;
                if (topp > 0.0f && topp < 1.0f) {
                    float cum = 0.f; int last = nc - 1;
                    for (int i = 0; i < nc; i++) { cum += S->uv[i]; if (cum > topp) { last = i; break; } }
                    nc = last + 1; sum = cum;
                }
                rng ^= rng >> 12; rng ^= rng << 25; rng ^= rng >> 27;
                const uint32_t u = (uint32_t)((rng * 0x2545F4914F6CDD1Dull) >> 32);
                const float coin = ((float)(u >> 8) / 16777216.0f) * sum;
                float cdf = 0.f;
                tok = __float_as_int(S->hv[nc - 1]);
                for (int i = 0; i < nc; i++) { cdf += S->uv[i]; if (coin < cdf) { tok = __float_as_int(S->hv[i]); break; } }
            }
            P.in->rng = rng;
            P.out->rng = rng;
        }
    }
    for (int i = tid; i < DIM; i += kNCT) {
        if (P.dbg_resid) P.dbg_resid[(size_t)(N_LAYERS - 1) * DIM + i] = __ldcg(P.acc + (size_t)(N_LAYERS - 1) * DIM + i);
        P.acc[(size_t)(N_LAYERS - 1) * DIM + i] = 0.f;
    }
    if (tid == 0) {
        P.out->out_token = tok;
        if (head) {
            const int nd = P.out->n_done;
            if (nd < P.tokens_cap) P.tokens_out[nd] = tok;
            P.out->n_done = nd + 1;
            P.in->token = tok;
        } else if (flags & kFlagPromptToken) {
            P.in->token = P.prompt[min(pos + 1, SEQ_LEN - 1)];
        }
        P.in->pos = pos + 1;
        __threadfence();
        P.out->epoch = epoch + 1;
    }
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeParams P) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    DecodeSmem* S = reinterpret_cast<DecodeSmem*>(smem + (size_t)kSlots * kSlotBytes);
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int s = 0; s < kSlots; s++) { mbar_init(&S->full[s], 1); mbar_init(&S->empty[s], kNCW); }
        S->abort = 0;
        fence_barrier_init();
    }
    __syncthreads();
    const int c = blockIdx.x, G = gridDim.x;
    int g, gr, gs;
    group_of(c, G, g, gr, gs);
    const int flags = P.in->flags;
    const int pos = P.in->pos;
    const int token = (flags & kFlagPromptToken) ? P.prompt[pos] : P.in->token;
    const uint32_t epoch = P.out->epoch;
    if ((tid >> 5) == kNCW) {
        if ((tid & 31) == 0) decode_producer(P, ring, S, c, G, g, gr, gs, pos, flags);
        return;
    }
    decode_consumer(P, ring, S, c, G, g, gr, gs, token, pos, flags, epoch);
}

}  // namespace qb
