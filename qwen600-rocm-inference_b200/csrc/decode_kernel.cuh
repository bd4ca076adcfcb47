// decode_kernel.cuh — one batch-1 decode position of Qwen3-0.6B as ONE
// persistent cooperative kernel (one CTA per SM).
//
// Replaces the reference's per-token chain of ~450 launches
// (qwen_model.cuh:772-851: rmsnorm_gpu, 7 cuBLAS GEMVs per layer,
// qk_norm_fused_gpu, rope_gpu_naive, attention_gpu with a device sync,
// swiglu_gpu, the LM head and the bf16->fp32 conversion) and, for the
// device-sampling entry points, the host sampler (sampler.h:120-175).
//
// Weight streaming.  Every CTA owns a fixed slice of every matrix.  A producer
// warp streams the CTA's slices, in consumption order, through a ring of
// kSlots x 32 KB shared-memory slots with 1-D bulk async copies (TMA engine,
// mbarrier completion, L2 evict-first); a second cursor issues bulk L2
// prefetches kPrefetchChunks further ahead, so the 126 MB L2 is the deep
// buffer and HBM keeps streaming while the ring is full.  The stream never
// waits on activations.  Sixteen consumer warps compute from the slots.
//
// Activation exchange.  Every value one CTA hands to another is an 8-byte word
// (fp32 value | 32-bit sequence tag) written with one relaxed 64-bit store;
// the consumer polls the words it needs until their tag equals this launch's
// sequence number.  No fences, no counters: a hop costs about one L2 round
// trip.  Per layer l (the 8 KV heads define 8 CTA groups of ~G/8 CTAs):
//
//   QKV   group g: x_l -> RMSNorm (input_layernorm) -> its rows of the
//         group's 512 projection rows (q heads 2g, 2g+1; k, v head g)  -> qkv
//   ATT   group g: QK-norm + RoPE of q/k; the CTA whose positions end at pos
//         appends bf16 K/V; split-K attention over its share of positions
//         with a per-warp online softmax                          -> partials
//   OPROJ group g: combine the group's partials -> o (256 values) -> its rows
//         of Wo[:, 256g:256g+256] (packed contiguous)             -> y[g]
//   MLP-A all: x_mid = x_l + sum_g y[g] (fixed order); RMSNorm
//         (post_attention_layernorm) -> its gate and up rows -> SwiGLU -> h
//   MLP-B all: its rows r of Wd: x_{l+1}[r] = x_mid[r] + Wd[r] . h  -> x_{l+1}
//   HEAD  all: final RMSNorm -> its LM-head rows -> fp32 logits and a local
//         top-K; the last CTA to finish (one atomic) merges the candidates
//         and samples (argmax, or temperature / top-k / top-p, xorshift64*).
//
// Numerics: weights and the KV cache are bf16; activations, the residual
// stream and all accumulations are fp32, and every reduction has a fixed
// order, so a launch is bit-reproducible for a given grid size.
//
// Every wait is bounded (kWaitNs): on expiry the kernel records an error in
// StepOut.err, stops waiting on other CTAs, still drains its own copies, and
// returns; the host then resets the exchange buffers.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "../host/config.h"

namespace qb {

constexpr int kNCW = 16;                    // consumer warps
constexpr int kNCT = kNCW * 32;             // consumer threads
constexpr int kThreads = kNCT + 64;         // + one producer warp + one L2-prefetch warp
constexpr int kSlots = 4;
constexpr int kSlotBytes = 32768;
constexpr int kGroups = N_KV_HEADS;         // one CTA group per KV head
constexpr int kMaxGS = 19;                  // max CTAs per group (grid <= 152)
constexpr int kMinGS = 8;                   // min CTAs per group (grid >= 64)
constexpr int kMaxCand = 64;                // device top-k limit
constexpr int kHeadPart = 4 + HEAD_DIM;     // m, l, pad, pad, acc[128]
constexpr int kPartStride = 2 * kHeadPart;  // both q heads of a group
constexpr int kMaxLocalRows = 1280;         // LM-head rows per CTA at most
constexpr int kMaxMlpRows = 64;             // hidden rows per CTA at most
constexpr int kQKVRows = 2 * HEAD_DIM + 2 * HEAD_DIM;   // 512 rows per group
constexpr int kCtrStride = 16;              // counters 64 B apart
constexpr uint64_t kWaitNs = 2000000000ull; // 2 s
constexpr int kNumCtr = 1;                  // the head's arrival counter
// trace slots per CTA: 0 start; 1 + 10l + k for layer l:
//   k = 0 x ready, 1 QKV done, 2 q/k/v ready, 3 ATT done, 4 partials ready,
//   5 OPROJ done, 6 y ready, 7 MLP-A done, 8 h ready, 9 MLP-B done;
// 281 HEAD in, 282 LM rows done, 283 arrival, 284 sample done;
// 288 + l producer issues layer l; 316 producer issues the head;
// 320 + l ns thread 0 spent waiting for ring chunks in layer l (348: head);
// 352 + l ns thread 0 spent waiting for exchange words in layer l (380: head)
constexpr int kTraceStride = 576;   // 384 + i: sub-stage stamps of layer 13; 448+: its ring chunks
constexpr int kTrHead = 1 + 10 * N_LAYERS;

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
    uint32_t seq;        // sequence number of the next launch (exchange-word tag), >= 1
    int n_done;          // tokens appended to tokens_out
    uint32_t err;        // nonzero: a bounded wait expired
    int err_where;       // stage code (or ring slot) whose wait expired
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
    const uint16_t* wd[N_LAYERS];
    const uint16_t* wo_g;    // [L][8][DIM][256]  Wo columns of group g, row-major
    uint16_t* kc;            // [L][8][SEQ][128]
    uint16_t* vc;            // [L][8][SEQ][128]
    const float* rope;       // [SEQ][128] cos[64] | sin[64]
    const int* prompt;       // [SEQ] prompt tokens (kFlagPromptToken)
    // exchange words (value | tag << 32)
    uint64_t* xw;            // [L+1][DIM]   residual at the start of layer l (l >= 1); [L] = final
    uint64_t* qkvw;          // [L][4096]    raw q | k | v projections
    uint64_t* partw;         // [L][8][kMaxGS][kPartStride]
    uint64_t* yw;            // [L][8][DIM]  O-projection partial of each group
    uint64_t* hw;            // [L][HIDDEN]  SwiGLU output
    float* logits;           // [VOCAB]
    float* cand_v;           // [G][kMaxCand]
    int* cand_i;             // [G][kMaxCand]
    float* top_v;            // [kMaxCand] merged top-K of the last launch
    int* top_i;              // [kMaxCand]
    uint32_t* ctr;           // [kNumCtr * kCtrStride]: arrival counter of the head
    StepIn* in;
    StepOut* out;
    int* tokens_out;         // [tokens_cap]
    int tokens_cap;
    int lm_begin, lm_end;    // LM-head rows served by this device
    int* chunk_count;        // [G][2] chunks issued (producer) / consumed (consumers)
    unsigned long long* trace;   // [G][kTraceStride] %globaltimer stamps, or nullptr
    int prefetch_chunks;     // L2 prefetch lead of the producer, in chunks (0 = none)
    int poll_ns;             // back-off between polls of an exchange word
    int ring_slots;          // ring slots in use, 2..kSlots (bounds the bulk bytes in flight)
};

struct Plan {          // this CTA's share of every stage
    int g, gr, gs;
    int qa, qb;        // QKV rows of the group's 512
    int p0, p1, pe;    // attention positions [p0, p1); cached ones [p0, pe)
    int oa, ob;        // Wo_g rows
    int ha, hb;        // hidden rows (gate / up)
    int da, db;        // output rows of Wd
    int va, vb;        // LM-head rows
    bool head;
    size_t kvbase;     // element offset of (layer 0, head g) in the K/V cache
};

struct __align__(16) DecodeSmem {
    uint64_t full[kSlots];
    uint64_t empty[kSlots];
    float xres[DIM];         // layer input x_l, then x_mid
    float xs[DIM];           // normed activation
    union {                  // one stage at a time (a barrier separates users)
        float hs[HIDDEN_DIM];                 // MLP-B: h; head merge: probabilities
        float comb[kNCW * HEAD_DIM];          // ATT: per-warp accumulators
        float pst[kMaxGS * kPartStride];      // OPROJ: the group's partials
        float lg[kMaxLocalRows];              // HEAD: local logits
    } w;
    float qs[2 * HEAD_DIM];
    float kn[HEAD_DIM];
    float vn[HEAD_DIM];
    float gq[HEAD_DIM];
    float gk[HEAD_DIM];
    float rope[HEAD_DIM];
    float os[2 * HEAD_DIM];
    float gv[kMaxMlpRows];
    float uv[kMaxMlpRows];
    float part[kNCW];
    float bred[2][kNCW];
    int bidx[kNCW];
    int flag;
    int abort;               // set after a ring wait expired: stop waiting on the ring
    unsigned int copied;     // chunks the producer has issued (read by the prefetch warp)
    Plan pl;                 // this CTA's share of every stage (one copy, in shared memory)
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

// Row r of group g's 512 QKV rows -> its index in the layer's q | k | v vector.
__device__ __forceinline__ int qkv_dst(int g, int r) {
    return r < 256 ? 256 * g + r : (r < 384 ? Q_DIM + 128 * g + (r - 256) : Q_DIM + KV_DIM + 128 * g + (r - 384));
}

__device__ __forceinline__ void better(float& v, int& i, float v2, int i2) {
    if (v2 > v || (v2 == v && i2 < i)) { v = v2; i = i2; }
}

// ---- exchange words ---------------------------------------------------------
__device__ __forceinline__ void xw_store(uint64_t* p, float v, uint32_t tag) {
    const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t xw_load(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// two consecutive words (16-byte aligned); each word is checked on its own
__device__ __forceinline__ void xw_load2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// ---------------------------------------------------------------------------
// The chunk sequence.  One CTA's weight / KV stream, in consumption order:
//   per layer: [gains: input_ln | q_norm | k_norm] [QKV rows, 16/chunk]
//              [K | V of cached positions, 64/chunk: K at 0, V at 16 KB]
//              [Wo_g rows, 64/chunk] [post_ln] [gate rows, 16/chunk]
//              [up rows, 16/chunk] [Wd rows (3072 wide), 5/chunk]
//   then (unless kFlagNoHead): [final_ln] [LM-head rows, 16/chunk]
// The producer walks it twice (an L2-prefetch cursor ahead of the copy
// cursor); the consumers' code visits the same chunks in the same order.
// ---------------------------------------------------------------------------
constexpr int kRowsK1024 = kSlotBytes / (2 * DIM);        // 16 rows of 1024 bf16
constexpr int kRowsK3072 = kSlotBytes / (2 * HIDDEN_DIM); // 5 rows of 3072 bf16
constexpr int kKVChunk = 64;                               // positions per K|V chunk
constexpr int kVOff = kKVChunk * 2 * HEAD_DIM;             // V offset in a K|V chunk
constexpr int kRowsWo = kSlotBytes / (2 * 256);            // 64 rows of 256 bf16

__device__ __forceinline__ Plan make_plan(const DecodeParams& P, int c, int G, int pos, int flags) {
    Plan p;
    group_of(c, G, p.g, p.gr, p.gs);
    const int L = pos + 1;
    p.qa = span_lo(kQKVRows, p.gs, p.gr); p.qb = span_lo(kQKVRows, p.gs, p.gr + 1);
    p.p0 = span_lo(L, p.gs, p.gr); p.p1 = span_lo(L, p.gs, p.gr + 1);
    p.pe = min(p.p1, pos);
    p.oa = span_lo(DIM, p.gs, p.gr); p.ob = span_lo(DIM, p.gs, p.gr + 1);
    p.ha = span_lo(HIDDEN_DIM, G, c); p.hb = span_lo(HIDDEN_DIM, G, c + 1);
    p.da = span_lo(DIM, G, c); p.db = span_lo(DIM, G, c + 1);
    const int nrows = P.lm_end - P.lm_begin;
    p.va = P.lm_begin + span_lo(nrows, G, c); p.vb = P.lm_begin + span_lo(nrows, G, c + 1);
    p.head = !(flags & kFlagNoHead);
    p.kvbase = (size_t)p.g * SEQ_LEN * HEAD_DIM;
    return p;
}

struct Seg {
    const uint8_t* src;
    uint32_t bytes;
    uint32_t off;      // destination offset inside the slot
};

struct ChunkIter {
    int l = 0, st = 0, r = 0;
    int cur_st = 0, cur_l = 0;   // stage and layer of the chunk last returned
    // Fills seg[] with the next chunk's copies; returns their count (0 at the end).
    __device__ int next(const DecodeParams& P, const Plan& pl, Seg* seg) {
        const int n = step(P, pl, seg);
        return n;
    }
    __device__ int step(const DecodeParams& P, const Plan& pl, Seg* seg) {
        for (;;) {
            cur_st = st; cur_l = l;
            switch (st) {
            case 0:
                seg[0] = {(const uint8_t*)P.in_ln[l], 2 * DIM, 0};
                seg[1] = {(const uint8_t*)P.qn[l], 2 * HEAD_DIM, 2 * DIM};
                seg[2] = {(const uint8_t*)P.kn[l], 2 * HEAD_DIM, 2 * DIM + 2 * HEAD_DIM};
                st = 1; r = pl.qa;
                return 3;
            case 1:
                if (r < pl.qb) {
                    const int n = min(kRowsK1024, pl.qb - r);
                    int i = 0, k = 0;
                    while (i < n) {
                        const int rr = r + i;
                        const uint16_t* src; int lim;
                        if (rr < 256) { src = P.wq[l] + (size_t)(256 * pl.g + rr) * DIM; lim = 256; }
                        else if (rr < 384) { src = P.wk[l] + (size_t)(128 * pl.g + rr - 256) * DIM; lim = 384; }
                        else { src = P.wv[l] + (size_t)(128 * pl.g + rr - 384) * DIM; lim = 512; }
                        const int m = min(n - i, lim - rr);
                        seg[k++] = {(const uint8_t*)src, (uint32_t)(m * 2 * DIM), (uint32_t)(i * 2 * DIM)};
                        i += m;
                    }
                    r += n;
                    return k;
                }
                st = 2; r = pl.p0;
                break;
            case 2:
                if (r < pl.pe) {
                    const int n = min(kKVChunk, pl.pe - r);
                    const size_t e = ((size_t)l * kGroups * SEQ_LEN * HEAD_DIM) + pl.kvbase + (size_t)r * HEAD_DIM;
                    seg[0] = {(const uint8_t*)(P.kc + e), (uint32_t)(n * 2 * HEAD_DIM), 0};
                    seg[1] = {(const uint8_t*)(P.vc + e), (uint32_t)(n * 2 * HEAD_DIM), (uint32_t)kVOff};
                    r += n;
                    return 2;
                }
                st = 3; r = pl.oa;
                break;
            case 3:
                if (r < pl.ob) {
                    const int n = min(kRowsWo, pl.ob - r);
                    seg[0] = {(const uint8_t*)(P.wo_g + ((size_t)(l * kGroups + pl.g) * DIM + r) * 256), (uint32_t)(n * 512), 0};
                    r += n;
                    return 1;
                }
                st = 4;
                break;
            case 4:
                seg[0] = {(const uint8_t*)P.post_ln[l], 2 * DIM, 0};
                st = 5; r = pl.ha;
                return 1;
            case 5:
            case 6:
                if (r < pl.hb) {
                    const int n = min(kRowsK1024, pl.hb - r);
                    const uint16_t* base = st == 5 ? P.wg[l] : P.wu[l];
                    seg[0] = {(const uint8_t*)(base + (size_t)r * DIM), (uint32_t)(n * 2 * DIM), 0};
                    r += n;
                    return 1;
                }
                if (st == 5) { st = 6; r = pl.ha; break; }
                st = 7; r = pl.da;
                break;
            case 7:
                if (r < pl.db) {
                    const int n = min(kRowsK3072, pl.db - r);
                    seg[0] = {(const uint8_t*)(P.wd[l] + (size_t)r * HIDDEN_DIM), (uint32_t)(n * 2 * HIDDEN_DIM), 0};
                    r += n;
                    return 1;
                }
                if (++l < N_LAYERS) { st = 0; break; }
                st = pl.head ? 8 : 10;
                break;
            case 8:
                seg[0] = {(const uint8_t*)P.final_ln, 2 * DIM, 0};
                st = 9; r = pl.va;
                return 1;
            case 9:
                if (r < pl.vb) {
                    const int n = min(kRowsK1024, pl.vb - r);
                    seg[0] = {(const uint8_t*)(P.lm + (size_t)r * DIM), (uint32_t)(n * 2 * DIM), 0};
                    r += n;
                    return 1;
                }
                st = 10;
                break;
            default:
                return 0;
            }
        }
    }
};

// ---------------------------------------------------------------------------
// Producer: one thread copies chunks into the ring.  A second warp (one
// thread) walks the same sequence issuing bulk L2 prefetches up to
// P.prefetch_chunks chunks ahead of the producer; it keeps HBM streaming while
// the ring is full because consumers wait on another CTA.
// ---------------------------------------------------------------------------
__device__ __noinline__ void decode_producer(const DecodeParams& P, uint8_t* ring, DecodeSmem* S, int c, const Plan& pl) {
    const uint64_t pol = policy_evict_first();
    unsigned long long* tr = P.trace ? P.trace + (size_t)c * kTraceStride : nullptr;
    ChunkIter it;
    Seg seg[3];
    uint32_t k = 0;
    int k13 = -1;
    bool dead = false;
    for (;;) {
        const int n = it.next(P, pl, seg);
        if (n == 0) break;
        const uint32_t ns = (uint32_t)P.ring_slots;
        const uint32_t s = k % ns, ph = (k / ns) & 1u;
        if (!dead && !mbar_wait(&S->empty[s], ph ^ 1u, 2 * kWaitNs)) {
            atomicOr(&P.out->err, 2u);
            atomicExch(&P.out->err_where, -1 - (int)s);
            dead = true;   // issue nothing more; consumers stop waiting after their own timeout
        }
        if (tr && it.cur_st == 0) tr[288 + it.cur_l] = global_ns();
        if (tr && it.cur_l == 13 && it.cur_st <= 7) {   // layer 13's chunks: issue cycle and stage
            if (k13 < 0) k13 = (int)k;
            if ((int)k - k13 < 32) { tr[448 + k - k13] = clock64(); tr[544 + k - k13] = it.cur_st; }
        }
        if (tr && it.cur_st == 8) tr[316] = global_ns();
        if (!dead) {
            uint32_t total = 0;
            for (int i = 0; i < n; i++) total += seg[i].bytes;
            mbar_arrive_expect_tx(&S->full[s], total);
            uint8_t* d = ring + (size_t)s * kSlotBytes;
            for (int i = 0; i < n; i++) bulk_g2s(d + seg[i].off, seg[i].src, seg[i].bytes, &S->full[s], pol);
        }
        k++;
        *(volatile unsigned int*)&S->copied = k;
    }
    *(volatile unsigned int*)&S->copied = 0x7fffffffu;   // lets the prefetch warp finish
    P.chunk_count[2 * c] = (int)k;
}

__device__ __noinline__ void decode_prefetcher(const DecodeParams& P, DecodeSmem* S, const Plan& pl) {
    ChunkIter it;
    Seg seg[3];
    uint32_t npf = 0;
    const uint32_t lead = (uint32_t)P.prefetch_chunks;
    if (lead == 0) return;
    const uint64_t t0 = global_ns();
    for (;;) {
        const int n = it.next(P, pl, seg);
        if (n == 0) return;
        // stay at most `lead` chunks ahead of the producer (bounded: prefetching is optional)
        while (npf >= *(volatile unsigned int*)&S->copied + lead) {
            __nanosleep(256);
            if (global_ns() - t0 > 4 * kWaitNs) return;
        }
        for (int i = 0; i < n; i++) bulk_prefetch_l2(seg[i].src, seg[i].bytes);
        npf++;
    }
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
    uint32_t tag = 0;
    bool failed = false;    // this thread stopped waiting after an error
    unsigned long long* tr = nullptr;   // thread 0's trace row while tracing
    int tl = 0;                          // layer being traced (N_LAYERS = head)
    int k13 = -1;                        // first ring chunk of layer 13 (cycle trace)
    unsigned long long ring_ns = 0, xw_ns = 0;   // thread 0's waits in layer tl (written by flush)
    __device__ __forceinline__ void flush() {                    // stores only: no global read on the timed path
        if (tr) { tr[320 + tl] = ring_ns; tr[352 + tl] = xw_ns; }
        ring_ns = 0; xw_ns = 0;
    }

    uint32_t ns = kSlots;   // ring slots in use
    __device__ __forceinline__ const uint8_t* wait_chunk() {
        const uint32_t s = k % ns, ph = (k / ns) & 1u;
        const uint64_t t0 = tr ? global_ns() : 0;
        if (tr && tl == 13) { if (k13 < 0) k13 = (int)k; if ((int)k - k13 < 32) tr[480 + k - k13] = clock64(); }
        const bool ok = *(volatile int*)&S->abort || mbar_wait(&S->full[s], ph, 3 * kWaitNs);
        if (tr) ring_ns += global_ns() - t0;
        if (tr && tl == 13 && (int)k - k13 < 32) tr[512 + k - k13] = clock64();
        if (!ok) {
            *(volatile int*)&S->abort = 1;
            atomicOr(&P->out->err, 4u);
            atomicExch(&P->out->err_where, -100 - (int)s);
        }
        return ring + (size_t)s * kSlotBytes;
    }
    __device__ __forceinline__ void release_chunk() {
        __syncwarp();
        if (lane == 0) mbar_arrive(&S->empty[k % ns]);
        k++;
    }
    __device__ __forceinline__ void bar() { named_bar(1, kNCT); }

    // Gathers up to N word pairs: pair i (16-byte aligned, at addr(i)) for each i
    // whose bit is set in `mask`, into v[2i], v[2i+1].  A round loads every pair
    // at once; until all carry this launch's tag the thread spins on the first
    // stale pair only, then runs another round.  Once the last writer has stored,
    // the gather costs about one round trip whatever the number of words, and a
    // waiting CTA polls one pair per thread.
    template <int N, typename A>
    __device__ __forceinline__ void gather(A addr, uint32_t mask, float* v, int where) {
        uint64_t t0 = 0;
        uint32_t it = 0;
        while (!failed) {
            uint64_t a[N], b[N];
            #pragma unroll
            for (int i = 0; i < N; i++) if (mask & (1u << i)) xw_load2(addr(i), a[i], b[i]);
            int stale = -1;
            #pragma unroll
            for (int i = N - 1; i >= 0; i--)
                if ((mask & (1u << i)) && ((uint32_t)(a[i] >> 32) != tag || (uint32_t)(b[i] >> 32) != tag)) stale = i;
            if (stale < 0) {
                #pragma unroll
                for (int i = 0; i < N; i++) { v[2 * i] = __uint_as_float((uint32_t)a[i]); v[2 * i + 1] = __uint_as_float((uint32_t)b[i]); }
                if (tr && t0) xw_ns += global_ns() - t0;
                return;
            }
            if (t0 == 0) t0 = global_ns();
            const uint64_t* q = addr(stale);
            for (;;) {
                if (P->poll_ns) __nanosleep(P->poll_ns);
                uint64_t x, y;
                xw_load2(q, x, y);
                if ((uint32_t)(x >> 32) == tag && (uint32_t)(y >> 32) == tag) break;
                if ((++it & 31u) == 0) {
                    if (ld_volatile(&P->out->err)) { failed = true; break; }
                    if (global_ns() - t0 > kWaitNs) {
                        atomicOr(&P->out->err, 1u);
                        atomicExch(&P->out->err_where, where);
                        failed = true;
                        break;
                    }
                }
            }
        }
        #pragma unroll
        for (int i = 0; i < 2 * N; i++) v[i] = 0.f;   // after an error the values are never used for a result
    }
    __device__ __forceinline__ float block_sum(float v) {
        v = warp_sum(v);
        if (lane == 0) S->bred[0][warp] = v;
        bar();
        float t = 0.f;
        #pragma unroll
        for (int i = 0; i < kNCW; i++) t += S->bred[0][i];
        bar();
        return t;
    }
    // argmax over the block: largest value, ties to the smallest index
    __device__ __forceinline__ void block_argmax(float& v, int& i) {
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
    // RMSNorm of S->xres (sum of squares `ss`) with the bf16 gains at `gain` -> S->xs
    __device__ __forceinline__ void norm_into_xs(const uint16_t* gain, float ss) {
        const float r = 1.0f / sqrtf(ss * (1.0f / DIM) + EPS);
        const int j = tid * 2;
        const uint32_t w = *(const uint32_t*)(gain + j);
        S->xs[j] = (S->xres[j] * r) * bf_lo(w);
        S->xs[j + 1] = (S->xres[j + 1] * r) * bf_hi(w);
    }
    // lane's 32 fp32 values of a 1024-wide vector v: v[256 i + 8 lane + e]
    __device__ __forceinline__ void load_regs(const float* v, float* xr) {
        #pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 a = *(const float4*)&v[256 * i + 8 * lane];
            const float4 b = *(const float4*)&v[256 * i + 8 * lane + 4];
            xr[8 * i + 0] = a.x; xr[8 * i + 1] = a.y; xr[8 * i + 2] = a.z; xr[8 * i + 3] = a.w;
            xr[8 * i + 4] = b.x; xr[8 * i + 5] = b.y; xr[8 * i + 6] = b.z; xr[8 * i + 7] = b.w;
        }
    }
    // dot of a 1024-wide bf16 row segment in shared memory with xr (full warp)
    __device__ __forceinline__ float row_dot(const uint8_t* row, const float* xr) {
        const uint4* w = (const uint4*)row;
        float a = 0.f;
        #pragma unroll
        for (int i = 0; i < 4; i++) a = dot8(w[i * 32 + lane], &xr[8 * i], a);
        return warp_sum(a);
    }
    // rows [a, b) of 1024 columns, 16 per chunk, one row per warp; f(row, value) on lane 0
    template <typename F>
    __device__ __forceinline__ void rows_1024(int a, int b, const float* xr, F&& f) {
        for (int r = a; r < b; r += kRowsK1024) {
            const int n = min(kRowsK1024, b - r);
            const uint8_t* ch = wait_chunk();
            if (warp < n) {
                const float v = row_dot(ch + (size_t)warp * 2 * DIM, xr);
                if (lane == 0) f(r + warp, v);
            }
            release_chunk();
        }
    }
};

__device__ __forceinline__ void decode_consumer(const DecodeParams& P, uint8_t* ring, DecodeSmem* S, int c, int G, const Plan& pl,
                                             int token, int pos, int flags, uint32_t seq) {
    Consumer C;
    C.P = &P; C.ring = ring; C.S = S;
    C.tid = threadIdx.x; C.warp = C.tid >> 5; C.lane = C.tid & 31;
    C.tag = seq;
    C.ns = (uint32_t)P.ring_slots;
    const int tid = C.tid, warp = C.warp, lane = C.lane;
    if (P.trace && tid == 0) {
        C.tr = P.trace + (size_t)c * kTraceStride;
    }
    const int g = pl.g, gs = pl.gs, gr = pl.gr;
    const bool owner = (gr == gs - 1);                 // its position range ends at pos
    const float sqrt_hd = sqrtf((float)HEAD_DIM);
    unsigned long long* tr = (P.trace && tid == 0) ? P.trace + (size_t)c * kTraceStride : nullptr;
#define QB_TRACE(i) do { if (tr) tr[(i)] = global_ns(); } while (0)
#define QB_SUB(i) do { if (tr && l == 13) tr[384 + (i)] = clock64(); } while (0)   // cycles: exact within a CTA
    QB_TRACE(0);
    if (tr) tr[384 + 50] = clock64();

    if (tid < HEAD_DIM) S->rope[tid] = __ldg(P.rope + (size_t)pos * HEAD_DIM + tid);

    for (int l = 0; l < N_LAYERS; l++) {
        const int TB = 1 + 10 * l;
        C.flush();
        C.tl = l;
        // ---------------- QKV ----------------
        float ss;
        {
            const int j = tid * 2;
            float2 v;
            if (l == 0) {
                const uint32_t w = __ldg((const uint32_t*)(P.embed + (size_t)token * DIM + j));
                v = make_float2(bf_lo(w), bf_hi(w));
            } else {
                const uint64_t* p = P.xw + (size_t)l * DIM + j;
                float xv[2];
                C.gather<1>([&](int) { return p; }, 1u, xv, 10 * l);
                v.x = xv[0]; v.y = xv[1];
            }
            S->xres[j] = v.x; S->xres[j + 1] = v.y;
            ss = C.block_sum(v.x * v.x + v.y * v.y);
        }
        QB_TRACE(TB + 0);
        QB_SUB(31);
        {
            const uint8_t* ch = C.wait_chunk();
            QB_SUB(0);
            C.norm_into_xs((const uint16_t*)ch, ss);
            if (tid < HEAD_DIM) S->gq[tid] = bf2f(((const uint16_t*)(ch + 2 * DIM))[tid]);
            else if (tid < 2 * HEAD_DIM) S->gk[tid - HEAD_DIM] = bf2f(((const uint16_t*)(ch + 2 * DIM + 2 * HEAD_DIM))[tid - HEAD_DIM]);
            C.release_chunk();
        }
        C.bar();
        QB_SUB(1);
        {
            float xr[32];
            C.load_regs(S->xs, xr);
            C.rows_1024(pl.qa, pl.qb, xr, [&](int r, float v) { S->gv[r - pl.qa] = v; });
        }
        C.bar();
        if (tid < pl.qb - pl.qa)   // one exchange store per thread, all in flight together
            xw_store(P.qkvw + (size_t)l * 4096 + qkv_dst(g, pl.qa + tid), S->gv[tid], seq);
        QB_TRACE(TB + 1);
        QB_SUB(32);

        // ---------------- ATT ----------------
        if (warp < 4) {   // warp w: q head 2g (0), q head 2g+1 (1), k (2), v (3); lane holds dims 4l..4l+3
            const int off = warp < 2 ? 256 * g + 128 * warp : (warp == 2 ? Q_DIM + 128 * g : Q_DIM + KV_DIM + 128 * g);
            const uint64_t* p = P.qkvw + (size_t)l * 4096 + off + 4 * lane;
            float x[4];
            C.gather<2>([&](int i) { return p + 2 * i; }, 3u, x, 10 * l + 2);
            if (warp < 3) {
                const float tot = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
                const float r = 1.0f / sqrtf(tot * (1.0f / HEAD_DIM) + EPS);
                const float* gn = warp < 2 ? S->gq : S->gk;
                #pragma unroll
                for (int e = 0; e < 4; e++) x[e] = (x[e] * r) * gn[4 * lane + e];
                // NeoX rotation: dim d pairs with d ^ 64, held by lane ^ 16
                #pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float pv = __shfl_xor_sync(0xffffffffu, x[e], 16);
                    const int d = 4 * lane + e, j = d & 63;
                    const float cj = S->rope[j], sj = S->rope[64 + j];
                    x[e] = d < 64 ? (x[e] * cj - pv * sj) : (pv * sj + x[e] * cj);
                }
            }
            if (warp < 2) {
                #pragma unroll
                for (int e = 0; e < 4; e++) S->qs[128 * warp + 4 * lane + e] = x[e];
            } else if (owner) {
                uint16_t b[4];
                #pragma unroll
                for (int e = 0; e < 4; e++) b[e] = f2bf(x[e]);
                const size_t at = ((size_t)l * kGroups * SEQ_LEN * HEAD_DIM) + pl.kvbase + (size_t)pos * HEAD_DIM + 4 * lane;
                uint16_t* dst = (warp == 2 ? P.kc : P.vc) + at;
                *(uint2*)dst = make_uint2((uint32_t)b[0] | ((uint32_t)b[1] << 16), (uint32_t)b[2] | ((uint32_t)b[3] << 16));
                float* sm = warp == 2 ? S->kn : S->vn;
                #pragma unroll
                for (int e = 0; e < 4; e++) sm[4 * lane + e] = bf2f(b[e]);
            }
        }
        QB_SUB(3);
        C.bar();
        QB_TRACE(TB + 2);
        QB_SUB(33);
        {
            // warps 0-7: q head 2g; warps 8-15: q head 2g+1.  Each warp runs an
            // online softmax over positions hw, hw+8, ... of every K|V chunk.
            const int hh = warp >> 3, hw = warp & 7;
            float q[4];
            #pragma unroll
            for (int e = 0; e < 4; e++) q[e] = S->qs[128 * hh + 4 * lane + e];
            float m = -INFINITY, lsum = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
            auto visit = [&](float k0, float k1, float k2, float k3, float v0, float v1, float v2, float v3) {
                float s = q[0] * k0; s = fmaf(q[1], k1, s); s = fmaf(q[2], k2, s); s = fmaf(q[3], k3, s);
                s = warp_sum(s) / sqrt_hd;
                const float mn = fmaxf(m, s);
                const float sc = expf(m - mn), p = expf(s - mn);
                lsum = fmaf(lsum, sc, p);
                a0 = fmaf(a0, sc, p * v0); a1 = fmaf(a1, sc, p * v1); a2 = fmaf(a2, sc, p * v2); a3 = fmaf(a3, sc, p * v3);
                m = mn;
            };
            for (int t0 = pl.p0; t0 < pl.pe; t0 += kKVChunk) {
                const int cnt = min(kKVChunk, pl.pe - t0);
                const uint8_t* ch = C.wait_chunk();
                for (int i = hw; i < cnt; i += 8) {
                    const uint2 kw = *(const uint2*)(ch + (size_t)i * 2 * HEAD_DIM + 8 * lane);
                    const uint2 vw = *(const uint2*)(ch + kVOff + (size_t)i * 2 * HEAD_DIM + 8 * lane);
                    visit(bf_lo(kw.x), bf_hi(kw.x), bf_lo(kw.y), bf_hi(kw.y), bf_lo(vw.x), bf_hi(vw.x), bf_lo(vw.y), bf_hi(vw.y));
                }
                C.release_chunk();
            }
            QB_SUB(5);
            if (owner && hw == ((pos - pl.p0) & 7)) {
                const float4 kk = *(const float4*)&S->kn[4 * lane], vv = *(const float4*)&S->vn[4 * lane];
                visit(kk.x, kk.y, kk.z, kk.w, vv.x, vv.y, vv.z, vv.w);
            }
            // combine the 8 warps of each head
            *(float4*)&S->w.comb[(size_t)warp * HEAD_DIM + 4 * lane] = make_float4(a0, a1, a2, a3);
            if (lane == 0) { S->bred[0][warp] = m; S->bred[1][warp] = lsum; }
            C.bar();
            QB_SUB(6);
            if (tid < 2 * HEAD_DIM) {
                const int h2 = tid >> 7, d = tid & 127;
                float M = -INFINITY;
                #pragma unroll
                for (int w = 0; w < 8; w++) M = fmaxf(M, S->bred[0][8 * h2 + w]);
                float Ls = 0.f, A = 0.f;
                #pragma unroll
                for (int w = 0; w < 8; w++) {
                    const float mw = S->bred[0][8 * h2 + w];
                    const float sc = mw == -INFINITY ? 0.f : expf(mw - M);
                    Ls = fmaf(S->bred[1][8 * h2 + w], sc, Ls);
                    A = fmaf(S->w.comb[(size_t)(8 * h2 + w) * HEAD_DIM + d], sc, A);
                }
                uint64_t* base = P.partw + ((size_t)(l * kGroups + g) * kMaxGS + gr) * kPartStride + h2 * kHeadPart;
                xw_store(base + 4 + d, A, seq);
                if (d < 4) xw_store(base + d, d == 0 ? M : (d == 1 ? Ls : 0.f), seq);   // m, l and the two pads
            }
        }
        QB_SUB(7);
        C.bar();     // the combine above reads S->w.comb, which OPROJ reuses
        QB_TRACE(TB + 3);

        // ---------------- OPROJ ----------------
        {
            // stage the group's gs x 264 partial words in shared memory, spread over all threads
            const uint64_t* gbase = P.partw + (size_t)(l * kGroups + g) * kMaxGS * kPartStride;
            const int nw = gs * kPartStride;
            constexpr int kPer = (kMaxGS * kPartStride + 2 * kNCT - 1) / (2 * kNCT);
            uint32_t pend = 0;
            #pragma unroll
            for (int i = 0; i < kPer; i++) if (2 * tid + 2 * kNCT * i < nw) pend |= 1u << i;
            float v[2 * kPer];
            QB_SUB(8);
            C.gather<kPer>([&](int i) { return gbase + 2 * tid + 2 * kNCT * i; }, pend, v, 10 * l + 4);
            #pragma unroll
            for (int i = 0; i < kPer; i++) {
                if (pend & (1u << i)) *(float2*)&S->w.pst[2 * tid + 2 * kNCT * i] = make_float2(v[2 * i], v[2 * i + 1]);
            }
            QB_SUB(9);
        }
        C.bar();
        QB_TRACE(TB + 4);
        if (warp < 2) {   // warp hh: the combine weights of head hh, lane cc = chunk
            const int hh = warp;
            const float* b = &S->w.pst[lane * kPartStride + hh * kHeadPart];
            const bool live = lane < gs && b[1] > 0.f;
            const float m = live ? b[0] : -INFINITY;
            const float M = warp_max(m);
            const float e = live ? expf(m - M) : 0.f;
            const float den = warp_sum(live ? b[1] * e : 0.f);
            if (lane < kMaxGS) S->gv[hh * 32 + lane] = e / den;
        }
        C.bar();
        if (tid < 2 * HEAD_DIM) {
            const int hh = tid >> 7, d = tid & 127;
            float num = 0.f;
            for (int cc = 0; cc < gs; cc++) num = fmaf(S->w.pst[cc * kPartStride + hh * kHeadPart + 4 + d], S->gv[hh * 32 + cc], num);
            S->os[tid] = num;
        }
        QB_SUB(11);
        C.bar();
        QB_SUB(12);
        {
            float o8[8];
            #pragma unroll
            for (int e = 0; e < 8; e++) o8[e] = S->os[8 * lane + e];
            uint64_t* y = P.yw + (size_t)(l * kGroups + g) * DIM;
            for (int r = pl.oa; r < pl.ob; r += kRowsWo) {
                const int cnt = min(kRowsWo, pl.ob - r);
                const uint8_t* ch = C.wait_chunk();
                QB_SUB(13);
                for (int i = warp; i < cnt; i += kNCW) {
                    const uint4 w = ((const uint4*)(ch + (size_t)i * 512))[lane];
                    const float a = warp_sum(dot8(w, o8, 0.f));
                    if (lane == 0) S->w.hs[r - pl.oa + i] = a;
                }
                QB_SUB(14);
                C.release_chunk();
            }
            C.bar();
            if (tid < pl.ob - pl.oa) xw_store(y + pl.oa + tid, S->w.hs[tid], seq);
        }
        QB_TRACE(TB + 5);

        // ---------------- MLP-A ----------------
        {
            const int j = tid * 2;
            const uint64_t* yb = P.yw + (size_t)l * kGroups * DIM + j;
            QB_SUB(16);
            float x0 = S->xres[j], x1 = S->xres[j + 1];
            {
                float yv[2 * kGroups];
                C.gather<kGroups>([&](int gg) { return yb + (size_t)gg * DIM; }, (1u << kGroups) - 1u, yv, 10 * l + 6);
                #pragma unroll
                for (int gg = 0; gg < kGroups; gg++) { x0 += yv[2 * gg]; x1 += yv[2 * gg + 1]; }
            }
            QB_SUB(17);
            S->xres[j] = x0; S->xres[j + 1] = x1;
            ss = C.block_sum(x0 * x0 + x1 * x1);
        }
        QB_TRACE(TB + 6);
        QB_SUB(34);
        {
            const uint8_t* ch = C.wait_chunk();
            C.norm_into_xs((const uint16_t*)ch, ss);
            C.release_chunk();
        }
        C.bar();
        {
            float xr[32];
            C.load_regs(S->xs, xr);
            QB_SUB(20);
            C.rows_1024(pl.ha, pl.hb, xr, [&](int r, float v) { S->gv[r - pl.ha] = v; });
            QB_SUB(21);
            C.rows_1024(pl.ha, pl.hb, xr, [&](int r, float v) { S->uv[r - pl.ha] = v; });
            QB_SUB(22);
        }
        C.bar();
        if (tid < pl.hb - pl.ha) {
            const float gt = S->gv[tid];
            xw_store(P.hw + (size_t)l * HIDDEN_DIM + pl.ha + tid, (gt / (1.0f + expf(-gt))) * S->uv[tid], seq);
        }
        QB_TRACE(TB + 7);
        QB_SUB(35);

        // ---------------- MLP-B ----------------
        {
            const uint64_t* hb = P.hw + (size_t)l * HIDDEN_DIM + 2 * tid;
            constexpr int kHP = HIDDEN_DIM / (2 * kNCT);
            float hv[2 * kHP];
            QB_SUB(25);
            C.gather<kHP>([&](int i) { return hb + 2 * kNCT * i; }, (1u << kHP) - 1u, hv, 10 * l + 8);
            #pragma unroll
            for (int i = 0; i < kHP; i++) *(float2*)&S->w.hs[2 * tid + 2 * kNCT * i] = make_float2(hv[2 * i], hv[2 * i + 1]);
        }
        C.bar();
        QB_TRACE(TB + 8);
        const long long cy0 = clock64();
        {
            // warp -> (row rw of the chunk, 1024-column segment sg); 5 rows x 3 segments
            const int rw = warp / 3, sg = warp % 3;
            float xr[32];
            C.load_regs(S->w.hs + 1024 * sg, xr);
            if (tr && l == 13) tr[384 + 40] = clock64() - cy0;
            uint64_t* xn = P.xw + (size_t)(l + 1) * DIM;
            for (int r = pl.da; r < pl.db; r += kRowsK3072) {
                const int n = min(kRowsK3072, pl.db - r);
                const uint8_t* ch = C.wait_chunk();
                if (tr && l == 13 && r == pl.da) tr[384 + 41] = clock64() - cy0;
                QB_SUB(28);
                if (rw < n) {
                    const float v = C.row_dot(ch + (size_t)rw * 2 * HIDDEN_DIM + (size_t)sg * 2 * 1024, xr);
                    if (lane == 0) S->part[warp] = v;
                }
                QB_SUB(29);
                if (tr && l == 13 && r == pl.da) tr[384 + 42] = clock64() - cy0;
                C.release_chunk();
                C.bar();
                if (tr && l == 13 && r == pl.da) tr[384 + 43] = clock64() - cy0;
                QB_SUB(30);
                if (tid < n) {
                    const float v = S->xres[r + tid] + ((S->part[3 * tid] + S->part[3 * tid + 1]) + S->part[3 * tid + 2]);
                    xw_store(xn + r + tid, v, seq);
                }
                C.bar();
            }
        }
        C.bar();     // S->w.hs and S->xres are reused by the next layer
        QB_TRACE(TB + 9);
        QB_SUB(36);
    }

    // ---------------- HEAD ----------------
    C.flush();
    C.tl = N_LAYERS;
    const bool head = pl.head;
    const bool greedy = (P.in->temperature == 0.0f || P.in->top_k == 1);
    const int K = greedy ? 1 : min(P.in->top_k, kMaxCand);
    if (head) {
        float ss;
        {
            const int j = tid * 2;
            const uint64_t* p = P.xw + (size_t)N_LAYERS * DIM + j;
            float xv[2];
            C.gather<1>([&](int) { return p; }, 1u, xv, 10 * N_LAYERS);
            const float x0 = xv[0], x1 = xv[1];
            S->xres[j] = x0; S->xres[j + 1] = x1;
            ss = C.block_sum(x0 * x0 + x1 * x1);
        }
        QB_TRACE(kTrHead);
        {
            const uint8_t* ch = C.wait_chunk();
            C.norm_into_xs((const uint16_t*)ch, ss);
            C.release_chunk();
        }
        C.bar();
        const int va = pl.va;
        const bool wl = (flags & kFlagWriteLogits) != 0;
        {
            float xr[32];
            C.load_regs(S->xs, xr);
            C.rows_1024(pl.va, pl.vb, xr, [&](int r, float v) {
                S->w.lg[r - va] = v;
                if (wl) P.logits[r] = v;
            });
        }
        C.bar();
        const int nloc = pl.vb - pl.va;
        for (int kk = 0; kk < K; kk++) {
            float v = -INFINITY; int i = 0x7fffffff;
            for (int t = tid; t < nloc; t += kNCT) better(v, i, S->w.lg[t], t);
            C.block_argmax(v, i);
            if (tid == 0) {
                P.cand_v[(size_t)c * kMaxCand + kk] = v;
                P.cand_i[(size_t)c * kMaxCand + kk] = (i < nloc) ? va + i : 0x7fffffff;
                if (i < nloc) S->w.lg[i] = -INFINITY;
            }
            C.bar();
        }
    }
    QB_TRACE(kTrHead + 1);
    if (tr) tr[384 + 51] = clock64();
    C.flush();
    // last CTA to arrive merges and samples
    C.bar();
    if (tid == 0) {
        P.chunk_count[2 * c + 1] = (int)C.k;
        __threadfence();
        const uint32_t old = atom_acq_rel_add(P.ctr, 1u);
        S->flag = (old == (uint32_t)G - 1u) ? 1 : 0;
    }
    C.bar();
    QB_TRACE(kTrHead + 2);
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
                S->gv[kk] = bv;
                ((int*)S->uv)[kk] = bi;
                if (ba >= 0) { cv[ba] = -INFINITY; ci[ba] = 0x7fffffff; }
            }
            C.bar();
        }
        if (tid == 0) {
            const int* ids = (const int*)S->uv;
            float* prob = S->w.hs;
            unsigned long long rng = P.in->rng;
            if (greedy) {
                tok = ids[0];
            } else {
                // sampler.h:137-174 over the K candidates, scanned in descending order
                const float T = P.in->temperature, topp = P.in->topp;
                int nc = K;
                const float mx = S->gv[0];
                float sum = 0.f;
                for (int i = 0; i < nc; i++) { const float e = expf((S->gv[i] - mx) / T); prob[i] = e; sum += e; }
                for (int i = 0; i < nc; i++) prob[i] /= sum;
                if (topp > 0.0f && topp < 1.0f) {
                    float cum = 0.f; int last = nc - 1;
                    for (int i = 0; i < nc; i++) { cum += prob[i]; if (cum > topp) { last = i; break; } }
                    nc = last + 1; sum = cum;
                }
                rng ^= rng >> 12; rng ^= rng << 25; rng ^= rng >> 27;
                const uint32_t u = (uint32_t)((rng * 0x2545F4914F6CDD1Dull) >> 32);
                const float coin = ((float)(u >> 8) / 16777216.0f) * sum;
                float cdf = 0.f;
                tok = ids[nc - 1];
                for (int i = 0; i < nc; i++) { cdf += prob[i]; if (coin < cdf) { tok = ids[i]; break; } }
            }
            if (tok < 0 || tok >= VOCAB_SIZE) {   // no finite candidate (NaN logits): report, never hand on
                atomicOr(&P.out->err, 16u);
                atomicExch(&P.out->err_where, -201);
                tok = 0;
            }
            P.in->rng = rng;
            P.out->rng = rng;
        }
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
        P.ctr[0] = 0;                 // every CTA has arrived: reset for the next launch
        __threadfence();
        P.out->seq = seq + 1;
    }
    QB_TRACE(kTrHead + 3);
#undef QB_TRACE
#undef QB_SUB
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeParams P) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    DecodeSmem* S = reinterpret_cast<DecodeSmem*>(smem + (size_t)kSlots * kSlotBytes);
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int s = 0; s < kSlots; s++) { mbar_init(&S->full[s], 1); mbar_init(&S->empty[s], kNCW); }
        S->abort = 0;
        S->copied = 0;
        fence_barrier_init();
    }
    __syncthreads();
    const int c = blockIdx.x, G = gridDim.x;
    const int flags = P.in->flags;
    const int pos = min(max(P.in->pos, 0), SEQ_LEN - 1);   // the host validates; never index past the cache
    int token = (flags & kFlagPromptToken) ? P.prompt[pos] : P.in->token;
    if (token < 0 || token >= VOCAB_SIZE) {                 // e.g. a chained step after NaN logits
        if (tid == 0 && c == 0) { atomicOr(&P.out->err, 8u); atomicExch(&P.out->err_where, -200); }
        token = 0;
    }
    const uint32_t seq = P.out->seq;
    if (tid == 0) S->pl = make_plan(P, c, G, pos, flags);
    __syncthreads();
    const Plan& pl = S->pl;
    if ((tid >> 5) == kNCW) {
        if ((tid & 31) == 0) decode_producer(P, ring, S, c, pl);
        return;
    }
    if ((tid >> 5) == kNCW + 1) {
        if ((tid & 31) == 0) decode_prefetcher(P, S, pl);
        return;
    }
    decode_consumer(P, ring, S, c, G, pl, token, pos, flags, seq);
}

}  // namespace qb
