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
// prefetches further ahead.  The stream never waits on activations, so the
// slots of the next stages are full while a CTA waits on another CTA.
// Sixteen consumer warps compute from the slots, two chunks at a time, so
// every warp has two or more independent rows in flight.
//
// Activation exchange.  Every value one CTA hands to another is an 8-byte word
// (fp32 value | 32-bit sequence tag) written with one relaxed 64-bit store;
// a reader loads the words it needs in 16-byte pairs, all at once, and polls
// until every tag equals this launch's sequence number.  No fences, no
// counters: a hop costs about one L2 round trip after the last writer.  Per
// layer l (the 8 KV heads define 8 CTA groups of ~G/8 CTAs):
//
//   QKV   group g: x_l -> RMSNorm (input_layernorm, folded into each lane's
//         registers) -> its rows of the group's 512 projection rows (q heads
//         2g, 2g+1; k, v head g)                                     -> qkv
//   ATT   group g: QK-norm + RoPE of q/k; the CTA whose positions end at pos
//         appends bf16 K/V; split-K attention over its share of positions:
//         four lanes per (head, position) score, one online softmax per warp
//                                                                -> partials
//   OPROJ group g: combine the group's partials -> o (256 values) -> its rows
//         of Wo[:, 256g:256g+256] (packed contiguous)             -> y[g]
//   MLP-A all: x_mid = x_l + sum_g y[g] (fixed order); RMSNorm
//         (post_attention_layernorm) -> its gate/up rows (one warp per
//         hidden unit) -> SwiGLU                                   -> h
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
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "../host/config.h"

namespace qb {

constexpr int kNCW = 16;                    // consumer warps
constexpr int kNCT = kNCW * 32;             // consumer threads
constexpr int kThreads = kNCT + 64;         // + one producer warp + one L2-prefetch warp
constexpr int kSlots = 5;
constexpr int kSlotBytes = 32768;
constexpr int kGroups = N_KV_HEADS;         // one CTA group per KV head
constexpr int kMaxGS = 19;                  // max CTAs per group (grid <= 152)
constexpr int kMinGS = 8;                   // min CTAs per group (grid >= 64)
constexpr int kMaxCand = 64;                // device top-k limit
constexpr int kHeadPart = 4 + HEAD_DIM;     // m, l, pad, pad, acc[128]
constexpr int kPartStride = 2 * kHeadPart;  // both q heads of a group
constexpr int kMaxLocalRows = 2048;         // LM-head rows per CTA at most
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
constexpr int kFlagCandidatesOnly = 8; // leave the shard's top-K in top_v / top_i; shard_merge_kernel picks the token

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
    const uint16_t* wo_g;    // [L][8][DIM][kWoCols]  Wo columns of group g, row-major, padded
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
    unsigned long long wait_ns;  // limit of each wait on another CTA's values (kWaitNs; shorter for failure tests)
    int debug_skip;          // >= 0: the CTAs of this KV-head group withhold their layer-0 q|k|v (failure tests)
    int prefetch_chunks;     // L2 prefetch lead of the producer, in chunks (0 = none)
    int poll_ns;             // back-off between polls of an exchange word
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

// B-operand fragments of an activation vector v for mma.m16n8k16: v is split
// into three bf16 parts (v = hi + mid + lo to fp32 precision) in columns 0, 1
// and 2; columns 3..7 are zero.  frag[kt][lane][reg] for k-tile kt and lanes
// 0..11 (the only lanes whose B registers are nonzero).
constexpr int kFragLanes = 12;
struct __align__(16) DecodeSmem {
    uint64_t full[kSlots];
    uint64_t empty[kSlots];
    alignas(16) float xres[DIM];         // layer input x_l, then x_mid
    alignas(16) union {                  // one stage at a time (a barrier separates users)
        uint32_t bh[HIDDEN_DIM / 16][kFragLanes][2];   // MLP-B: fragments of h
        float comb[kNCW * HEAD_DIM];          // ATT: per-warp accumulators
        float pst[kMaxGS * kPartStride];      // OPROJ: the group's partials
        float lg[kMaxLocalRows];              // HEAD: local logits; merge: probabilities
    } w;
    alignas(16) uint32_t bx[DIM / 16][kFragLanes][2];          // fragments of the RMSNorm output in use (HEAD: the fp32 output)
    alignas(16) uint32_t bo[2 * HEAD_DIM / 16][kFragLanes][2]; // fragments of the group's attention output
    alignas(16) float red[2][kNCW][32];  // per-warp MMA partial sums (two 16-row tiles), two buffers used alternately
    alignas(16) float qs[2 * HEAD_DIM];  // the group's two q heads (normed, rotated)
    alignas(16) float kn[HEAD_DIM];      // the new position's k and v (bf16-rounded)
    alignas(16) float vn[HEAD_DIM];
    alignas(16) float rope[HEAD_DIM];    // cos | sin of this position
    float bsum[2][kNCW];     // block sums, two buffers used alternately
    float am[kNCW], al[kNCW];   // ATT: per-warp running max and sum
    float av[kNCW];          // block argmax
    int ai[kNCW];
    float tv[kMaxCand];      // merged top-K (head)
    int ti[kMaxCand];
    int flag;
    int abort;               // set after a ring wait expired: stop waiting on the ring
    unsigned int copied;     // chunks the producer has issued (read by the prefetch warp)
    Plan pl;                 // this CTA's share of every stage (one copy, in shared memory)
};
// every array read or written with 8- or 16-byte vector accesses starts on a 16-byte boundary
static_assert(sizeof(DecodeSmem::bx) >= DIM * sizeof(float), "the head keeps its fp32 RMSNorm output in bx");
static_assert(offsetof(DecodeSmem, xres) % 16 == 0 && offsetof(DecodeSmem, w) % 16 == 0 &&
              offsetof(DecodeSmem, qs) % 16 == 0 && offsetof(DecodeSmem, kn) % 16 == 0 &&
              offsetof(DecodeSmem, vn) % 16 == 0 && offsetof(DecodeSmem, bx) % 16 == 0 &&
              offsetof(DecodeSmem, bo) % 16 == 0 && offsetof(DecodeSmem, red) % 16 == 0,
              "shared-memory arrays must be 16-byte aligned");
static_assert((kSlots * kSlotBytes) % 16 == 0, "the ring keeps DecodeSmem 16-byte aligned");
constexpr size_t kDecodeSmemBytes = (size_t)kSlots * kSlotBytes + sizeof(DecodeSmem);
static_assert(kDecodeSmemBytes <= 227 * 1024, "one CTA per SM: at most 227 KB of shared memory");

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
//   per layer: [QKV rows, 15/chunk]
//              [K | V of cached positions, 64/chunk: K at 0, V at 16 KB]
//              [Wo_g rows (packed, padded), 62/chunk]
//              [gate|up units, 7/chunk: gate rows 0..6, up rows 7..13]
//              [Wd rows (3072 wide), 4/chunk]
//   then (unless kFlagNoHead): [LM-head rows, 16/chunk, one bulk copy]
// Layer weight rows land kPad bytes apart beyond their length (one bulk copy
// per row), the layout the tensor-core tiles read conflict-free.  The LM head
// is pure streaming (no hop, 2.1 MB per CTA): its rows stay contiguous and are
// dotted on the FP32 pipe.
// RMSNorm gains are not streamed: every lane loads the few it needs from L2.
// The producer walks the sequence twice (an L2-prefetch cursor ahead of the
// copy cursor); the consumers' code visits the same chunks in the same order.
// ---------------------------------------------------------------------------
// Weight rows land in a slot 16 bytes apart beyond their length, so the eight
// rows an ldmatrix reads start in eight different bank groups.
constexpr int kPad = 16;
constexpr int kStride1024 = 2 * DIM + kPad;                // 2064 B per 1024-wide row
constexpr int kRowsK1024 = kSlotBytes / kStride1024;       // 15 rows per chunk
constexpr int kUnitsGU = 7;                                // gate rows 0..6, up rows 7..13 of a chunk
constexpr int kStrideWd = 2 * HIDDEN_DIM + kPad;           // 6160 B per Wd row
constexpr int kRowsWd = 4;                                 // Wd rows per chunk
constexpr int kWoCols = 256 + kPad / 2;                    // packed Wo row, padded in HBM
constexpr int kStrideWo = 2 * kWoCols;                     // 528 B
constexpr int kRowsWo = kSlotBytes / kStrideWo;            // 62 rows per chunk
constexpr int kRowsLM = kSlotBytes / (2 * DIM);            // 16 LM-head rows per chunk (unpadded: FFMA path)
constexpr int kKVChunk = 64;                               // positions per K|V chunk
constexpr int kVOff = kKVChunk * 2 * HEAD_DIM;             // V offset in a K|V chunk
static_assert(2 * kUnitsGU * kStride1024 <= kSlotBytes && kRowsWd * kStrideWd <= kSlotBytes, "chunks fit a slot");

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

struct Seg {            // `rows` copies of `bytes` each: source rows src_stride apart, slot rows dst_stride apart
    const uint8_t* src;
    uint32_t bytes;
    uint32_t off;      // destination offset of the first row inside the slot
    uint32_t rows;
    uint32_t src_stride;
    uint32_t dst_stride;
};

struct ChunkIter {
    int l = 0, st = 0, r = 0;
    int cur_st = 0, cur_l = 0;   // stage and layer of the chunk last returned
    // Fills seg[] with the next chunk's copies; returns their count (0 at the end).
    __device__ int next(const DecodeParams& P, const Plan& pl, Seg* seg) {
        for (;;) {
            cur_st = st; cur_l = l;
            switch (st) {
            case 0:
                st = 1; r = pl.qa;
                break;
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
                        seg[k++] = {(const uint8_t*)src, (uint32_t)(2 * DIM), (uint32_t)(i * kStride1024), (uint32_t)m,
                                    (uint32_t)(2 * DIM), (uint32_t)kStride1024};
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
                    seg[0] = {(const uint8_t*)(P.kc + e), (uint32_t)(n * 2 * HEAD_DIM), 0, 1, 0, 0};
                    seg[1] = {(const uint8_t*)(P.vc + e), (uint32_t)(n * 2 * HEAD_DIM), (uint32_t)kVOff, 1, 0, 0};
                    r += n;
                    return 2;
                }
                st = 3; r = pl.oa;
                break;
            case 3:
                if (r < pl.ob) {
                    const int n = min(kRowsWo, pl.ob - r);
                    seg[0] = {(const uint8_t*)(P.wo_g + ((size_t)(l * kGroups + pl.g) * DIM + r) * kWoCols), (uint32_t)(n * kStrideWo), 0,
                              1, 0, 0};
                    r += n;
                    return 1;
                }
                st = 5; r = pl.ha;
                break;
            case 5:
                if (r < pl.hb) {
                    const int n = min(kUnitsGU, pl.hb - r);
                    seg[0] = {(const uint8_t*)(P.wg[l] + (size_t)r * DIM), (uint32_t)(2 * DIM), 0, (uint32_t)n,
                              (uint32_t)(2 * DIM), (uint32_t)kStride1024};
                    seg[1] = {(const uint8_t*)(P.wu[l] + (size_t)r * DIM), (uint32_t)(2 * DIM), (uint32_t)(kUnitsGU * kStride1024),
                              (uint32_t)n, (uint32_t)(2 * DIM), (uint32_t)kStride1024};
                    r += n;
                    return 2;
                }
                st = 7; r = pl.da;
                break;
            case 7:
                if (r < pl.db) {
                    const int n = min(kRowsWd, pl.db - r);
                    seg[0] = {(const uint8_t*)(P.wd[l] + (size_t)r * HIDDEN_DIM), (uint32_t)(2 * HIDDEN_DIM), 0, (uint32_t)n,
                              (uint32_t)(2 * HIDDEN_DIM), (uint32_t)kStrideWd};
                    r += n;
                    return 1;
                }
                if (++l < N_LAYERS) { st = 0; break; }
                st = pl.head ? 9 : 10; r = pl.va;
                break;
            case 9:
                if (r < pl.vb) {
                    const int n = min(kRowsLM, pl.vb - r);
                    seg[0] = {(const uint8_t*)(P.lm + (size_t)r * DIM), (uint32_t)(n * 2 * DIM), 0, 1, 0, 0};
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
template <bool kTr>
__device__ __noinline__ void decode_producer(const DecodeParams& P, uint8_t* ring, DecodeSmem* S, int c, const Plan& pl) {
    const uint64_t pol = policy_evict_first();
    unsigned long long* tr = (kTr && P.trace) ? P.trace + (size_t)c * kTraceStride : nullptr;
    ChunkIter it;
    Seg seg[3];
    uint32_t k = 0;
    int k13 = -1, last_l = -1;
    bool dead = false, head_seen = false;
    for (;;) {
        const int n = it.next(P, pl, seg);
        if (n == 0) break;
        const uint32_t s = k % kSlots, ph = (k / kSlots) & 1u;
        if (!dead && !mbar_wait(&S->empty[s], ph ^ 1u, 2 * kWaitNs)) {
            atomicOr(&P.out->err, 2u);
            atomicExch(&P.out->err_where, -1 - (int)s);
            dead = true;   // issue nothing more; consumers stop waiting after their own timeout
        }
        if (tr && it.cur_st <= 7 && it.cur_l != last_l) { tr[288 + it.cur_l] = global_ns(); last_l = it.cur_l; }
        if (tr && it.cur_l == 13 && it.cur_st <= 7) {   // layer 13's chunks: issue cycle and stage
            if (k13 < 0) k13 = (int)k;
            if ((int)k - k13 < 32) { tr[448 + k - k13] = clock64(); tr[544 + k - k13] = it.cur_st; }
        }
        if (tr && it.cur_st == 9 && !head_seen) { tr[316] = global_ns(); head_seen = true; }
        if (!dead) {
            uint32_t total = 0;
            for (int i = 0; i < n; i++) total += seg[i].bytes * seg[i].rows;
            mbar_arrive_expect_tx(&S->full[s], total);
            uint8_t* d = ring + (size_t)s * kSlotBytes;
            for (int i = 0; i < n; i++)
                for (uint32_t r = 0; r < seg[i].rows; r++)
                    bulk_g2s(d + seg[i].off + r * seg[i].dst_stride, seg[i].src + (size_t)r * seg[i].src_stride, seg[i].bytes,
                             &S->full[s], pol);
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
        for (int i = 0; i < n; i++)
            for (uint32_t r = 0; r < seg[i].rows; r++) bulk_prefetch_l2(seg[i].src + (size_t)r * seg[i].src_stride, seg[i].bytes);
        npf++;
    }
}

// ---------------------------------------------------------------------------
// Consumers
// ---------------------------------------------------------------------------
template <bool kTr>
struct Consumer {
    const DecodeParams* P;
    uint8_t* ring;
    DecodeSmem* S;
    int tid, warp, lane;
    uint32_t k = 0;          // first ring chunk not yet released by this warp
    uint32_t tag = 0;
    uint32_t bsp = 0;        // block_sum buffer parity
    bool failed = false;     // this thread stopped waiting after an error
    unsigned long long* tr = nullptr;   // thread 0's trace row while tracing
    int tl = 0;                          // layer being traced (N_LAYERS = head)
    int k13 = -1;                        // first ring chunk of layer 13 (cycle trace)
    unsigned long long ring_ns = 0, xw_ns = 0;   // thread 0's waits in layer tl (written by flush)
    __device__ __forceinline__ void flush() {                    // stores only: no global read on the timed path
        if (kTr && tr) { tr[320 + tl] = ring_ns; tr[352 + tl] = xw_ns; }
        ring_ns = 0; xw_ns = 0;
    }

    // Ring chunk k + i (i < kSlots), once it has landed.  Every warp takes every
    // chunk in order and releases it after use; a warp may hold two at once.
    __device__ __forceinline__ const uint8_t* chunk(uint32_t i) {
        const uint32_t kk = k + i;
        const uint32_t s = kk % kSlots, ph = (kk / kSlots) & 1u;
        const uint64_t t0 = kTr && tr ? global_ns() : 0;
        if (kTr && tr && tl == 13) { if (k13 < 0) k13 = (int)kk; if ((int)kk - k13 < 32) tr[480 + kk - k13] = clock64(); }
        const bool ok = *(volatile int*)&S->abort || mbar_wait(&S->full[s], ph, 3 * kWaitNs);
        if (kTr && tr) ring_ns += global_ns() - t0;
        if (kTr && tr && tl == 13 && (int)kk - k13 < 32) tr[512 + kk - k13] = clock64();
        if (!ok) {
            *(volatile int*)&S->abort = 1;
            atomicOr(&P->out->err, 4u);
            atomicExch(&P->out->err_where, -100 - (int)s);
        }
        return ring + (size_t)s * kSlotBytes;
    }
    __device__ __forceinline__ void release(uint32_t n) {
        __syncwarp();
        if (lane == 0)
            for (uint32_t i = 0; i < n; i++) mbar_arrive(&S->empty[(k + i) % kSlots]);
        k += n;
    }
    __device__ __forceinline__ void bar() { named_bar(1, kNCT); }

    // Gathers up to N word pairs: pair i (16-byte aligned, at addr(i)) for each i
    // whose bit is set in `mask`, into v[2i], v[2i+1].  Called by whole warps.
    // A round loads every pair of every lane at once; while any carries an old
    // tag the warp runs another round, so the last store is seen one round trip
    // after it lands.  (Every gather here is at most 8 pairs per lane; letting
    // one lane spin on a stale pair between rounds measured 2.5 % slower.)
    template <int N, typename A>
    __device__ __forceinline__ void gather(A addr, uint32_t mask, float* v, int where) {
        static_assert(N >= 1 && N <= 8, "gathers poll by full rounds of at most 8 pairs per lane");
        uint64_t t0 = 0;
        uint32_t it = 0;
        while (!failed) {
            uint64_t a[N], b[N];
            #pragma unroll
            for (int i = 0; i < N; i++) if (mask & (1u << i)) xw_load2(addr(i), a[i], b[i]);
            int stale = -1;   // (an index, not a flag: the flag form costs spills at 96 registers)
            #pragma unroll
            for (int i = N - 1; i >= 0; i--)
                if ((mask & (1u << i)) && ((uint32_t)(a[i] >> 32) != tag || (uint32_t)(b[i] >> 32) != tag)) stale = i;
            if (__ballot_sync(0xffffffffu, stale >= 0) == 0u) {
                #pragma unroll
                for (int i = 0; i < N; i++) { v[2 * i] = __uint_as_float((uint32_t)a[i]); v[2 * i + 1] = __uint_as_float((uint32_t)b[i]); }
                if (kTr && tr && t0) xw_ns += global_ns() - t0;
                return;
            }
            if (t0 == 0) t0 = global_ns();
            if (P->poll_ns) __nanosleep(P->poll_ns);
            if ((++it & 31u) == 0) {
                if (ld_volatile(&P->out->err)) failed = true;
                else if (global_ns() - t0 > P->wait_ns) {
                    atomicOr(&P->out->err, 1u);
                    atomicExch(&P->out->err_where, where);
                    failed = true;
                }
            }
            failed = __any_sync(0xffffffffu, failed);
        }
        #pragma unroll
        for (int i = 0; i < 2 * N; i++) v[i] = 0.f;   // after an error the values are never used for a result
    }
    // Sum over the 512 consumer threads.  One barrier: consecutive calls use
    // alternate buffers, and a call's buffer is not written again before every
    // thread has passed the next call's barrier.
    __device__ __forceinline__ float block_sum(float v) {
        v = warp_sum(v);
        float* b = S->bsum[bsp];
        bsp ^= 1u;
        if (lane == 0) b[warp] = v;
        bar();
        float t = 0.f;
        #pragma unroll
        for (int i = 0; i < kNCW; i++) t += b[i];
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
        if (lane == 0) { S->av[warp] = v; S->ai[warp] = i; }
        bar();
        v = S->av[0]; i = S->ai[0];
        #pragma unroll
        for (int w = 1; w < kNCW; w++) better(v, i, S->av[w], S->ai[w]);
        bar();
    }
    __device__ __forceinline__ uint32_t gain_fetch(const uint16_t* g) { return __ldg((const uint32_t*)(g + 2 * tid)); }
    // Writes the B fragments of elements k, k+1 (k even) of a vector: the
    // bf16 high parts to lanes 0..3, the next bf16 parts to lanes 4..7 and the
    // last to lanes 8..11 (each subtraction is exact in fp32).
    __device__ __forceinline__ void put_pair(uint32_t* frag, int k, float v0, float v1) {
        const int kt = k >> 4, w = k & 15, q = (w & 7) >> 1, reg = w >> 3;
        const uint16_t h0 = f2bf(v0), h1 = f2bf(v1);
        const float r0 = v0 - bf2f(h0), r1 = v1 - bf2f(h1);
        const uint16_t m0 = f2bf(r0), m1 = f2bf(r1);
        const uint16_t l0 = f2bf(r0 - bf2f(m0)), l1 = f2bf(r1 - bf2f(m1));
        uint32_t* f = frag + (kt * kFragLanes + q) * 2 + reg;
        f[0] = (uint32_t)h0 | ((uint32_t)h1 << 16);
        f[8] = (uint32_t)m0 | ((uint32_t)m1 << 16);    // lane q + 4
        f[16] = (uint32_t)l0 | ((uint32_t)l1 << 16);   // lane q + 8
    }
    // RMSNorm input of a projection, for the 1024-wide x whose pair 2 tid,
    // 2 tid + 1 this thread holds (x0, x1; g2 = its two bf16 gains): writes the
    // fragments S->bx of g * x and returns 1 / rms(x) once the block's sum of
    // squares is in — one barrier for both.  The projections are linear, so
    // their row results are scaled by the returned factor instead of the
    // input: W (g * x / rms) = (W (g * x)) / rms.
    __device__ __forceinline__ float gain_bx(float x0, float x1, uint32_t g2) {
        put_pair(&S->bx[0][0][0], 2 * tid, x0 * bf_lo(g2), x1 * bf_hi(g2));
        const float ss = block_sum(x0 * x0 + x1 * x1);
        return 1.0f / sqrtf(ss * (1.0f / DIM) + EPS);
    }
    // Row tile x k-tile products on the tensor cores (mma.m16n8k16, bf16 in,
    // fp32 accumulate): ta[t] = this lane's ldmatrix address (shared space) of
    // tile t at k-tile 0 — row lane % 16, 16-byte half lane / 16 — and bfr the
    // fragments.  Accumulates k-tiles [kt0, kt0 + nkt) into d[t].
    template <int NT>
    __device__ __forceinline__ void mma_tiles(const uint32_t (&ta)[NT], const uint32_t* bfr, int kt0, int nkt, float (&d)[NT][4]) {
        #pragma unroll 4
        for (int kt = kt0; kt < kt0 + nkt; kt++) {
            uint32_t b0 = 0u, b1 = 0u;
            if (lane < kFragLanes) { const uint2 b = *(const uint2*)&bfr[(kt * kFragLanes + lane) * 2]; b0 = b.x; b1 = b.y; }
            #pragma unroll
            for (int t = 0; t < NT; t++) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(ta[t] + kt * 32, a0, a1, a2, a3);
                mma_bf16_16816(d[t], a0, a1, a2, a3, b0, b1);
            }
        }
    }
    // This warp's 16-row partial sums of tile t (d = its accumulator) into
    // red[warp][16 t ..]: columns 0 + 1 + 2 = the dot with v's three parts;
    // lane 4g holds columns 0, 1 and lane 4g + 1 column 2 of rows g and g + 8.
    __device__ __forceinline__ void put_red(float* red, int t, const float (&d)[4]) {
        const float c2a = __shfl_down_sync(0xffffffffu, d[0], 1), c2b = __shfl_down_sync(0xffffffffu, d[2], 1);
        if ((lane & 3) == 0) {
            const int r = lane >> 2;
            red[warp * 32 + 16 * t + r] = (d[0] + d[1]) + c2a;
            red[warp * 32 + 16 * t + r + 8] = (d[2] + d[3]) + c2b;
        }
    }
    uint32_t rbp = 0;   // S->red buffer parity
    __device__ __forceinline__ float* next_red() { float* r = &S->red[rbp][0][0]; rbp ^= 1u; return r; }
    // ---- LM head (FP32 pipe) ----
    // RMSNorm output as fp32 into v (a 1024-float shared buffer), then a barrier.
    __device__ __forceinline__ void norm_f32(float* v, float x0, float x1, uint32_t g2, float ss) {
        const float r = 1.0f / sqrtf(ss * (1.0f / DIM) + EPS);
        *(float2*)&v[2 * tid] = make_float2((x0 * r) * bf_lo(g2), (x1 * r) * bf_hi(g2));
        bar();
    }
    // This lane's 32 values of a 1024-wide vector: xr[4i + e] = v[128 i + 4 lane + e]
    // (each warp-wide load is 512 contiguous bytes: no bank conflicts).
    __device__ __forceinline__ void load_regs(const float* v, float* xr) {
        #pragma unroll
        for (int i = 0; i < 8; i++) {
            const float4 a = *(const float4*)&v[128 * i + 4 * lane];
            xr[4 * i + 0] = a.x; xr[4 * i + 1] = a.y; xr[4 * i + 2] = a.z; xr[4 * i + 3] = a.w;
        }
    }
    // This lane's partial dot of a 1024-wide bf16 row with xr, four chains.
    __device__ __forceinline__ float row_part_f32(const uint8_t* row, const float* xr) {
        const uint2* w = (const uint2*)row;
        float a[4] = {0.f, 0.f, 0.f, 0.f};
        #pragma unroll
        for (int i = 0; i < 8; i++) {
            const uint2 v = w[i * 32 + lane];
            float& t = a[i & 3];
            t = fmaf(bf_lo(v.x), xr[4 * i + 0], t); t = fmaf(bf_hi(v.x), xr[4 * i + 1], t);
            t = fmaf(bf_lo(v.y), xr[4 * i + 2], t); t = fmaf(bf_hi(v.y), xr[4 * i + 3], t);
        }
        return (a[0] + a[1]) + (a[2] + a[3]);
    }
    // LM-head rows [a, b), 16 per chunk, two chunks at a time: warp w takes
    // rows 2w and 2w + 1 of the 32; f(row, value) runs on lanes 0 and 1.
    template <typename F>
    __device__ __forceinline__ void rows_lm(int a, int b, const float* xr, F&& f) {
        for (int r = a; r < b; r += 2 * kRowsLM) {
            const int n = min(2 * kRowsLM, b - r);
            const uint32_t nc = n > kRowsLM ? 2 : 1;
            const uint8_t* c0 = chunk(0);
            const uint8_t* c1 = nc == 2 ? chunk(1) : c0;
            const uint8_t* ch = (2 * warp < kRowsLM ? c0 : c1) + (size_t)((2 * warp) & (kRowsLM - 1)) * 2 * DIM;
            const bool v0 = 2 * warp < n, v1 = 2 * warp + 1 < n;
            float s0 = 0.f, s1 = 0.f;
            if (v0) s0 = row_part_f32(ch, xr);
            if (v1) s1 = row_part_f32(ch + 2 * DIM, xr);
            #pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                s0 += __shfl_xor_sync(0xffffffffu, s0, o);
                s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            }
            if (lane < 2 && 2 * warp + lane < n) f(r + 2 * warp + lane, lane == 0 ? s0 : s1);
            release(nc);
        }
    }
    // Rows [a, b) of 1024 columns (15 per chunk), two chunks per round: tile t
    // = the rows of chunk t; warp w takes k-tiles 4w .. 4w+3 of both tiles; the
    // sixteen partial sums of a row are added in warp order by thread i after
    // one barrier, which calls f(row, value).
    template <typename F>
    __device__ __forceinline__ void rows_1024(int a, int b, const uint32_t* bfr, F&& f) {
        const int lr = lane & 15;
        for (int r = a; r < b; r += 2 * kRowsK1024) {
            const int n = min(2 * kRowsK1024, b - r);
            const uint32_t nc = n > kRowsK1024 ? 2 : 1;
            const int n0 = min(n, kRowsK1024), n1 = n - n0;
            const uint8_t* c0 = chunk(0);
            const uint8_t* c1 = nc == 2 ? chunk(1) : c0;
            uint32_t ta[2];
            ta[0] = smem_addr(c0 + (size_t)(lr < n0 ? lr : 0) * kStride1024) + (lane >> 4) * 16;
            ta[1] = smem_addr(c1 + (size_t)(lr < n1 ? lr : 0) * kStride1024) + (lane >> 4) * 16;
            float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
            mma_tiles<2>(ta, bfr, 4 * warp, 4, d);
            float* red = next_red();
            put_red(red, 0, d[0]);
            put_red(red, 1, d[1]);
            release(nc);
            bar();
            if (tid < n) {
                const int i = tid < kRowsK1024 ? tid : 16 + tid - kRowsK1024;
                float v = 0.f;
                #pragma unroll
                for (int w = 0; w < kNCW; w++) v += red[w * 32 + i];
                f(r + tid, v);
            }
        }
    }
};

// sampler.h:137-174 over K candidates already in descending order (values v,
// ids): argmax when greedy, else temperature softmax, the top-p cut (when 0 <
// topp < 1), an xorshift64* coin (advancing rng) and the inverse CDF.  prob:
// K floats of scratch.  Returns the id, or -1 if none is a valid token.
__device__ __forceinline__ int sample_sorted(const float* v, const int* ids, int K, bool greedy, float T, float topp, unsigned long long& rng,
                                             float* prob) {
    int tok;
    if (greedy) {
        tok = ids[0];
    } else {
        int nc = K;
        const float mx = v[0];
        float sum = 0.f;
        for (int i = 0; i < nc; i++) { const float e = expf((v[i] - mx) / T); prob[i] = e; sum += e; }
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
    return (tok < 0 || tok >= VOCAB_SIZE) ? -1 : tok;
}

// The last CTA to finish: merges the G x K candidates of the CTAs (their
// local top-K of the LM-head rows), samples the next token (argmax, or
// sampler.h:137-174 over the K candidates in descending order: temperature
// softmax, top-p cut, xorshift64* coin, inverse CDF), hands it to the next
// chained launch and advances the launch tag.
__device__ __noinline__ void decode_merge_sample(const DecodeParams& P, uint8_t* ring, DecodeSmem* S, int tid, int G, int K, bool greedy,
                                                 bool head, int pos, int flags, uint32_t seq) {
    const int warp = tid >> 5, lane = tid & 31;
    struct { __device__ void bar() const { named_bar(1, kNCT); } } C;
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
            if (lane == 0) { S->av[warp] = v; S->ai[warp] = i; S->am[warp] = __int_as_float(at); }
            C.bar();
            if (tid == 0) {
                float bv = S->av[0]; int bi = S->ai[0]; int ba = __float_as_int(S->am[0]);
                for (int w = 1; w < kNCW; w++) {
                    const float v2 = S->av[w]; const int i2 = S->ai[w];
                    if (v2 > bv || (v2 == bv && i2 < bi)) { bv = v2; bi = i2; ba = __float_as_int(S->am[w]); }
                }
                P.top_v[kk] = bv; P.top_i[kk] = bi;
                S->tv[kk] = bv;
                S->ti[kk] = bi;
                if (ba >= 0) { cv[ba] = -INFINITY; ci[ba] = 0x7fffffff; }
            }
            C.bar();
        }
        if (tid == 0 && !(flags & kFlagCandidatesOnly)) {
            unsigned long long rng = P.in->rng;
            tok = sample_sorted(S->tv, S->ti, K, greedy, P.in->temperature, P.in->topp, rng, S->w.lg);
            if (tok < 0) {   // no finite candidate (NaN logits): report, never hand on
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
        if (flags & kFlagCandidatesOnly) {
            // the token comes from shard_merge_kernel after the candidate exchange
        } else if (head) {
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
}

template <bool kTr>
__device__ __forceinline__ void decode_consumer(const DecodeParams& P, uint8_t* ring, DecodeSmem* S, int c, int G, const Plan& pl,
                                             int token, int pos, int flags, uint32_t seq) {
    Consumer<kTr> C;
    C.P = &P; C.ring = ring; C.S = S;
    C.tid = threadIdx.x; C.warp = C.tid >> 5; C.lane = C.tid & 31;
    C.tag = seq;
    const int tid = C.tid, warp = C.warp, lane = C.lane;
    if (kTr && P.trace && tid == 0) C.tr = P.trace + (size_t)c * kTraceStride;
    const int g = pl.g, gs = pl.gs, gr = pl.gr;
    const bool owner = (gr == gs - 1);                 // its position range ends at pos
    const float sqrt_hd = sqrtf((float)HEAD_DIM);
    unsigned long long* tr = (kTr && P.trace && tid == 0) ? P.trace + (size_t)c * kTraceStride : nullptr;
#define QB_TRACE(i) do { if (kTr && tr) tr[(i)] = global_ns(); } while (0)
#define QB_SUB(i) do { if (kTr && tr && l == 13) tr[384 + (i)] = clock64(); } while (0)   // cycles: exact within a CTA
    QB_TRACE(0);

    if (tid < HEAD_DIM) S->rope[tid] = __ldg(P.rope + (size_t)pos * HEAD_DIM + tid);

    for (int l = 0; l < N_LAYERS; l++) {
        const int TB = 1 + 10 * l;
        C.flush();
        C.tl = l;
        // ---------------- QKV ----------------
        {
            const uint32_t g2 = C.gain_fetch(P.in_ln[l]);
            const int j = tid * 2;
            float xv[2];
            if (l == 0) {
                const uint32_t w = __ldg((const uint32_t*)(P.embed + (size_t)token * DIM + j));
                xv[0] = bf_lo(w); xv[1] = bf_hi(w);
            } else {
                const uint64_t* p = P.xw + (size_t)l * DIM + j;
                C.template gather<1>([&](int) { return p; }, 1u, xv, 10 * l);
            }
            S->xres[j] = xv[0]; S->xres[j + 1] = xv[1];
            const float rn = C.gain_bx(xv[0], xv[1], g2);
            QB_SUB(31);
            QB_TRACE(TB + 0);
            uint64_t* qkv = P.qkvw + (size_t)l * 4096;
            const bool withhold = l == 0 && g == P.debug_skip;   // failure tests only
            C.rows_1024(pl.qa, pl.qb, &S->bx[0][0][0], [&](int row, float v) {
                if (!withhold) xw_store(qkv + qkv_dst(g, row), v * rn, seq);
            });
        }
        QB_TRACE(TB + 1);
        QB_SUB(32);

        // ---------------- ATT ----------------
        if (warp < 4) {   // warp w: q head 2g (0), q head 2g+1 (1), k (2), v (3); lane holds dims 4l..4l+3
            const int off = warp < 2 ? 256 * g + 128 * warp : (warp == 2 ? Q_DIM + 128 * g : Q_DIM + KV_DIM + 128 * g);
            const uint64_t* p = P.qkvw + (size_t)l * 4096 + off + 4 * lane;
            uint2 gn = make_uint2(0u, 0u);
            if (warp < 3) gn = __ldg((const uint2*)((warp < 2 ? P.qn[l] : P.kn[l]) + 4 * lane));
            float x[4];
            C.template gather<2>([&](int i) { return p + 2 * i; }, 3u, x, 10 * l + 2);
            if (warp < 3) {
                const float tot = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
                const float r = 1.0f / sqrtf(tot * (1.0f / HEAD_DIM) + EPS);
                x[0] = (x[0] * r) * bf_lo(gn.x); x[1] = (x[1] * r) * bf_hi(gn.x);
                x[2] = (x[2] * r) * bf_lo(gn.y); x[3] = (x[3] * r) * bf_hi(gn.y);
                // NeoX rotation: dim d pairs with d ^ 64, held by lane ^ 16
                #pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float pv = __shfl_xor_sync(0xffffffffu, x[e], 16);
                    const int d = 4 * lane + e, jj = d & 63;
                    const float cj = S->rope[jj], sj = S->rope[64 + jj];
                    x[e] = d < 64 ? (x[e] * cj - pv * sj) : (pv * sj + x[e] * cj);
                }
            }
            if (warp < 2) {
                *(float4*)&S->qs[128 * warp + 4 * lane] = make_float4(x[0], x[1], x[2], x[3]);
            } else if (owner) {
                uint16_t b[4];
                #pragma unroll
                for (int e = 0; e < 4; e++) b[e] = f2bf(x[e]);
                const size_t at = ((size_t)l * kGroups * SEQ_LEN * HEAD_DIM) + pl.kvbase + (size_t)pos * HEAD_DIM + 4 * lane;
                uint16_t* dst = (warp == 2 ? P.kc : P.vc) + at;
                *(uint2*)dst = make_uint2((uint32_t)b[0] | ((uint32_t)b[1] << 16), (uint32_t)b[2] | ((uint32_t)b[3] << 16));
                float* sm = warp == 2 ? S->kn : S->vn;
                *(float4*)&sm[4 * lane] = make_float4(bf2f(b[0]), bf2f(b[1]), bf2f(b[2]), bf2f(b[3]));
            }
        }
        C.bar();
        QB_TRACE(TB + 2);
        QB_SUB(33);
        {
            // Warp w: q head hh = w / 8 and positions 8 (w % 8) .. +7 of every
            // K|V chunk.  Four lanes score one position: lane quarter qq takes
            // the 16 bf16 pairs 4 (j ^ x) + qq, j = 0..15, x = position % 16 —
            // a rotation that spreads the warp's 32 reads over all 32 banks.
            // Then one online-softmax step per chunk; for P.V lane l holds
            // dims 4l..4l+3.
            const int hh = warp >> 3, sub = warp & 7;
            const int ti = 8 * sub + (lane >> 2), qq = lane & 3, xr4 = (ti & 15) << 2;
            float2 qv[16];
            #pragma unroll
            for (int j = 0; j < 16; j++) qv[j] = *(const float2*)&S->qs[128 * hh + 2 * (((4 * j) ^ xr4) + qq)];
            float m = -INFINITY, lsum = 0.f, a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
            for (int t0 = pl.p0; t0 < pl.pe; t0 += kKVChunk) {
                const int cnt = min(kKVChunk, pl.pe - t0);
                const uint8_t* ch = C.chunk(0);
                const bool valid = ti < cnt;
                float s = 0.f;
                if (valid) {
                    const uint32_t* kr = (const uint32_t*)(ch + (size_t)ti * 2 * HEAD_DIM) + qq;
                    float c4[4] = {0.f, 0.f, 0.f, 0.f};
                    #pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const uint32_t w = kr[(4 * j) ^ xr4];
                        c4[j & 3] = fmaf(bf_lo(w), qv[j].x, c4[j & 3]);
                        c4[j & 3] = fmaf(bf_hi(w), qv[j].y, c4[j & 3]);
                    }
                    s = (c4[0] + c4[1]) + (c4[2] + c4[3]);
                }
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                s += __shfl_xor_sync(0xffffffffu, s, 2);
                s = valid ? s / sqrt_hd : -INFINITY;
                float mc = fmaxf(s, __shfl_xor_sync(0xffffffffu, s, 4));
                mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 8));
                mc = fmaxf(mc, __shfl_xor_sync(0xffffffffu, mc, 16));
                const float mn = fmaxf(m, mc);
                if (mn != -INFINITY) {   // warp-uniform
                    const float sc = expf(m - mn);
                    const float pr = valid ? expf(s - mn) : 0.f;
                    float ps = pr + __shfl_xor_sync(0xffffffffu, pr, 4);
                    ps += __shfl_xor_sync(0xffffffffu, ps, 8);
                    ps += __shfl_xor_sync(0xffffffffu, ps, 16);
                    lsum = fmaf(lsum, sc, ps);
                    a0 *= sc; a1 *= sc; a2 *= sc; a3 *= sc;
                    const uint8_t* vb = ch + kVOff + 8 * lane;
                    #pragma unroll
                    for (int i = 0; i < 8; i++) {
                        const float pi = __shfl_sync(0xffffffffu, pr, 4 * i);
                        if (8 * sub + i < cnt) {
                            const uint2 vw = *(const uint2*)(vb + (size_t)(8 * sub + i) * 2 * HEAD_DIM);
                            a0 = fmaf(pi, bf_lo(vw.x), a0); a1 = fmaf(pi, bf_hi(vw.x), a1);
                            a2 = fmaf(pi, bf_lo(vw.y), a2); a3 = fmaf(pi, bf_hi(vw.y), a3);
                        }
                    }
                    m = mn;
                }
                C.release(1);
            }
            QB_SUB(5);
            if (owner && sub == 0) {   // the new position, from shared memory (warps 0 and 8)
                const float4 kk = *(const float4*)&S->kn[4 * lane], vv = *(const float4*)&S->vn[4 * lane];
                const float4 qh = *(const float4*)&S->qs[128 * hh + 4 * lane];
                float s = qh.x * kk.x; s = fmaf(qh.y, kk.y, s); s = fmaf(qh.z, kk.z, s); s = fmaf(qh.w, kk.w, s);
                s = warp_sum(s) / sqrt_hd;
                const float mn = fmaxf(m, s);
                const float sc = expf(m - mn), pr = expf(s - mn);
                lsum = fmaf(lsum, sc, pr);
                a0 = fmaf(a0, sc, pr * vv.x); a1 = fmaf(a1, sc, pr * vv.y); a2 = fmaf(a2, sc, pr * vv.z); a3 = fmaf(a3, sc, pr * vv.w);
                m = mn;
            }
            // combine the 8 warps of each head
            *(float4*)&S->w.comb[(size_t)warp * HEAD_DIM + 4 * lane] = make_float4(a0, a1, a2, a3);
            if (lane == 0) { S->am[warp] = m; S->al[warp] = lsum; }
            C.bar();
            QB_SUB(6);
            if (tid < 2 * HEAD_DIM) {
                const int h2 = tid >> 7, d = tid & 127;
                float M = -INFINITY;
                #pragma unroll
                for (int w = 0; w < 8; w++) M = fmaxf(M, S->am[8 * h2 + w]);
                float Ls = 0.f, A = 0.f;
                #pragma unroll
                for (int w = 0; w < 8; w++) {
                    const float mw = S->am[8 * h2 + w];
                    const float sc = mw == -INFINITY ? 0.f : expf(mw - M);
                    Ls = fmaf(S->al[8 * h2 + w], sc, Ls);
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
            // stage the group's gs x 264 partial words in shared memory, in pairs over all threads
            const uint64_t* gbase = P.partw + (size_t)(l * kGroups + g) * kMaxGS * kPartStride;
            const int nw = gs * kPartStride;
            constexpr int kPer = (kMaxGS * kPartStride + 2 * kNCT - 1) / (2 * kNCT);
            uint32_t pend = 0;
            #pragma unroll
            for (int i = 0; i < kPer; i++) if (2 * tid + 2 * kNCT * i < nw) pend |= 1u << i;
            float v[2 * kPer];
            QB_SUB(8);
            C.template gather<kPer>([&](int i) { return gbase + 2 * tid + 2 * kNCT * i; }, pend, v, 10 * l + 4);
            #pragma unroll
            for (int i = 0; i < kPer; i++) {
                if (pend & (1u << i)) *(float2*)&S->w.pst[2 * tid + 2 * kNCT * i] = make_float2(v[2 * i], v[2 * i + 1]);
            }
            QB_SUB(9);
        }
        C.bar();
        QB_TRACE(TB + 4);
        {
            // warp w: head hh = w / 8; lane c computes partial c's weight, then
            // lanes (d, half) of the warp add the even / odd partials of dim d.
            const int hh = warp >> 3;
            const float* b = &S->w.pst[lane * kPartStride + hh * kHeadPart];
            const bool live = lane < gs && b[1] > 0.f;
            const float mm = live ? b[0] : -INFINITY;
            const float M = warp_max(mm);
            const float e = live ? expf(mm - M) : 0.f;
            const float den = warp_sum(live ? b[1] * e : 0.f);
            const float wgt = e / den;
            const int d = 16 * (warp & 7) + (lane & 15), half = lane >> 4;
            float num = 0.f;
            for (int i = 0; i < (gs + 1) / 2; i++) {
                const int cc = 2 * i + half;
                const float wc = __shfl_sync(0xffffffffu, wgt, cc & 31);
                if (cc < gs) num = fmaf(S->w.pst[cc * kPartStride + hh * kHeadPart + 4 + d], wc, num);
            }
            num += __shfl_xor_sync(0xffffffffu, num, 16);
            const float nx = __shfl_down_sync(0xffffffffu, num, 1);   // dim d + 1
            if (half == 0 && (d & 1) == 0) C.put_pair(&S->bo[0][0][0], hh * HEAD_DIM + d, num, nx);
        }
        QB_SUB(11);
        C.bar();
        QB_SUB(12);
        {
            // tile t = rows 16t .. 16t+15 of the chunk (up to 62 rows); warp w:
            // tile w % 4, k-tiles 4 (w / 4) .. +3 of the 16; four warps per row
            uint64_t* y = P.yw + (size_t)(l * kGroups + g) * DIM;
            const int t = warp & 3, lr = lane & 15;
            for (int r = pl.oa; r < pl.ob; r += kRowsWo) {
                const int cnt = min(kRowsWo, pl.ob - r);
                const uint8_t* ch = C.chunk(0);
                QB_SUB(13);
                const int row = 16 * t + lr;
                uint32_t ta[1] = {smem_addr(ch + (size_t)(row < cnt ? row : 0) * kStrideWo) + (lane >> 4) * 16};
                float d[1][4] = {{0.f, 0.f, 0.f, 0.f}};
                C.template mma_tiles<1>(ta, &S->bo[0][0][0], 4 * (warp >> 2), 4, d);
                float* red = C.next_red();
                C.put_red(red, 0, d[0]);          // this warp's tile rows at red[warp][0..15]
                C.release(1);
                C.bar();
                if (tid < cnt) {                  // row tid: tile tt, summed over warps tt, tt+4, tt+8, tt+12
                    const int tt = tid >> 4, ri = tid & 15;
                    const float v = ((red[tt * 32 + ri] + red[(tt + 4) * 32 + ri]) + red[(tt + 8) * 32 + ri]) + red[(tt + 12) * 32 + ri];
                    xw_store(y + r + tid, v, seq);
                }
                QB_SUB(14);
            }
        }
        QB_TRACE(TB + 5);

        // ---------------- MLP-A ----------------
        {
            const uint32_t g2 = C.gain_fetch(P.post_ln[l]);
            const int j = tid * 2;
            const uint64_t* yb = P.yw + (size_t)l * kGroups * DIM + j;
            QB_SUB(16);
            float x0 = S->xres[j], x1 = S->xres[j + 1];
            {
                float yv[2 * kGroups];
                C.template gather<kGroups>([&](int gg) { return yb + (size_t)gg * DIM; }, (1u << kGroups) - 1u, yv, 10 * l + 6);
                #pragma unroll
                for (int gg = 0; gg < kGroups; gg++) { x0 += yv[2 * gg]; x1 += yv[2 * gg + 1]; }
            }
            QB_SUB(17);
            S->xres[j] = x0; S->xres[j + 1] = x1;
            const float rn = C.gain_bx(x0, x1, g2);
            QB_TRACE(TB + 6);
            QB_SUB(34);
            QB_SUB(20);
            // gate|up units, 7 per chunk (gate rows 0..6, up rows 7..13), two
            // chunks per round: tile t = chunk t; warp w takes k-tiles 4w..4w+3
            uint64_t* hw = P.hw + (size_t)l * HIDDEN_DIM;
            const int lr = lane & 15, lu = lr < kUnitsGU ? lr : lr - kUnitsGU;
            for (int u = pl.ha; u < pl.hb; u += 2 * kUnitsGU) {
                const int n = min(2 * kUnitsGU, pl.hb - u);
                const uint32_t nc = n > kUnitsGU ? 2 : 1;
                const int n0 = min(n, kUnitsGU), n1 = n - n0;
                const uint8_t* c0 = C.chunk(0);
                const uint8_t* c1 = nc == 2 ? C.chunk(1) : c0;
                uint32_t ta[2];
                ta[0] = smem_addr(c0 + (size_t)(lr < 2 * kUnitsGU && lu < n0 ? lr : 0) * kStride1024) + (lane >> 4) * 16;
                ta[1] = smem_addr(c1 + (size_t)(lr < 2 * kUnitsGU && lu < n1 ? lr : 0) * kStride1024) + (lane >> 4) * 16;
                float d[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
                C.template mma_tiles<2>(ta, &S->bx[0][0][0], 4 * warp, 4, d);
                float* red = C.next_red();
                C.put_red(red, 0, d[0]);
                C.put_red(red, 1, d[1]);
                C.release(nc);
                C.bar();
                if (tid < n) {   // unit tid of the round
                    const int t = tid < kUnitsGU ? 0 : 1, uu = tid - t * kUnitsGU;
                    float gt = 0.f, up = 0.f;
                    #pragma unroll
                    for (int w = 0; w < kNCW; w++) { gt += red[w * 32 + 16 * t + uu]; up += red[w * 32 + 16 * t + kUnitsGU + uu]; }
                    gt *= rn; up *= rn;
                    xw_store(hw + u + tid, (gt / (1.0f + expf(-gt))) * up, seq);
                }
            }
            QB_SUB(22);
        }
        QB_TRACE(TB + 7);
        QB_SUB(35);

        // ---------------- MLP-B ----------------
        {
            const uint64_t* hb = P.hw + (size_t)l * HIDDEN_DIM + 2 * tid;
            constexpr int kHP = HIDDEN_DIM / (2 * kNCT);
            float hv[2 * kHP];
            QB_SUB(25);
            C.template gather<kHP>([&](int i) { return hb + 2 * kNCT * i; }, (1u << kHP) - 1u, hv, 10 * l + 8);
            #pragma unroll
            for (int i = 0; i < kHP; i++) C.put_pair(&S->w.bh[0][0][0], 2 * tid + 2 * kNCT * i, hv[2 * i], hv[2 * i + 1]);
        }
        C.bar();
        QB_TRACE(TB + 8);
        {
            // rows of Wd, two chunks (8 rows) per round as one tile: tile rows
            // 0..3 = chunk 0, 4..7 = chunk 1; warp w takes k-tiles 12w..12w+11
            uint64_t* xn = P.xw + (size_t)(l + 1) * DIM;
            const int lr = lane & 15;
            for (int r = pl.da; r < pl.db; r += 2 * kRowsWd) {
                const int n = min(2 * kRowsWd, pl.db - r);
                const uint32_t nc = n > kRowsWd ? 2 : 1;
                const uint8_t* c0 = C.chunk(0);
                const uint8_t* c1 = nc == 2 ? C.chunk(1) : c0;
                QB_SUB(28);
                const uint8_t* rp = lr < n ? (lr < kRowsWd ? c0 + (size_t)lr * kStrideWd : c1 + (size_t)(lr - kRowsWd) * kStrideWd) : c0;
                uint32_t ta[1] = {smem_addr(rp) + (lane >> 4) * 16};
                float d[1][4] = {{0.f, 0.f, 0.f, 0.f}};
                C.template mma_tiles<1>(ta, &S->w.bh[0][0][0], 12 * warp, HIDDEN_DIM / 16 / kNCW, d);
                float* red = C.next_red();
                C.put_red(red, 0, d[0]);
                C.release(nc);
                C.bar();
                QB_SUB(30);
                if (tid < n) {
                    float v = 0.f;
                    #pragma unroll
                    for (int w = 0; w < kNCW; w++) v += red[w * 32 + tid];
                    xw_store(xn + r + tid, S->xres[r + tid] + v, seq);
                }
            }
        }
        C.bar();     // S->w.bh and S->xres are reused by the next layer
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
        const uint32_t g2 = C.gain_fetch(P.final_ln);
        float ss, x0, x1;
        {
            const int j = tid * 2;
            float xv[2];
            {
                const uint64_t* p = P.xw + (size_t)N_LAYERS * DIM + j;
                C.template gather<1>([&](int) { return p; }, 1u, xv, 10 * N_LAYERS);
            }
            x0 = xv[0]; x1 = xv[1];
            ss = C.block_sum(x0 * x0 + x1 * x1);
        }
        QB_TRACE(kTrHead);
        const int va = pl.va;
        const bool wl = (flags & kFlagWriteLogits) != 0;
        {
            float* xs = reinterpret_cast<float*>(&S->bx[0][0][0]);   // 4 KB of the 6 KB fragment buffer
            C.norm_f32(xs, x0, x1, g2, ss);
            float xr[32];
            C.load_regs(xs, xr);
            C.rows_lm(pl.va, pl.vb, xr, [&](int row, float v) {
                S->w.lg[row - va] = v;
                if (wl) P.logits[row] = v;
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
    if (S->flag) decode_merge_sample(P, ring, S, tid, G, K, greedy, head, pos, flags, seq);
    QB_TRACE(kTrHead + 3);
#undef QB_TRACE
#undef QB_SUB
}

// kTr: the tracing build (stage time stamps into P.trace); the other build has
// no trace code at all.
template <bool kTr>
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
        if ((tid & 31) == 0) decode_producer<kTr>(P, ring, S, c, pl);
        return;
    }
    if ((tid >> 5) == kNCW + 1) {
        if ((tid & 31) == 0) decode_prefetcher(P, S, pl);
        return;
    }
    decode_consumer<kTr>(P, ring, S, c, G, pl, token, pos, flags, seq);
}

// ---------------------------------------------------------------------------
// Vocabulary-sharded LM head: after every rank's launch left its shard's top K
// in top_v / top_i (kFlagCandidatesOnly) and the ranks exchanged them (an
// all-gather on the handle's stream: n_ranks x K values and global ids), this
// kernel merges them in (value descending, id ascending) order — the order of
// the one-GPU device sampler — and samples the step's token with the same
// math and RNG state on every rank, then hands it to the next launch (StepIn)
// and records it (StepOut, tokens_out).  One CTA of kMergeThreads threads;
// n_ranks * K <= 2 * kMergeThreads.
// ---------------------------------------------------------------------------
constexpr int kMergeThreads = 256;

__global__ void __launch_bounds__(kMergeThreads) shard_merge_kernel(const float* __restrict__ gv, const int* __restrict__ gi, int n_ranks,
                                                                    int K, int stride, StepIn* in, StepOut* out, int* tokens_out,
                                                                    int tokens_cap) {
    __shared__ float sv[2 * kMergeThreads];
    __shared__ int si[2 * kMergeThreads];
    __shared__ float prob[kMaxCand];
    const int n = n_ranks * K, tid = threadIdx.x;
    // every candidate's rank: the candidates that precede it (NaN counts as -inf;
    // equal (value, id) pairs, which only padding entries share, by position)
    // candidate e = (rank e / K, entry e % K) at gv / gi + rank * stride + entry
    auto at = [&](int e) { return (e / K) * stride + e % K; };
    for (int e = tid; e < n; e += kMergeThreads) {
        float v = gv[at(e)];
        const int id = gi[at(e)];
        if (v != v) v = -INFINITY;
        int rank = 0;
        for (int f = 0; f < n; f++) {
            float w = gv[at(f)];
            if (w != w) w = -INFINITY;
            const int jd = gi[at(f)];
            rank += (w > v || (w == v && (jd < id || (jd == id && f < e)))) ? 1 : 0;
        }
        sv[rank] = v;
        si[rank] = id;
    }
    __syncthreads();
    if (tid == 0) {
        const bool greedy = in->temperature == 0.0f || in->top_k == 1;
        unsigned long long rng = in->rng;
        int tok = sample_sorted(sv, si, greedy ? 1 : K, greedy, in->temperature, in->topp, rng, prob);
        if (tok < 0) {
            atomicOr(&out->err, 16u);
            atomicExch(&out->err_where, -202);
            tok = 0;
        }
        in->rng = rng;
        out->rng = rng;
        in->token = tok;
        out->out_token = tok;
        const int nd = out->n_done;
        if (nd < tokens_cap) tokens_out[nd] = tok;
        out->n_done = nd + 1;
    }
}

}  // namespace qb
