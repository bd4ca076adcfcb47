// decode_cluster.cuh — one batch-1 decode position of Qwen3-0.6B as ONE
// persistent launch of 8-CTA thread-block clusters (15 clusters, 120 CTAs on a
// B200; one CTA per SM).
//
// Replaces the same reference chain as decode_kernel.cuh (qwen_model.cuh:772-851
// and, for the device-sampling entry points, sampler.h:120-175) and reuses its
// weight streaming (a producer warp, a 5 x 32 KB bulk-copy ring), its
// tensor-core row tiles and its device sampler.  What changes is where the
// values between stages travel.  A hop through L2 (an 8-byte word tagged with
// the launch sequence number, polled by the readers) costs about 1.1 us on a
// B200; a hop through distributed shared memory inside a cluster (st.async
// into the peer CTAs' shared memory, completing bytes on their mbarriers)
// about 0.2 us.  So the KV head g's work is done by cluster g (g < 8), whose
// hops stay on chip, and the MLP's down projection is fused into the stage
// that computes its input, reduced inside each cluster:
//
//   X     all: x_l = x_mid_{l-1} + sum over clusters k of P_k (L2, tagged words)
//   QKV   cluster g, CTA r: RMSNorm(x_l) -> rows [64r, 64r+64) of the group's
//         512 q|k|v rows -> every CTA of the cluster (DSMEM)             -> Q
//   ATT   cluster g: QK-norm + RoPE (every CTA), the CTA owning `pos` appends
//         bf16 K/V; split-K attention over the CTA's share of the positions
//         -> (max, sum, accumulator) to every CTA of the cluster (DSMEM)  -> P
//   OPROJ cluster g, CTA r: combine the 8 partials -> o (256) -> rows
//         [128r, 128r+128) of Wo[:, 256g:256g+256] -> y_g (L2, tagged)    -> Y
//   MLP   all: x_mid = x_l + sum_g y_g (fixed order); RMSNorm; the CTA's hidden
//         units: gate, up, SwiGLU -> h (kept in shared memory); its columns of
//         W_down (rows of W_down^T) times h -> a 1024-vector; in the cluster,
//         CTA r receives rows [128r, 128r+128) of all 8 vectors (DSMEM), adds
//         them in rank order and publishes P_k's rows (L2, tagged)       -> X
//   HEAD  all: x_L -> final RMSNorm -> LM-head rows -> top-K -> last CTA samples.
//
// Two L2 hops and three cluster hops per layer, instead of five L2 hops.
// Clusters 8.. (no KV head) take a larger share of the hidden units, since the
// KV-head clusters also stream the attention weights and the K/V cache.
//
// Numerics: as decode_kernel.cuh (bf16 weights and KV cache, fp32 everything
// else, every sum in a fixed order: bit-reproducible for a given grid).
// Every wait is bounded (P.wait_ns on another CTA's values, kWaitNs multiples
// on the ring): on expiry the kernel records an error,
// stops waiting and still drains its copies; the host resets the device state.
#pragma once
#include "decode_kernel.cuh"

namespace qb {

constexpr int kCl = 8;                       // CTAs per cluster
constexpr int kClQRows = kQKVRows / kCl;     // 64 q|k|v rows per CTA of a KV-head cluster
constexpr int kClORows = DIM / kCl;          // 128 Wo rows per CTA, and 128 published x rows
constexpr int kClMaxClusters = 18;
constexpr int kClAttUnits = 20;              // hidden units of each CTA of a KV-head cluster
constexpr int kClThreads = kNCT + 32;        // 16 consumer warps + the producer warp (no prefetch warp)

struct ClPlan {
    int k, r, ncl, G;    // cluster, rank in it, clusters, CTAs
    bool att;            // k < kGroups: the cluster of KV head g = k
    int g;
    int p0, p1, pe;      // attention positions [p0, p1); cached ones [p0, pe)
    int ha, hb;          // hidden units
    int va, vb;          // LM-head rows
    bool head;
    size_t kvbase;
};

struct __align__(16) ClSmem {
    DecodeSmem base;                              // ring barriers, fragments, reductions, sampler state
    alignas(16) float qkv[kQKVRows];              // the group's raw q | k | v projections
    alignas(16) float part[kCl][kPartStride];     // attention partials of the 8 CTAs
    alignas(16) float xred[kCl][kClORows];        // the 8 CTAs' MLP sums for this CTA's 128 rows
    uint64_t mb_q, mb_p, mb_r;                    // completed by the peers' st.async bytes
    ClPlan pl;                                    // this CTA's share of every stage
};
static_assert(offsetof(ClSmem, qkv) % 16 == 0 && offsetof(ClSmem, part) % 16 == 0 && offsetof(ClSmem, xred) % 16 == 0,
              "cluster exchange buffers must be 16-byte aligned");
constexpr size_t kClSmemBytes = (size_t)kSlots * kSlotBytes + sizeof(ClSmem);
static_assert(kClSmemBytes <= 227 * 1024, "one CTA per SM: at most 227 KB of shared memory");

// Hidden units of CTA (k, r): the KV-head clusters' CTAs take kClAttUnits each,
// the other clusters share the rest.
__host__ __device__ __forceinline__ void cl_units(int k, int r, int ncl, int& a, int& b) {
    const int att_ctas = kGroups * kCl, att_units = att_ctas * kClAttUnits;
    if (k < kGroups) {
        a = (k * kCl + r) * kClAttUnits;
        b = a + kClAttUnits;
    } else {
        const int rest = (ncl - kGroups) * kCl, i = (k - kGroups) * kCl + r;
        a = att_units + span_lo(HIDDEN_DIM - att_units, rest, i);
        b = att_units + span_lo(HIDDEN_DIM - att_units, rest, i + 1);
    }
}

__device__ __forceinline__ ClPlan cl_make_plan(const DecodeParams& P, int k, int r, int ncl, int pos, int flags) {
    ClPlan p;
    p.k = k; p.r = r; p.ncl = ncl; p.G = ncl * kCl;
    p.att = k < kGroups;
    p.g = p.att ? k : 0;
    const int L = pos + 1;
    p.p0 = span_lo(L, kCl, r); p.p1 = span_lo(L, kCl, r + 1);
    p.pe = min(p.p1, pos);
    cl_units(k, r, ncl, p.ha, p.hb);
    const int c = k * kCl + r, nrows = P.lm_end - P.lm_begin;
    p.va = P.lm_begin + span_lo(nrows, p.G, c); p.vb = P.lm_begin + span_lo(nrows, p.G, c + 1);
    p.head = !(flags & kFlagNoHead);
    p.kvbase = (size_t)p.g * SEQ_LEN * HEAD_DIM;
    return p;
}

// One CTA's weight / KV stream, in consumption order:
//   per layer, KV-head clusters: [q|k|v rows 64r.., 15/chunk][K | V of cached
//   positions, 64/chunk][Wo_g rows 128r.., 62/chunk]; every CTA: [gate|up units,
//   7/chunk][W_down^T rows of the same units, 16/chunk]
//   then (unless kFlagNoHead): [LM-head rows, 16/chunk]
struct ClChunkIter {
    int l = 0, st = 0, r = 0;
    __device__ int next(const DecodeParams& P, const ClPlan& pl, Seg* seg) {
        for (;;) {
            switch (st) {
            case 0:
                if (pl.att) { st = 1; r = kClQRows * pl.r; } else { st = 5; r = pl.ha; }
                break;
            case 1:
                if (r < kClQRows * (pl.r + 1)) {
                    const int n = min(kRowsK1024, kClQRows * (pl.r + 1) - r);
                    int i = 0, kk = 0;
                    while (i < n) {
                        const int rr = r + i;
                        const uint16_t* src; int lim;
                        if (rr < 256) { src = P.wq[l] + (size_t)(256 * pl.g + rr) * DIM; lim = 256; }
                        else if (rr < 384) { src = P.wk[l] + (size_t)(128 * pl.g + rr - 256) * DIM; lim = 384; }
                        else { src = P.wv[l] + (size_t)(128 * pl.g + rr - 384) * DIM; lim = 512; }
                        const int m = min(n - i, lim - rr);
                        seg[kk++] = {(const uint8_t*)src, (uint32_t)(2 * DIM), (uint32_t)(i * kStride1024), (uint32_t)m,
                                     (uint32_t)(2 * DIM), (uint32_t)kStride1024};
                        i += m;
                    }
                    r += n;
                    return kk;
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
                st = 3; r = kClORows * pl.r;
                break;
            case 3:
                if (r < kClORows * (pl.r + 1)) {
                    const int n = min(kRowsWo, kClORows * (pl.r + 1) - r);
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
                st = 7; r = pl.ha;
                break;
            case 7:
                if (r < pl.hb) {
                    const int n = min(kRowsWdT, pl.hb - r);
                    seg[0] = {(const uint8_t*)(P.wdt[l] + (size_t)r * DIM), (uint32_t)(n * 2 * DIM), 0, 1, 0, 0};
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

__device__ __noinline__ void cl_producer(const DecodeParams& P, uint8_t* ring, DecodeSmem* S, int c, const ClPlan& pl) {
    const uint64_t pol = policy_evict_first();
    ClChunkIter it;
    Seg seg[3];
    uint32_t k = 0;
    bool dead = false;
    for (;;) {
        const int n = it.next(P, pl, seg);
        if (n == 0) break;
        const uint32_t s = k % kSlots, ph = (k / kSlots) & 1u;
        if (!dead && !mbar_wait(&S->empty[s], ph ^ 1u, 2 * kWaitNs)) {
            atomicOr(&P.out->err, 2u);
            atomicExch(&P.out->err_where, -1 - (int)s);
            dead = true;   // issue nothing more; consumers stop waiting after their own timeout
        }
        if (!dead) {
            uint32_t total = 0;
            for (int i = 0; i < n; i++) total += seg[i].bytes * seg[i].rows;
            mbar_arrive_expect_tx(&S->full[s], total);
            uint8_t* d = ring + (size_t)s * kSlotBytes;
            for (int i = 0; i < n; i++)
                for (uint32_t q = 0; q < seg[i].rows; q++)
                    bulk_g2s(d + seg[i].off + q * seg[i].dst_stride, seg[i].src + (size_t)q * seg[i].src_stride, seg[i].bytes, &S->full[s],
                             pol);
        }
        k++;
    }
    // drain: the copies still in flight land before the CTA leaves (bounded)
    for (uint32_t j = k > (uint32_t)kSlots ? k - kSlots : 0u; j < k; j++) mbar_wait(&S->full[j % kSlots], (j / kSlots) & 1u, kWaitNs);
    P.chunk_count[2 * c] = (int)k;
}

template <bool kTr>
struct ClConsumer : Consumer<kTr> {
    ClSmem* CS;
    uint32_t rank;
    // Waits (every consumer thread) for the phase of a DSMEM exchange barrier;
    // bounded.  Thread 0 arms it with the bytes the 8 CTAs send first.
    __device__ __forceinline__ void dsmem_wait(uint64_t* mb, uint32_t bytes, uint32_t parity, int where) {
        if (this->tid == 0) mbar_arrive_expect_tx(mb, bytes);
        if (this->failed) return;
        if (mbar_try_wait_cluster(mb, parity)) return;
        const uint64_t t0 = global_ns();
        uint32_t it = 0;
        while (!mbar_try_wait_cluster(mb, parity)) {
            if ((++it & 63u) == 0 && global_ns() - t0 > this->P->wait_ns) {
                atomicOr(&this->P->out->err, 32u);
                atomicExch(&this->P->out->err_where, where);
                this->failed = true;
                return;
            }
        }
    }
    // Remote addresses in CTA `dst` of this CTA's shared-memory offset `local`.
    __device__ __forceinline__ uint32_t remote(const void* local, uint32_t dst) { return dsmem_map(smem_addr(local), dst); }
};

template <bool kTr>
__device__ __forceinline__ void cl_consumer(const DecodeParams& P, uint8_t* ring, ClSmem* CS, int c, const ClPlan& pl, int token, int pos,
                                         int flags, uint32_t seq) {
    ClConsumer<kTr> C;
    DecodeSmem* S = &CS->base;
    C.P = &P; C.ring = ring; C.S = S; C.CS = CS;
    C.tid = threadIdx.x; C.warp = C.tid >> 5; C.lane = C.tid & 31;
    C.tag = seq;
    C.rank = (uint32_t)pl.r;
    const int tid = C.tid, warp = C.warp, lane = C.lane;
    const int G = pl.G, g = pl.g;
    const bool owner = (pl.r == kCl - 1);              // its position range ends at pos
    const float sqrt_hd = sqrtf((float)HEAD_DIM);
    if (kTr && P.trace && tid == 0) C.tr = P.trace + (size_t)c * kTraceStride;
    unsigned long long* tr = (kTr && P.trace && tid == 0) ? P.trace + (size_t)c * kTraceStride : nullptr;
#define QB_TRACE(i) do { if (kTr && tr) tr[(i)] = global_ns(); } while (0)
    QB_TRACE(0);
    if (tid < HEAD_DIM) S->rope[tid] = __ldg(P.rope + (size_t)pos * HEAD_DIM + tid);
    const int j = 2 * tid;
    // x_l's cluster partials: [L+1][kClMaxClusters][DIM] tagged words
    auto xpw = [&](int l, int k) { return P.xw + ((size_t)l * kClMaxClusters + k) * DIM; };

    for (int l = 0; l < N_LAYERS; l++) {
        const int TB = 1 + 10 * l;
        C.flush();
        C.tl = l;
        const uint32_t par = (uint32_t)l & 1u;
        // ---------------- x_l ----------------
        float x0, x1;
        if (l == 0) {
            const uint32_t w = __ldg((const uint32_t*)(P.embed + (size_t)token * DIM + j));
            x0 = bf_lo(w); x1 = bf_hi(w);
        } else {
            // x_l = x_mid_{l-1} + the clusters' partial sums, in cluster order
            x0 = S->xres[j]; x1 = S->xres[j + 1];
            const int n1 = min(pl.ncl, 8), n2 = pl.ncl - n1;
            float v[16];
            C.template gather<8>([&](int i) { return xpw(l, i) + j; }, (1u << n1) - 1u, v, 10 * l);
            #pragma unroll
            for (int i = 0; i < 8; i++) if (i < n1) { x0 += v[2 * i]; x1 += v[2 * i + 1]; }
            if (n2 > 0) {
                C.template gather<8>([&](int i) { return xpw(l, 8 + i) + j; }, (1u << n2) - 1u, v, 10 * l);
                #pragma unroll
                for (int i = 0; i < 8; i++) if (i < n2) { x0 += v[2 * i]; x1 += v[2 * i + 1]; }
            }
        }
        S->xres[j] = x0; S->xres[j + 1] = x1;      // (each thread reads and writes only its own two entries)
        QB_TRACE(TB + 0);

        if (pl.att) {
            // ---------------- QKV (cluster g) ----------------
            {
                const float rn = C.gain_bx(x0, x1, C.gain_fetch(P.in_ln[l]));
                const bool withhold = l == 0 && pl.k == P.debug_skip;   // failure tests only
                C.rows_1024(kClQRows * pl.r, kClQRows * (pl.r + 1), &S->bx[0][0][0], [&](int row, float v) {
                    // row's raw projection to every CTA of the cluster
                    const float val = v * rn;
                    if (!withhold)
                        for (uint32_t d = 0; d < (uint32_t)kCl; d++) st_async_v1(C.remote(&CS->qkv[row], d), val, C.remote(&CS->mb_q, d));
                });
            }
            QB_TRACE(TB + 1);
            C.dsmem_wait(&CS->mb_q, kQKVRows * 4, par, 10 * l + 2);
            // ---------------- ATT ----------------
            if (warp < 4) {   // warp w: q head 2g (0), q head 2g+1 (1), k (2), v (3); lane holds dims 4l..4l+3
                const int off = 128 * warp;
                uint2 gn = make_uint2(0u, 0u);
                if (warp < 3) gn = __ldg((const uint2*)((warp < 2 ? P.qn[l] : P.kn[l]) + 4 * lane));
                const float4 q4 = *(const float4*)&CS->qkv[off + 4 * lane];
                float x[4] = {q4.x, q4.y, q4.z, q4.w};
                if (warp < 3) {
                    const float tot = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
                    const float rr = 1.0f / sqrtf(tot * (1.0f / HEAD_DIM) + EPS);
                    x[0] = (x[0] * rr) * bf_lo(gn.x); x[1] = (x[1] * rr) * bf_hi(gn.x);
                    x[2] = (x[2] * rr) * bf_lo(gn.y); x[3] = (x[3] * rr) * bf_hi(gn.y);
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
                } else {
                    uint16_t b[4];
                    #pragma unroll
                    for (int e = 0; e < 4; e++) b[e] = f2bf(x[e]);
                    if (owner) {
                        const size_t at = ((size_t)l * kGroups * SEQ_LEN * HEAD_DIM) + pl.kvbase + (size_t)pos * HEAD_DIM + 4 * lane;
                        uint16_t* dst = (warp == 2 ? P.kc : P.vc) + at;
                        *(uint2*)dst = make_uint2((uint32_t)b[0] | ((uint32_t)b[1] << 16), (uint32_t)b[2] | ((uint32_t)b[3] << 16));
                        float* sm = warp == 2 ? S->kn : S->vn;
                        *(float4*)&sm[4 * lane] = make_float4(bf2f(b[0]), bf2f(b[1]), bf2f(b[2]), bf2f(b[3]));
                    }
                }
            }
            C.bar();
            {
                // as decode_kernel.cuh: warp w takes q head w / 8 and positions
                // 8 (w % 8) .. +7 of every K|V chunk; one online-softmax step per chunk
                const int hh = warp >> 3, sub = warp & 7;
                const int ti = 8 * sub + (lane >> 2), qq = lane & 3, xr4 = (ti & 15) << 2;
                float2 qv[16];
                #pragma unroll
                for (int jj = 0; jj < 16; jj++) qv[jj] = *(const float2*)&S->qs[128 * hh + 2 * (((4 * jj) ^ xr4) + qq)];
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
                        for (int jj = 0; jj < 16; jj++) {
                            const uint32_t w = kr[(4 * jj) ^ xr4];
                            c4[jj & 3] = fmaf(bf_lo(w), qv[jj].x, c4[jj & 3]);
                            c4[jj & 3] = fmaf(bf_hi(w), qv[jj].y, c4[jj & 3]);
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
                    if (mn != -INFINITY) {
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
                *(float4*)&S->w.comb[(size_t)warp * HEAD_DIM + 4 * lane] = make_float4(a0, a1, a2, a3);
                if (lane == 0) { S->am[warp] = m; S->al[warp] = lsum; }
                C.bar();
                if (tid < 2 * HEAD_DIM) {   // this CTA's partial of head h2, dim d -> every CTA of the cluster
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
                    float* base = &CS->part[pl.r][h2 * kHeadPart];
                    for (uint32_t dd = 0; dd < (uint32_t)kCl; dd++) {
                        const uint32_t mb = C.remote(&CS->mb_p, dd);
                        st_async_v1(C.remote(base + 4 + d, dd), A, mb);
                        if (d < 4) st_async_v1(C.remote(base + d, dd), d == 0 ? M : (d == 1 ? Ls : 0.f), mb);
                    }
                }
            }
            QB_TRACE(TB + 3);
            C.dsmem_wait(&CS->mb_p, kCl * kPartStride * 4, par, 10 * l + 4);
            C.bar();     // S->w.comb (read above) is reused below
            QB_TRACE(TB + 4);
            // ---------------- OPROJ ----------------
            {
                // warp w: head hh = w / 8; lane cc computes partial cc's weight, then
                // lanes (d, half) add the even / odd partials of dim d
                const int hh = warp >> 3;
                const float* b = &CS->part[lane & (kCl - 1)][hh * kHeadPart];
                const bool live = lane < kCl && b[1] > 0.f;
                const float mm = live ? b[0] : -INFINITY;
                const float M = warp_max(mm);
                const float e = live ? expf(mm - M) : 0.f;
                const float den = warp_sum(live ? b[1] * e : 0.f);
                const float wgt = e / den;
                const int d = 16 * (warp & 7) + (lane & 15), half = lane >> 4;
                float num = 0.f;
                #pragma unroll
                for (int i = 0; i < kCl / 2; i++) {
                    const int cc = 2 * i + half;
                    const float wc = __shfl_sync(0xffffffffu, wgt, cc);
                    num = fmaf(CS->part[cc][hh * kHeadPart + 4 + d], wc, num);
                }
                num += __shfl_xor_sync(0xffffffffu, num, 16);
                const float nx = __shfl_down_sync(0xffffffffu, num, 1);
                if (half == 0 && (d & 1) == 0) C.put_pair(&S->bo[0][0][0], hh * HEAD_DIM + d, num, nx);
            }
            C.bar();
            {
                uint64_t* y = P.yw + (size_t)(l * kGroups + g) * DIM;
                const int t = warp & 3, lr = lane & 15;
                for (int r0 = kClORows * pl.r; r0 < kClORows * (pl.r + 1); r0 += kRowsWo) {
                    const int cnt = min(kRowsWo, kClORows * (pl.r + 1) - r0);
                    const uint8_t* ch = C.chunk(0);
                    const int row = 16 * t + lr;
                    uint32_t ta[1] = {smem_addr(ch + (size_t)(row < cnt ? row : 0) * kStrideWo) + (lane >> 4) * 16};
                    float d[1][4] = {{0.f, 0.f, 0.f, 0.f}};
                    C.template mma_tiles<1>(ta, &S->bo[0][0][0], 4 * (warp >> 2), 4, d);
                    float* red = C.next_red();
                    C.put_red(red, 0, d[0]);
                    C.release(1);
                    C.bar();
                    if (tid < cnt) {
                        const int tt = tid >> 4, ri = tid & 15;
                        const float v = ((red[tt * 32 + ri] + red[(tt + 4) * 32 + ri]) + red[(tt + 8) * 32 + ri]) + red[(tt + 12) * 32 + ri];
                        xw_store(y + r0 + tid, v, seq);
                    }
                }
            }
            QB_TRACE(TB + 5);
        }

        // ---------------- MLP ----------------
        {
            const uint32_t g2 = C.gain_fetch(P.post_ln[l]);
            x0 = S->xres[j]; x1 = S->xres[j + 1];        // x_l (reloaded: not kept live across the attention stage)
            float yv[2 * kGroups];
            C.template gather<kGroups>([&](int gg) { return P.yw + ((size_t)l * kGroups + gg) * DIM + j; }, (1u << kGroups) - 1u, yv,
                                       10 * l + 6);
            #pragma unroll
            for (int gg = 0; gg < kGroups; gg++) { x0 += yv[2 * gg]; x1 += yv[2 * gg + 1]; }
            S->xres[j] = x0; S->xres[j + 1] = x1;        // x_mid
            const float rn = C.gain_bx(x0, x1, g2);
            QB_TRACE(TB + 6);
            // gate|up units, 7 per chunk, two chunks per round (as decode_kernel.cuh)
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
                if (tid < n) {
                    const int t = tid < kUnitsGU ? 0 : 1, uu = tid - t * kUnitsGU;
                    float gt = 0.f, up = 0.f;
                    #pragma unroll
                    for (int w = 0; w < kNCW; w++) { gt += red[w * 32 + 16 * t + uu]; up += red[w * 32 + 16 * t + kUnitsGU + uu]; }
                    gt *= rn; up *= rn;
                    S->hl[u + tid - pl.ha] = (gt / (1.0f + expf(-gt))) * up;
                }
            }
            C.bar();     // S->hl complete
            QB_TRACE(TB + 7);
            // W_down h over this CTA's units: thread t owns outputs 2t, 2t+1
            float a0 = 0.f, a1 = 0.f;
            for (int u = pl.ha; u < pl.hb; u += kRowsWdT) {
                const int n = min(kRowsWdT, pl.hb - u);
                const uint8_t* ch = C.chunk(0);
                const float* hs = &S->hl[u - pl.ha];
                #pragma unroll 4
                for (int i = 0; i < n; i++) {
                    const uint32_t w = *(const uint32_t*)(ch + (size_t)i * 2 * DIM + 4 * tid);
                    const float h = hs[i];
                    a0 = fmaf(bf_lo(w), h, a0);
                    a1 = fmaf(bf_hi(w), h, a1);
                }
                C.release(1);
            }
            // rows [128d, 128d+128) go to CTA d of the cluster
            {
                const uint32_t d = (uint32_t)(j / kClORows);
                st_async_v2(C.remote(&CS->xred[pl.r][j - kClORows * (int)d], d), a0, a1, C.remote(&CS->mb_r, d));
            }
            C.dsmem_wait(&CS->mb_r, kCl * kClORows * 4, par, 10 * l + 8);
            QB_TRACE(TB + 8);
            if (tid < kClORows) {   // the cluster's sum for row 128 r + tid, in rank order
                float sum = 0.f;
                #pragma unroll
                for (int s2 = 0; s2 < kCl; s2++) sum += CS->xred[s2][tid];
                xw_store(xpw(l + 1, pl.k) + kClORows * pl.r + tid, sum, seq);
            }
        }
        QB_TRACE(TB + 9);
    }

    // ---------------- HEAD ----------------
    C.flush();
    C.tl = N_LAYERS;
    const bool head = pl.head;
    const bool greedy = (P.in->temperature == 0.0f || P.in->top_k == 1);
    const int K = greedy ? 1 : min(P.in->top_k, kMaxCand);
    if (head) {
        const uint32_t g2 = C.gain_fetch(P.final_ln);
        float x0 = S->xres[j], x1 = S->xres[j + 1];
        {
            const int n1 = min(pl.ncl, 8), n2 = pl.ncl - n1;
            float v[16];
            C.template gather<8>([&](int i) { return xpw(N_LAYERS, i) + j; }, (1u << n1) - 1u, v, 10 * N_LAYERS);
            #pragma unroll
            for (int i = 0; i < 8; i++) if (i < n1) { x0 += v[2 * i]; x1 += v[2 * i + 1]; }
            if (n2 > 0) {
                C.template gather<8>([&](int i) { return xpw(N_LAYERS, 8 + i) + j; }, (1u << n2) - 1u, v, 10 * N_LAYERS);
                #pragma unroll
                for (int i = 0; i < 8; i++) if (i < n2) { x0 += v[2 * i]; x1 += v[2 * i + 1]; }
            }
        }
        const float ss = C.block_sum(x0 * x0 + x1 * x1);
        QB_TRACE(kTrHead);
        const int va = pl.va;
        const bool wl = (flags & kFlagWriteLogits) != 0;
        {
            float* xs = reinterpret_cast<float*>(&S->bx[0][0][0]);
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
}

// kTr: the tracing build.  Launched with cluster dimension kCl; grid = clusters x kCl.
template <bool kTr>
__global__ void __launch_bounds__(kClThreads, 1) decode_cluster_kernel(const __grid_constant__ DecodeParams P) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    ClSmem* CS = reinterpret_cast<ClSmem*>(smem + (size_t)kSlots * kSlotBytes);
    DecodeSmem* S = &CS->base;
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int s = 0; s < kSlots; s++) { mbar_init(&S->full[s], 1); mbar_init(&S->empty[s], kNCW); }
        mbar_init(&CS->mb_q, 1); mbar_init(&CS->mb_p, 1); mbar_init(&CS->mb_r, 1);
        S->abort = 0;
        S->hfail = 0;
        S->copied = 0;
        fence_barrier_init();
    }
    // every CTA's barriers exist before any peer sends to them
    cluster_sync_all();
    const int k = (int)cluster_id_x(), r = (int)cluster_ctarank(), ncl = (int)cluster_count_x();
    const int c = k * kCl + r;
    const int flags = P.in->flags;
    const int pos = min(max(P.in->pos, 0), SEQ_LEN - 1);
    int token = (flags & kFlagPromptToken) ? P.prompt[pos] : P.in->token;
    if (token < 0 || token >= VOCAB_SIZE) {
        if (tid == 0 && c == 0) { atomicOr(&P.out->err, 8u); atomicExch(&P.out->err_where, -200); }
        token = 0;
    }
    const uint32_t seq = P.out->seq;
    if (tid == 0) CS->pl = cl_make_plan(P, k, r, ncl, pos, flags);
    __syncthreads();
    const ClPlan& pl = CS->pl;
    if ((tid >> 5) == kNCW) {
        if ((tid & 31) == 0) cl_producer(P, ring, S, c, pl);
    } else {
        cl_consumer<kTr>(P, ring, CS, c, pl, token, pos, flags, seq);
    }
    __syncwarp();
    // no CTA leaves while a peer may still write into its shared memory
    cluster_sync_all();
}

}  // namespace qb
