// prefill_kernels.cuh — the non-GEMM steps of the prompt pass (a16: no
// reference counterpart; the reference runs forward() once per prompt token,
// main.cu:141-145).  Rows are prompt positions pos0 + r; the contractions run
// on the tensor cores (gemm_tc.cuh) with every activation split into three bf16
// parts (hi, mid, lo: exact to fp32 precision) laid side by side along K, so
// the fp32 numerics of the decode chain carry over.
//
// Per layer (qwen_model.cuh:791-832 for one row, here for all rows at once):
//   norm_split    X (+= the previous GEMM's output) -> RMSNorm -> As = [hi|mid|lo]
//   GEMM          As . [Wq; Wk; Wv]^T -> Y (fp32)
//   qkv_post      QK-norm + RoPE; q -> Q (fp32); k, v -> the bf16 KV cache
//   attention     causal GQA over the cache on the tensor cores -> As (the
//                 output split into three bf16 parts);  GEMM As . Wo^T -> Y
//   norm_split    X += Y -> RMSNorm (post_attention_layernorm) -> As
//   GEMM          As . Wg^T, As . Wu^T -> Y;  swiglu_split -> As
//   GEMM          As . Wd^T -> Y   (added into X by the next layer's norm_split)
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "../host/config.h"

namespace qb {
namespace pf {

constexpr int kMaxRows = 2048;          // prompt rows per pass
constexpr int kAttBlock = 64;           // query rows and key positions per attention tile

__device__ __forceinline__ void split3(float v, uint16_t& h, uint16_t& m, uint16_t& l) {
    h = f2bf(v);
    const float r = v - bf2f(h);
    m = f2bf(r);
    l = f2bf(r - bf2f(m));
}
// The attention output as the O projection's A operand: value(s) at column col
// of an As row whose three parts are Q_DIM columns apart.
__device__ __forceinline__ void put_split2(uint16_t* as_row, int col, float a, float b) {
    uint32_t h, m, l;
    split3x2(a, b, h, m, l);
    *(uint32_t*)(as_row + col) = h;
    *(uint32_t*)(as_row + Q_DIM + col) = m;
    *(uint32_t*)(as_row + 2 * Q_DIM + col) = l;
}
__device__ __forceinline__ void put_split1(uint16_t* as_row, int col, float v) {
    uint16_t h, m, l;
    split3(v, h, m, l);
    as_row[col] = h;
    as_row[Q_DIM + col] = m;
    as_row[2 * Q_DIM + col] = l;
}
// v (4 consecutive columns c..c+3 of a K-wide row) -> the first `parts` (1-3)
// part blocks of As row r (the parts the next GEMM reads)
__device__ __forceinline__ void put_split4(uint16_t* As_row, int K, int c, float4 v, int parts) {
    uint16_t h[4], m[4], l[4];
    split3(v.x, h[0], m[0], l[0]); split3(v.y, h[1], m[1], l[1]);
    split3(v.z, h[2], m[2], l[2]); split3(v.w, h[3], m[3], l[3]);
    *(uint2*)(As_row + c) = make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
    if (parts > 1) *(uint2*)(As_row + K + c) = make_uint2(m[0] | ((uint32_t)m[1] << 16), m[2] | ((uint32_t)m[3] << 16));
    if (parts > 2) *(uint2*)(As_row + 2 * K + c) = make_uint2(l[0] | ((uint32_t)l[1] << 16), l[2] | ((uint32_t)l[3] << 16));
}

// X[r] = embed[token[r]] (fp32) for r < m; 0 for m <= r < rows.
__global__ void embed_kernel(const uint16_t* __restrict__ embed, const int* __restrict__ tokens, int m, int rows, float* __restrict__ X) {
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x, t = threadIdx.x;   // 256 threads x 4 columns
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < m) {
        const int tok = min(max(tokens[r], 0), VOCAB_SIZE - 1);
        const uint2 w = *(const uint2*)(embed + (size_t)tok * DIM + 4 * t);
        v = make_float4(bf_lo(w.x), bf_hi(w.x), bf_lo(w.y), bf_hi(w.y));
    }
    *(float4*)(X + (size_t)r * DIM + 4 * t) = v;
}

// a += p[s * stride] for s = 1 .. n - 1, in that order (the partial sums of a
// GEMM whose K was split; p[0] is already in a): the loads go out eight at a
// time, so n partials cost about n / 8 round trips to L2 instead of n.
__device__ __forceinline__ void add_partials(float4& a, const float* p, size_t stride, int n) {
    for (int s0 = 1; s0 < n; s0 += 8) {
        float4 b[8];
        #pragma unroll
        for (int i = 0; i < 8; i++)
            if (s0 + i < n) b[i] = *reinterpret_cast<const float4*>(p + (size_t)(s0 + i) * stride);
        #pragma unroll
        for (int i = 0; i < 8; i++)
            if (s0 + i < n) { a.x += b[i].x; a.y += b[i].y; a.z += b[i].z; a.w += b[i].w; }
    }
}

// One block (256 threads, 4 columns each) per row: X[r] += add[r] (if add),
// then RMSNorm with `gain` (the decode chain's formula: (x * (1 / sqrt(mean(x^2)
// + eps))) * g) into As as `parts` bf16 parts.  `add` may hold n_add partial sums side by side
// (columns s * DIM ..): a GEMM whose K was split; they are added in order
// s = 0, 1, ... and then to X.
__global__ void __launch_bounds__(256) norm_split_kernel(float* __restrict__ X, const float* __restrict__ add, int ld_add, int n_add,
                                                         const uint16_t* __restrict__ gain, uint16_t* __restrict__ As, int ld_as, int rows,
                                                         int parts) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float part[8];
    const int r = blockIdx.x, t = threadIdx.x, c = 4 * t;
    if (r >= rows) return;
    float* x = X + (size_t)r * DIM;
    float4 v = *(const float4*)(x + c);
    if (add) {
        const float* ar = add + (size_t)r * ld_add + c;
        float4 a = *(const float4*)ar;
        add_partials(a, ar, DIM, n_add);
        v.x += a.x; v.y += a.y; v.z += a.z; v.w += a.w;
        *(float4*)(x + c) = v;
    }
    float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
    if ((t & 31) == 0) part[t >> 5] = ss;
    __syncthreads();
    ss = 0.f;
    #pragma unroll
    for (int w = 0; w < 8; w++) ss += part[w];
    const float rs = 1.0f / sqrtf(ss * (1.0f / DIM) + EPS);
    const uint2 g = *(const uint2*)(gain + c);
    const float4 y = make_float4((v.x * rs) * bf_lo(g.x), (v.y * rs) * bf_hi(g.x), (v.z * rs) * bf_lo(g.y), (v.w * rs) * bf_hi(g.y));
    put_split4(As + (size_t)r * ld_as, DIM, c, y, parts);
}

// Y: gate | up (n_add partial sums of both, part_stride columns apart, added in order)
__global__ void swiglu_split_kernel(const float* __restrict__ Y, int ld_y, int n_add, int part_stride, uint16_t* __restrict__ As, int ld_as,
                                    int rows, int parts) {
    pdl_launch_dependents();
    pdl_wait();
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int q = HIDDEN_DIM / 4;
    if (i >= (size_t)rows * q) return;
    const int r = (int)(i / q), c = (int)(i % q) * 4;
    const float* yr = Y + (size_t)r * ld_y + c;
    float4 g = *(const float4*)yr, u = *(const float4*)(yr + HIDDEN_DIM);
    add_partials(g, yr, part_stride, n_add);
    add_partials(u, yr + HIDDEN_DIM, part_stride, n_add);
    const float4 h = make_float4((g.x / (1.0f + expf(-g.x))) * u.x, (g.y / (1.0f + expf(-g.y))) * u.y,
                                 (g.z / (1.0f + expf(-g.z))) * u.z, (g.w / (1.0f + expf(-g.w))) * u.w);
    put_split4(As + (size_t)r * ld_as, HIDDEN_DIM, c, h, parts);
}

// q/k/v of row r (position pos0 + r), one warp per (row, slot): slots 0..15 q
// heads, 16..23 k heads, 24..31 v heads; lane l holds dims 4l..4l+3.  QK-norm
// (qwen_model.cuh:215-245) and NeoX RoPE (:327-364) as in the decode chain; k
// and v go to the bf16 cache (rows < m only), q to Q (fp32).
// Rows r < m are prompt positions pos0 + r of one sequence (pos_rows NULL), or
// (batched decode) one position pos_rows[r] each of sequence r, whose cache
// starts row_cache_stride elements after sequence r - 1's.
// Y may hold n_add partial sums (a GEMM with split K) part_stride columns apart;
// they are added in order.
__global__ void qkv_post_kernel(const float* __restrict__ Y, int ld_y, int n_add, int part_stride, int m, int rows, int pos0,
                                const uint16_t* __restrict__ qn, const uint16_t* __restrict__ kn, const float* __restrict__ rope,
                                float* __restrict__ Q, uint16_t* __restrict__ kc_l, uint16_t* __restrict__ vc_l,
                                const int* __restrict__ pos_rows, size_t row_cache_stride) {
    pdl_launch_dependents();
    pdl_wait();
    const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int r = w >> 5, slot = w & 31;
    if (r >= rows) return;
    const int pos = pos_rows ? (r < m ? min(max(pos_rows[r], 0), SEQ_LEN - 1) : 0) : min(pos0 + r, SEQ_LEN - 1);
    const int col = slot < 16 ? 128 * slot : (slot < 24 ? Q_DIM + 128 * (slot - 16) : Q_DIM + KV_DIM + 128 * (slot - 24));
    const float* yr = Y + (size_t)r * ld_y + col + 4 * lane;
    float4 a = *(const float4*)yr;
    add_partials(a, yr, part_stride, n_add);
    float x[4] = {a.x, a.y, a.z, a.w};
    if (slot < 24) {
        const uint2 gn = *(const uint2*)((slot < 16 ? qn : kn) + 4 * lane);
        const float tot = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
        const float rs = 1.0f / sqrtf(tot * (1.0f / HEAD_DIM) + EPS);
        x[0] = (x[0] * rs) * bf_lo(gn.x); x[1] = (x[1] * rs) * bf_hi(gn.x);
        x[2] = (x[2] * rs) * bf_lo(gn.y); x[3] = (x[3] * rs) * bf_hi(gn.y);
        const float* cs = rope + (size_t)pos * HEAD_DIM;
        const int j0 = (4 * lane) & 63;   // this lane's 4 rotation angles, cos and sin as one 16-byte load each
        const float4 c4 = *(const float4*)(cs + j0), s4 = *(const float4*)(cs + 64 + j0);
        const float cj[4] = {c4.x, c4.y, c4.z, c4.w}, sj[4] = {s4.x, s4.y, s4.z, s4.w};
        #pragma unroll
        for (int e = 0; e < 4; e++) {
            const float pv = __shfl_xor_sync(0xffffffffu, x[e], 16);
            x[e] = 4 * lane + e < 64 ? (x[e] * cj[e] - pv * sj[e]) : (pv * sj[e] + x[e] * cj[e]);
        }
    }
    if (slot < 16) {
        *(float4*)(Q + (size_t)r * Q_DIM + 128 * slot + 4 * lane) = make_float4(x[0], x[1], x[2], x[3]);
    } else if (r < m) {
        const int h = slot < 24 ? slot - 16 : slot - 24;
        uint16_t* dst = (slot < 24 ? kc_l : vc_l) + (pos_rows ? (size_t)r * row_cache_stride : 0) + ((size_t)h * SEQ_LEN + pos) * HEAD_DIM +
                        4 * lane;
        *(uint2*)dst = make_uint2((uint32_t)f2bf(x[0]) | ((uint32_t)f2bf(x[1]) << 16), (uint32_t)f2bf(x[2]) | ((uint32_t)f2bf(x[3]) << 16));
    }
}

// The prompt's last row after the last layer: x = X[row] + the down
// projection's n_add partial sums, then the final RMSNorm (the decode chain's
// formula, qwen_model.cuh:836-839) into xn (fp32).  One block of 256 threads.
__global__ void final_norm_row_kernel(const float* __restrict__ X, const float* __restrict__ add, int ld_add, int n_add,
                                      const uint16_t* __restrict__ gain, int row, float* __restrict__ xn) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float part[8];
    const int t = threadIdx.x, c = 4 * t;
    float4 v = *(const float4*)(X + (size_t)row * DIM + c);
    const float* ar = add + (size_t)row * ld_add + c;
    float4 a = *(const float4*)ar;
    add_partials(a, ar, DIM, n_add);
    v.x += a.x; v.y += a.y; v.z += a.z; v.w += a.w;
    float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
    if ((t & 31) == 0) part[t >> 5] = ss;
    __syncthreads();
    ss = 0.f;
    #pragma unroll
    for (int w = 0; w < 8; w++) ss += part[w];
    const float rs = 1.0f / sqrtf(ss * (1.0f / DIM) + EPS);
    const uint2 g = *(const uint2*)(gain + c);
    *(float4*)(xn + c) = make_float4((v.x * rs) * bf_lo(g.x), (v.y * rs) * bf_hi(g.x), (v.z * rs) * bf_lo(g.y), (v.w * rs) * bf_hi(g.y));
}

// logits[r] = LM[r] . xn for r in [r0, r1): fp32 input, bf16 weights, fp32
// accumulation (the decode chain's head, qwen_model.cuh:841-845).  One warp per
// row, two rows in flight per warp; lane l holds xn[8 (l + 32 i) .. +7].
__global__ void __launch_bounds__(256) lm_head_f32_kernel(const uint16_t* __restrict__ lm, const float* __restrict__ xn, int r0, int r1,
                                                          float* __restrict__ logits) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    float xr[4][8];
    #pragma unroll
    for (int i = 0; i < 4; i++) {
        const float4 a = *(const float4*)(xn + 8 * (lane + 32 * i)), b = *(const float4*)(xn + 8 * (lane + 32 * i) + 4);
        xr[i][0] = a.x; xr[i][1] = a.y; xr[i][2] = a.z; xr[i][3] = a.w;
        xr[i][4] = b.x; xr[i][5] = b.y; xr[i][6] = b.z; xr[i][7] = b.w;
    }
    const int warps = gridDim.x * (blockDim.x >> 5);
    for (int r = r0 + 2 * (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)); r < r1; r += 2 * warps) {
        const bool two = r + 1 < r1;
        const uint4* w0 = reinterpret_cast<const uint4*>(lm + (size_t)r * DIM);
        const uint4* w1 = reinterpret_cast<const uint4*>(lm + (size_t)(two ? r + 1 : r) * DIM);
        uint4 a[4], b[4];
        #pragma unroll
        for (int i = 0; i < 4; i++) { a[i] = __ldcs(w0 + lane + 32 * i); b[i] = __ldcs(w1 + lane + 32 * i); }
        float s0 = 0.f, s1 = 0.f;
        #pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t wa[4] = {a[i].x, a[i].y, a[i].z, a[i].w}, wb[4] = {b[i].x, b[i].y, b[i].z, b[i].w};
            #pragma unroll
            for (int j = 0; j < 4; j++) {
                s0 = fmaf(bf_lo(wa[j]), xr[i][2 * j], s0); s0 = fmaf(bf_hi(wa[j]), xr[i][2 * j + 1], s0);
                s1 = fmaf(bf_lo(wb[j]), xr[i][2 * j], s1); s1 = fmaf(bf_hi(wb[j]), xr[i][2 * j + 1], s1);
            }
        }
        s0 = warp_sum(s0);
        s1 = warp_sum(s1);
        if (lane == 0) {
            logits[r] = s0;
            if (two) logits[r + 1] = s1;
        }
    }
}

// ---------------------------------------------------------------------------
// Batched decode: one query row per sequence.
// ---------------------------------------------------------------------------
// Row r (sequence r, its position pos_rows[r]; its cache already holds that
// position) against keys 0 .. pos_rows[r] of its own cache, for the two q heads
// of KV head hk: the decode chain's attention (qwen_model.cuh:809-810,
// attention_gpu) in fp32 — q fp32, K and V bf16, scores / sqrt(d), online
// softmax.  Block b: row b / (N_KV_HEADS S), KV head (b / S) % N_KV_HEADS, key
// split b % S of S (the keys cut into S contiguous ranges, so small batches
// still fill the GPU).  8 warps take keys 8 at a time (four lanes per key, 32
// dims each; the 8 keys' V rows are loaded with their K rows), one softmax
// step per warp and head per 8 keys; P.V with lane l holding dims 4l .. 4l+3.
// The warps are merged in shared memory; with S = 1 the result goes to As (the
// O projection's input, three bf16 parts), else (max, sum, accumulator) per
// head to part[b] for attention_combine_kernel.
constexpr int kDecAttThreads = 256;
constexpr int kPartFloats = 2 * (HEAD_DIM + 2);   // per block: per head 128 accumulators, max, sum
__global__ void __launch_bounds__(kDecAttThreads) attention_rows_kernel(const float* __restrict__ Q, const int* __restrict__ pos_rows,
                                                                        const uint16_t* __restrict__ kc_l, const uint16_t* __restrict__ vc_l,
                                                                        size_t row_cache_stride, int S, uint16_t* __restrict__ As,
                                                                        int ld_as, float* __restrict__ part) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ float qs[2][HEAD_DIM];
    __shared__ float wm[8][2], wl[8][2];
    __shared__ __align__(16) float wacc[8][2][HEAD_DIM];
    const int sp = blockIdx.x % S, hk = (blockIdx.x / S) % N_KV_HEADS, r = blockIdx.x / (S * N_KV_HEADS);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, kq = lane >> 2, qq = lane & 3;
    const int npos = min(max(pos_rows[r], 0), SEQ_LEN - 1) + 1;
    const int per = (npos + S - 1) / S, kb0 = sp * per, kb1 = min(npos, kb0 + per);
    const float sqrt_hd = sqrtf((float)HEAD_DIM);
    qs[tid >> 7][tid & 127] = Q[(size_t)r * Q_DIM + 128 * (2 * hk) + tid];
    __syncthreads();
    float qr[2][32];
    #pragma unroll
    for (int j = 0; j < 32; j++) { qr[0][j] = qs[0][32 * qq + j]; qr[1][j] = qs[1][32 * qq + j]; }
    const size_t base = (size_t)r * row_cache_stride + (size_t)hk * SEQ_LEN * HEAD_DIM;
    const uint16_t* kb = kc_l + base;
    const uint16_t* vb = vc_l + base;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    for (int k0 = kb0 + 8 * warp; k0 < kb1; k0 += 64) {
        const int key = k0 + kq;
        const bool valid = key < kb1;
        uint4 kw[4];
        uint2 vw[8];
        #pragma unroll
        for (int i = 0; i < 4; i++) kw[i] = valid ? reinterpret_cast<const uint4*>(kb + (size_t)key * HEAD_DIM + 32 * qq)[i] : make_uint4(0, 0, 0, 0);
        #pragma unroll
        for (int i = 0; i < 8; i++)
            vw[i] = k0 + i < kb1 ? *reinterpret_cast<const uint2*>(vb + (size_t)(k0 + i) * HEAD_DIM + 4 * lane) : make_uint2(0u, 0u);
        float s[2] = {0.f, 0.f};
        #pragma unroll
        for (int i = 0; i < 4; i++) {
            const uint32_t w[4] = {kw[i].x, kw[i].y, kw[i].z, kw[i].w};
            #pragma unroll
            for (int e = 0; e < 4; e++) {
                #pragma unroll
                for (int h = 0; h < 2; h++) {
                    s[h] = fmaf(bf_lo(w[e]), qr[h][8 * i + 2 * e], s[h]);
                    s[h] = fmaf(bf_hi(w[e]), qr[h][8 * i + 2 * e + 1], s[h]);
                }
            }
        }
        float p[2];
        #pragma unroll
        for (int h = 0; h < 2; h++) {
            s[h] += __shfl_xor_sync(0xffffffffu, s[h], 1);
            s[h] += __shfl_xor_sync(0xffffffffu, s[h], 2);
            s[h] = valid ? s[h] / sqrt_hd : -INFINITY;
            float mx = fmaxf(s[h], __shfl_xor_sync(0xffffffffu, s[h], 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mn = fmaxf(m[h], mx);   // finite: key k0 is valid
            const float sc = expf(m[h] - mn);
            p[h] = valid ? expf(s[h] - mn) : 0.f;
            float ps = p[h] + __shfl_xor_sync(0xffffffffu, p[h], 4);
            ps += __shfl_xor_sync(0xffffffffu, ps, 8);
            ps += __shfl_xor_sync(0xffffffffu, ps, 16);
            l[h] = fmaf(l[h], sc, ps);
            #pragma unroll
            for (int e = 0; e < 4; e++) acc[h][e] *= sc;
            m[h] = mn;
        }
        #pragma unroll
        for (int i = 0; i < 8; i++) {
            const float p0 = __shfl_sync(0xffffffffu, p[0], 4 * i), p1 = __shfl_sync(0xffffffffu, p[1], 4 * i);
            const float v[4] = {bf_lo(vw[i].x), bf_hi(vw[i].x), bf_lo(vw[i].y), bf_hi(vw[i].y)};
            #pragma unroll
            for (int e = 0; e < 4; e++) { acc[0][e] = fmaf(p0, v[e], acc[0][e]); acc[1][e] = fmaf(p1, v[e], acc[1][e]); }
        }
    }
    if (lane == 0) { wm[warp][0] = m[0]; wm[warp][1] = m[1]; wl[warp][0] = l[0]; wl[warp][1] = l[1]; }
    #pragma unroll
    for (int h = 0; h < 2; h++) *(float4*)&wacc[warp][h][4 * lane] = make_float4(acc[h][0], acc[h][1], acc[h][2], acc[h][3]);
    __syncthreads();
    const int h = tid >> 7, d = tid & 127;
    float M = -INFINITY;
    #pragma unroll
    for (int w = 0; w < 8; w++) M = fmaxf(M, wm[w][h]);
    float L = 0.f, A = 0.f;
    #pragma unroll
    for (int w = 0; w < 8; w++) {
        const float sc = wm[w][h] == -INFINITY ? 0.f : expf(wm[w][h] - M);
        L = fmaf(wl[w][h], sc, L);
        A = fmaf(wacc[w][h][d], sc, A);
    }
    if (S == 1) {
        put_split1(As + (size_t)r * ld_as, 128 * (2 * hk + h) + d, A / L);
    } else {
        float* pb = part + (size_t)blockIdx.x * kPartFloats + h * (HEAD_DIM + 2);
        pb[d] = A;
        if (d == 0) { pb[HEAD_DIM] = M; pb[HEAD_DIM + 1] = L; }
    }
}

// Merges the S key ranges of attention_rows_kernel: block b = (row, KV head),
// thread (h, d) -> As.  An empty range (max -inf) contributes nothing.
__global__ void __launch_bounds__(kDecAttThreads) attention_combine_kernel(const float* __restrict__ part, int S, uint16_t* __restrict__ As,
                                                                           int ld_as) {
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x / N_KV_HEADS, hk = blockIdx.x % N_KV_HEADS, h = threadIdx.x >> 7, d = threadIdx.x & 127;
    const float* pb = part + (size_t)blockIdx.x * S * kPartFloats + h * (HEAD_DIM + 2);
    float M = -INFINITY;
    for (int i = 0; i < S; i++) M = fmaxf(M, pb[(size_t)i * kPartFloats + HEAD_DIM]);
    float L = 0.f, A = 0.f;
    for (int i = 0; i < S; i++) {
        const float mi = pb[(size_t)i * kPartFloats + HEAD_DIM];
        const float sc = mi == -INFINITY ? 0.f : expf(mi - M);
        L = fmaf(pb[(size_t)i * kPartFloats + HEAD_DIM + 1], sc, L);
        A = fmaf(pb[(size_t)i * kPartFloats + d], sc, A);
    }
    put_split1(As + (size_t)r * ld_as, 128 * (2 * hk + h) + d, A / L);
}

// Top-k of every row of fp32 logits, in levels: each warp takes a group of 512
// consecutive entries of a row and keeps its k best (value descending, ties to
// the smaller id: each entry's key is its value in an order-preserving uint32,
// and the k-th best key is found by a radix select over the 32 key bits, one
// warp-wide count per bit), writing them in entry order.  The next level runs
// the same over the concatenated survivors until one group is left; because
// every level keeps entry order and level one's entries are in id order, a
// position in a survivor list orders ties exactly as the id does.  k = 1 is a
// plain warp argmax.  NaN ranks below every number; -0 counts as +0.  k <= 64
// (at most 512 / 8 per group).
constexpr int kTopkGroup = 512;                 // entries per warp
constexpr int kTopkPerLane = kTopkGroup / 32;
constexpr int kTopkWarps = 8;                   // warps per block

__device__ __forceinline__ uint32_t order_key(float x) {
    if (x != x) return 0u;
    if (x == 0.f) x = 0.f;
    const uint32_t u = __float_as_uint(x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
    if (k == 0u) return -INFINITY;
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Level over `n` entries per row: logits (kFirst: fp32, ids = columns) or the
// keys / ids of the previous level (rows in_ld apart).  Writes k survivors per
// group to out_key / out_id (rows out_ld apart), or, when one group covers the
// row (n <= 512), the k values and ids to fin_v / fin_i (rows k apart; an id
// past the row, possible only for rows with fewer than k numbers, reads 0).
template <bool kFirst>
__global__ void __launch_bounds__(32 * kTopkWarps) topk_level_kernel(const float* __restrict__ logits, const uint32_t* __restrict__ in_key,
                                                                     const int* __restrict__ in_id, int in_ld, int n, int k,
                                                                     uint32_t* __restrict__ out_key, int* __restrict__ out_id, int out_ld,
                                                                     float* __restrict__ fin_v, int* __restrict__ fin_i, int n_ids) {
    const int lane = threadIdx.x & 31;
    const int groups = (n + kTopkGroup - 1) / kTopkGroup;
    const int g = blockIdx.x * kTopkWarps + (threadIdx.x >> 5);
    if (g >= groups) return;
    const int row = blockIdx.y;
    const size_t rb = (size_t)row * in_ld;
    const int base = g * kTopkGroup;
    uint32_t key[kTopkPerLane];
    int idv[kTopkPerLane];   // ids, loaded with the keys (a later level's ids are not its positions)
    #pragma unroll
    for (int e = 0; e < kTopkPerLane; e++) {
        const int j = base + e * 32 + lane;
        key[e] = j < n ? (kFirst ? order_key(logits[rb + j]) : in_key[rb + j]) : 0u;
        idv[e] = j < n ? (kFirst ? j : in_id[rb + j]) : 0x7fffffff;
    }
    const bool fin = groups == 1;
    auto put = [&](int slot, uint32_t kv, int id) {
        if (fin) {
            fin_v[(size_t)row * k + slot] = key_value(kv);
            fin_i[(size_t)row * k + slot] = id < n_ids ? id : 0;
        } else {
            out_key[(size_t)row * out_ld + (size_t)g * k + slot] = kv;
            out_id[(size_t)row * out_ld + (size_t)g * k + slot] = id;
        }
    };
    if (k == 1) {   // argmax: best key, first position among equals
        uint32_t bk = key[0];
        int bp = lane, bid = idv[0];
        #pragma unroll
        for (int e = 1; e < kTopkPerLane; e++)
            if (key[e] > bk) { bk = key[e]; bp = e * 32 + lane; bid = idv[e]; }
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint32_t k2 = __shfl_xor_sync(0xffffffffu, bk, o);
            const int p2 = __shfl_xor_sync(0xffffffffu, bp, o);
            const int i2 = __shfl_xor_sync(0xffffffffu, bid, o);
            if (k2 > bk || (k2 == bk && p2 < bp)) { bk = k2; bp = p2; bid = i2; }
        }
        if (lane == 0) put(0, bk, bid);
        return;
    }
    uint32_t T = 0u;
    int need = k;
    #pragma unroll 1
    for (int bit = 31; bit >= 0; bit--) {
        const uint32_t m = ~0u << bit, cand = T | (1u << bit);
        int cnt = 0;
        #pragma unroll
        for (int e = 0; e < kTopkPerLane; e++) cnt += (key[e] & m) == cand;
        cnt = __reduce_add_sync(0xffffffffu, cnt);
        if (cnt >= need) T = cand;
        else need -= cnt;
    }
    // T: the k-th best key of the group; take every key above it and the first `need` equal to it
    const uint32_t lt = (1u << lane) - 1u;
    int taken = 0, eq_seen = 0;
    #pragma unroll
    for (int e = 0; e < kTopkPerLane; e++) {
        const uint32_t beq = __ballot_sync(0xffffffffu, key[e] == T);
        const bool sel = key[e] > T || (key[e] == T && eq_seen + __popc(beq & lt) < need);
        eq_seen += __popc(beq);
        const uint32_t bsel = __ballot_sync(0xffffffffu, sel);
        if (sel) put(taken + __popc(bsel & lt), key[e], idv[e]);
        taken += __popc(bsel);
    }
}

// ---------------------------------------------------------------------------
// Causal GQA attention on the tensor cores (mma.m16n8k16, bf16 in, fp32
// accumulate).  One CTA per (64 query rows, KV head): its 8 warps cover both q
// heads of the group (warp w: head 2 hk + w / 4, rows 16 (w % 4) .. +15), so
// each K/V tile is loaded once for two heads.  S = Q K^T with Q split into
// kAttParts bf16 parts (K is bf16 in the cache: exact), online softmax on the
// accumulator fragments in base 2 with the 1/sqrt(d) scale folded into the
// exponent, O += P V with P split into kAttParts bf16 parts (V exact).  K/V tiles are double-buffered (cp.async, 16-byte
// row pads: conflict-free ldmatrix, V through .trans); the CTAs with the most
// causal work are numbered first.
// ---------------------------------------------------------------------------
constexpr int kTcRowE = HEAD_DIM + 8;     // padded smem row, elements (272 B)
constexpr int kTcThreads = 256;
// bf16 parts of Q and P in the attention products: 2 (hi + mid) keeps 16
// mantissa bits of each (relative error <= 2^-17); K and V are bf16 already
constexpr int kAttParts = 2;

struct AttTcSmem {
    uint16_t q[2][kAttParts][kAttBlock][kTcRowE];    // per q head: the bf16 parts (hi, mid) of the 64 query rows
    uint16_t k[2][kAttBlock][kTcRowE];       // two K tiles (double buffer)
    uint16_t v[2][kAttBlock][kTcRowE];
};
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr) : "memory");
}
__device__ __forceinline__ uint32_t pack_bf16(uint16_t a, uint16_t b) { return (uint32_t)a | ((uint32_t)b << 16); }
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// grid: rows / 64 * N_KV_HEADS CTAs (1-D), kTcThreads threads, sizeof(AttTcSmem) bytes.
__global__ void __launch_bounds__(kTcThreads, 1)
attention_tc_kernel(const float* __restrict__ Q, int pos0, const uint16_t* __restrict__ kc_l, const uint16_t* __restrict__ vc_l,
                    uint16_t* __restrict__ As, int ld_as) {
    extern __shared__ __align__(16) uint8_t att_tc_smem[];
    AttTcSmem& S = *reinterpret_cast<AttTcSmem*>(att_tc_smem);
    const int nqb = gridDim.x / N_KV_HEADS;
    const int qb = nqb - 1 - (int)blockIdx.x / N_KV_HEADS, hk = (int)blockIdx.x % N_KV_HEADS;
    const int q0 = qb * kAttBlock, tid = threadIdx.x;
    const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, qd = lane & 3;
    const int hl = warp >> 2, wr = warp & 3, h = 2 * hk + hl;     // this warp's q head, and its 16-row slice
    const int last = min(pos0 + q0 + kAttBlock - 1, SEQ_LEN - 1);
    const int ntiles = last / kAttBlock + 1;
    const uint16_t* kb = kc_l + (size_t)hk * SEQ_LEN * HEAD_DIM;
    const uint16_t* vb = vc_l + (size_t)hk * SEQ_LEN * HEAD_DIM;
    // tile t of K and V into buffer t & 1: 64 rows x 16 chunks of 16 bytes each, 8 per thread
    auto load_tile = [&](int t) {
        const int k0 = t * kAttBlock, bf = t & 1;
        #pragma unroll
        for (int i = 0; i < (kAttBlock * HEAD_DIM / 8) / kTcThreads; i++) {
            const int e = tid + i * kTcThreads, r = e >> 4, c = (e & 15) * 8;
            const size_t src = (size_t)min(k0 + r, SEQ_LEN - 1) * HEAD_DIM + c;
            cp_async16(&S.k[bf][r][c], kb + src);
            cp_async16(&S.v[bf][r][c], vb + src);
        }
        cp_async_commit();
    };
    load_tile(0);
    // the block's query rows of both heads, split
    for (int i = tid; i < 2 * kAttBlock * HEAD_DIM / 4; i += kTcThreads) {
        const int hh = i / (kAttBlock * HEAD_DIM / 4), rem = i % (kAttBlock * HEAD_DIM / 4);
        const int r = rem / (HEAD_DIM / 4), c = (rem % (HEAD_DIM / 4)) * 4;
        const float4 v = *(const float4*)(Q + (size_t)(q0 + r) * Q_DIM + 128 * (2 * hk + hh) + c);
        uint32_t h0, m0, l0, h1, m1, l1;
        split3x2(v.x, v.y, h0, m0, l0);
        split3x2(v.z, v.w, h1, m1, l1);
        *(uint2*)&S.q[hh][0][r][c] = make_uint2(h0, h1);
        *(uint2*)&S.q[hh][1][r][c] = make_uint2(m0, m1);
        if constexpr (kAttParts > 2) *(uint2*)&S.q[hh][kAttParts - 1][r][c] = make_uint2(l0, l1);
    }
    const int rowA = 16 * wr + (lane & 15);                       // ldmatrix row of this lane for A tiles
    const uint32_t qa = smem_addr(&S.q[hl][0][rowA][(lane >> 4) * 8]);
    constexpr uint32_t kQPart = kAttBlock * kTcRowE * 2;         // bytes between q parts
    constexpr uint32_t kKVBuf = kAttBlock * kTcRowE * 2;         // bytes between the two K (or V) buffers
    // B fragments of K (keys x dims, row-major = col-major B): lanes 0-7 keys 0-7 @ d, 8-15 keys 0-7 @ d+8,
    // 16-23 keys 8-15 @ d, 24-31 keys 8-15 @ d+8
    const uint32_t kb_addr = smem_addr(&S.k[0][(lane & 7) + ((lane >> 4) << 3)][((lane >> 3) & 1) * 8]);
    // B fragments of V via .trans: lanes 0-7 keys 0-7 @ n, 8-15 keys 8-15 @ n, 16-23 keys 0-7 @ n+8, 24-31 keys 8-15 @ n+8
    const uint32_t vb_addr = smem_addr(&S.v[0][(lane & 15)][(lane >> 4) * 8]);
    // scores stay in raw units; p = 2^((s - max) * c), c = log2(e) / sqrt(d)
    const float c2 = 1.4426950408889634f / sqrtf((float)HEAD_DIM);
    float o[16][4];
    #pragma unroll
    for (int i = 0; i < 16; i++) { o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f; }
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f};
    const int qmin = pos0 + q0 + 16 * wr;                         // the warp's first query position
    const int qp0 = qmin + g, qp1 = qp0 + 8;                       // this lane's two query positions
    for (int t = 0; t < ntiles; t++) {
        if (t + 1 < ntiles) { load_tile(t + 1); cp_async_wait<1>(); }
        else cp_async_wait<0>();
        __syncthreads();   // tile t (and, at t = 0, the split q rows) visible to every warp
        const int k0 = t * kAttBlock;
        const uint32_t kbuf = kb_addr + (t & 1) * kKVBuf, vbuf = vb_addr + (t & 1) * kKVBuf;
        // S (16 rows x 64 keys) = Q K^T: 8 n-tiles of 8 keys
        float sc[8][4];
        #pragma unroll
        for (int n = 0; n < 8; n++) { sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f; }
        #pragma unroll
        for (int kt = 0; kt < HEAD_DIM / 16; kt++) {
            uint32_t a[kAttParts][4];
            #pragma unroll
            for (int p = 0; p < kAttParts; p++) ldsm_x4(qa + p * kQPart + kt * 32, a[p][0], a[p][1], a[p][2], a[p][3]);
            #pragma unroll
            for (int np = 0; np < 4; np++) {   // keys 16np .. 16np+15: two n-tiles
                uint32_t b0, b1, b2, b3;
                ldsm_x4(kbuf + np * 16 * kTcRowE * 2 + kt * 32, b0, b1, b2, b3);
                #pragma unroll
                for (int p = 0; p < kAttParts; p++) {
                    mma_bf16_16816(sc[2 * np], a[p][0], a[p][1], a[p][2], a[p][3], b0, b1);
                    mma_bf16_16816(sc[2 * np + 1], a[p][0], a[p][1], a[p][2], a[p][3], b2, b3);
                }
            }
        }
        // causal mask, only where the tile reaches past the warp's first query
        if (k0 + kAttBlock - 1 > qmin) {
            #pragma unroll
            for (int n = 0; n < 8; n++) {
                #pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int kp = k0 + 8 * n + 2 * qd + (e & 1);
                    if (kp > (e < 2 ? qp0 : qp1)) sc[n][e] = -INFINITY;
                }
            }
        }
        // online softmax over this tile (rows g and g + 8 of the warp)
        float mx[2] = {-INFINITY, -INFINITY};
        #pragma unroll
        for (int n = 0; n < 8; n++) {
            mx[0] = fmaxf(mx[0], fmaxf(sc[n][0], sc[n][1]));
            mx[1] = fmaxf(mx[1], fmaxf(sc[n][2], sc[n][3]));
        }
        float scale[2], mc[2];
        #pragma unroll
        for (int r = 0; r < 2; r++) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
            const float mn = fmaxf(mrow[r], mx[r]);   // finite: key 0 precedes every query
            scale[r] = exp2f((mrow[r] - mn) * c2);    // 0 on the first tile (mrow = -inf)
            mrow[r] = mn;
            mc[r] = mn * c2;
        }
        float ps[2] = {0.f, 0.f};
        #pragma unroll
        for (int n = 0; n < 8; n++) {
            #pragma unroll
            for (int e = 0; e < 4; e++) {
                const float pr = exp2f(fmaf(sc[n][e], c2, -mc[e >> 1]));   // masked: 2^-inf = 0
                sc[n][e] = pr;
                ps[e >> 1] += pr;
            }
        }
        #pragma unroll
        for (int r = 0; r < 2; r++) {
            ps[r] += __shfl_xor_sync(0xffffffffu, ps[r], 1);
            ps[r] += __shfl_xor_sync(0xffffffffu, ps[r], 2);
            lrow[r] = fmaf(lrow[r], scale[r], ps[r]);
        }
        #pragma unroll
        for (int i = 0; i < 16; i++) { o[i][0] *= scale[0]; o[i][1] *= scale[0]; o[i][2] *= scale[1]; o[i][3] *= scale[1]; }
        // O += P V: 4 k-tiles of 16 keys; P's A fragment comes from S n-tiles 2kt, 2kt + 1
        #pragma unroll
        for (int kt = 0; kt < 4; kt++) {
            uint32_t a[3][4];
            #pragma unroll
            for (int j = 0; j < 4; j++) {   // a0: (g, keys 2qd..) = n-tile 2kt d0,d1; a1: rows g+8 = d2,d3; a2, a3: n-tile 2kt+1
                const float* src = &sc[2 * kt + (j >> 1)][(j & 1) * 2];
                split3x2(src[0], src[1], a[0][j], a[1][j], a[2][j]);
            }
            #pragma unroll
            for (int np = 0; np < 8; np++) {   // dims 16np .. 16np+15: two n-tiles
                uint32_t b0, b1, b2, b3;
                ldsm_x4_trans(vbuf + kt * 16 * kTcRowE * 2 + np * 32, b0, b1, b2, b3);
                #pragma unroll
                for (int p = 0; p < kAttParts; p++) {
                    mma_bf16_16816(o[2 * np], a[p][0], a[p][1], a[p][2], a[p][3], b0, b1);
                    mma_bf16_16816(o[2 * np + 1], a[p][0], a[p][1], a[p][2], a[p][3], b2, b3);
                }
            }
        }
        __syncthreads();   // every warp is done with buffer t & 1 before tile t + 2 is copied into it
    }
    // O rows g, g + 8 of the warp; dims 8n + 2qd, +1 — straight into As, split
    const float inv0 = 1.0f / lrow[0], inv1 = 1.0f / lrow[1];
    uint16_t* a0 = As + (size_t)(q0 + 16 * wr + g) * ld_as;
    uint16_t* a1 = a0 + (size_t)8 * ld_as;
    #pragma unroll
    for (int n = 0; n < 16; n++) {
        put_split2(a0, 128 * h + 8 * n + 2 * qd, o[n][0] * inv0, o[n][1] * inv0);
        put_split2(a1, 128 * h + 8 * n + 2 * qd, o[n][2] * inv1, o[n][3] * inv1);
    }
}

}  // namespace pf
}  // namespace qb
