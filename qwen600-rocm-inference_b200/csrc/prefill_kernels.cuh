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
//   attention     causal GQA over the cache -> O (fp32)
//   split         O -> As;  GEMM As . Wo^T -> Y
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
constexpr int kAttThreads = 256;

__device__ __forceinline__ void split3(float v, uint16_t& h, uint16_t& m, uint16_t& l) {
    h = f2bf(v);
    const float r = v - bf2f(h);
    m = f2bf(r);
    l = f2bf(r - bf2f(m));
}
// v (4 consecutive columns c..c+3 of a K-wide row) -> the three part blocks of As row r
__device__ __forceinline__ void put_split4(uint16_t* As_row, int K, int c, float4 v) {
    uint16_t h[4], m[4], l[4];
    split3(v.x, h[0], m[0], l[0]); split3(v.y, h[1], m[1], l[1]);
    split3(v.z, h[2], m[2], l[2]); split3(v.w, h[3], m[3], l[3]);
    *(uint2*)(As_row + c) = make_uint2(h[0] | ((uint32_t)h[1] << 16), h[2] | ((uint32_t)h[3] << 16));
    *(uint2*)(As_row + K + c) = make_uint2(m[0] | ((uint32_t)m[1] << 16), m[2] | ((uint32_t)m[3] << 16));
    *(uint2*)(As_row + 2 * K + c) = make_uint2(l[0] | ((uint32_t)l[1] << 16), l[2] | ((uint32_t)l[3] << 16));
}

// X[r] = embed[token[r]] (fp32) for r < m; 0 for m <= r < rows.
__global__ void embed_kernel(const uint16_t* __restrict__ embed, const int* __restrict__ tokens, int m, int rows, float* __restrict__ X) {
    const int r = blockIdx.x, t = threadIdx.x;   // 256 threads x 4 columns
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < m) {
        const int tok = min(max(tokens[r], 0), VOCAB_SIZE - 1);
        const uint2 w = *(const uint2*)(embed + (size_t)tok * DIM + 4 * t);
        v = make_float4(bf_lo(w.x), bf_hi(w.x), bf_lo(w.y), bf_hi(w.y));
    }
    *(float4*)(X + (size_t)r * DIM + 4 * t) = v;
}

// One warp per row: X[r] += add[r] (if add), then RMSNorm with `gain` (the
// decode chain's formula: (x * (1 / sqrt(mean(x^2) + eps))) * g) into As.
__global__ void norm_split_kernel(float* __restrict__ X, const float* __restrict__ add, int ld_add, const uint16_t* __restrict__ gain,
                                  uint16_t* __restrict__ As, int ld_as, int rows) {
    const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (r >= rows) return;
    float* x = X + (size_t)r * DIM;
    float4 v[8];
    float ss = 0.f;
    #pragma unroll
    for (int i = 0; i < 8; i++) {
        const int c = 128 * i + 4 * lane;
        v[i] = *(const float4*)(x + c);
        if (add) {
            const float4 a = *(const float4*)(add + (size_t)r * ld_add + c);
            v[i].x += a.x; v[i].y += a.y; v[i].z += a.z; v[i].w += a.w;
            *(float4*)(x + c) = v[i];
        }
        ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    ss = warp_sum(ss);
    const float rs = 1.0f / sqrtf(ss * (1.0f / DIM) + EPS);
    uint16_t* a_row = As + (size_t)r * ld_as;
    #pragma unroll
    for (int i = 0; i < 8; i++) {
        const int c = 128 * i + 4 * lane;
        const uint2 g = *(const uint2*)(gain + c);
        const float4 y = make_float4((v[i].x * rs) * bf_lo(g.x), (v[i].y * rs) * bf_hi(g.x), (v[i].z * rs) * bf_lo(g.y), (v[i].w * rs) * bf_hi(g.y));
        put_split4(a_row, DIM, c, y);
    }
}

// As[r] = split(src[r][0..K)), one thread per 4 columns.
__global__ void split_kernel(const float* __restrict__ src, int ld_src, int K, uint16_t* __restrict__ As, int ld_as, int rows) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int q = K / 4;
    if (i >= (size_t)rows * q) return;
    const int r = (int)(i / q), c = (int)(i % q) * 4;
    put_split4(As + (size_t)r * ld_as, K, c, *(const float4*)(src + (size_t)r * ld_src + c));
}

// h = silu(g) * u for the gate (Y columns 0..H) and up (H..2H) outputs, then split into As.
__global__ void swiglu_split_kernel(const float* __restrict__ Y, int ld_y, uint16_t* __restrict__ As, int ld_as, int rows) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int q = HIDDEN_DIM / 4;
    if (i >= (size_t)rows * q) return;
    const int r = (int)(i / q), c = (int)(i % q) * 4;
    const float4 g = *(const float4*)(Y + (size_t)r * ld_y + c), u = *(const float4*)(Y + (size_t)r * ld_y + HIDDEN_DIM + c);
    const float4 h = make_float4((g.x / (1.0f + expf(-g.x))) * u.x, (g.y / (1.0f + expf(-g.y))) * u.y,
                                 (g.z / (1.0f + expf(-g.z))) * u.z, (g.w / (1.0f + expf(-g.w))) * u.w);
    put_split4(As + (size_t)r * ld_as, HIDDEN_DIM, c, h);
}

// q/k/v of row r (position pos0 + r), one warp per (row, slot): slots 0..15 q
// heads, 16..23 k heads, 24..31 v heads; lane l holds dims 4l..4l+3.  QK-norm
// (qwen_model.cuh:215-245) and NeoX RoPE (:327-364) as in the decode chain; k
// and v go to the bf16 cache (rows < m only), q to Q (fp32).
__global__ void qkv_post_kernel(const float* __restrict__ Y, int ld_y, int m, int rows, int pos0, const uint16_t* __restrict__ qn,
                                const uint16_t* __restrict__ kn, const float* __restrict__ rope, float* __restrict__ Q,
                                uint16_t* __restrict__ kc_l, uint16_t* __restrict__ vc_l) {
    const int w = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int r = w >> 5, slot = w & 31;
    if (r >= rows) return;
    const int pos = min(pos0 + r, SEQ_LEN - 1);
    const int col = slot < 16 ? 128 * slot : (slot < 24 ? Q_DIM + 128 * (slot - 16) : Q_DIM + KV_DIM + 128 * (slot - 24));
    const float4 a = *(const float4*)(Y + (size_t)r * ld_y + col + 4 * lane);
    float x[4] = {a.x, a.y, a.z, a.w};
    if (slot < 24) {
        const uint2 gn = *(const uint2*)((slot < 16 ? qn : kn) + 4 * lane);
        const float tot = warp_sum(x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3]);
        const float rs = 1.0f / sqrtf(tot * (1.0f / HEAD_DIM) + EPS);
        x[0] = (x[0] * rs) * bf_lo(gn.x); x[1] = (x[1] * rs) * bf_hi(gn.x);
        x[2] = (x[2] * rs) * bf_lo(gn.y); x[3] = (x[3] * rs) * bf_hi(gn.y);
        const float* cs = rope + (size_t)pos * HEAD_DIM;
        #pragma unroll
        for (int e = 0; e < 4; e++) {
            const float pv = __shfl_xor_sync(0xffffffffu, x[e], 16);
            const int d = 4 * lane + e, j = d & 63;
            const float cj = cs[j], sj = cs[64 + j];
            x[e] = d < 64 ? (x[e] * cj - pv * sj) : (pv * sj + x[e] * cj);
        }
    }
    if (slot < 16) {
        *(float4*)(Q + (size_t)r * Q_DIM + 128 * slot + 4 * lane) = make_float4(x[0], x[1], x[2], x[3]);
    } else if (r < m) {
        const int h = slot < 24 ? slot - 16 : slot - 24;
        uint16_t* dst = (slot < 24 ? kc_l : vc_l) + ((size_t)h * SEQ_LEN + pos) * HEAD_DIM + 4 * lane;
        *(uint2*)dst = make_uint2((uint32_t)f2bf(x[0]) | ((uint32_t)f2bf(x[1]) << 16), (uint32_t)f2bf(x[2]) | ((uint32_t)f2bf(x[3]) << 16));
    }
}

// Causal GQA attention, fp32: one CTA per (64 query rows, q head h); key/value
// head h / 2 from the cache, positions 0 .. pos0 + r for row r, in tiles of 64
// with an online softmax (scores / sqrt(128), as qwen_model.cuh:566-585).
// Scores: thread (ty, tx) takes query rows 4ty..4ty+3 and keys tx + 16c;
// P.V: the same query rows and dims 8tx..8tx+7.
struct AttSmem {
    float q[kAttBlock][HEAD_DIM];
    float k[kAttBlock][HEAD_DIM + 1];
    float v[kAttBlock][HEAD_DIM];
    float p[kAttBlock][kAttBlock + 1];
};
__global__ void __launch_bounds__(kAttThreads)
attention_kernel(const float* __restrict__ Q, int pos0, const uint16_t* __restrict__ kc_l, const uint16_t* __restrict__ vc_l, float* __restrict__ O) {
    extern __shared__ __align__(16) uint8_t att_smem[];
    AttSmem& S = *reinterpret_cast<AttSmem*>(att_smem);
    const int h = blockIdx.y, hk = h >> 1, q0 = blockIdx.x * kAttBlock, tid = threadIdx.x;
    const int ty = tid >> 4, tx = tid & 15;
    const float sqrt_hd = sqrtf((float)HEAD_DIM);
    for (int i = tid; i < kAttBlock * HEAD_DIM / 4; i += kAttThreads) {
        const int r = i / (HEAD_DIM / 4), c = (i % (HEAD_DIM / 4)) * 4;
        *(float4*)&S.q[r][c] = *(const float4*)(Q + (size_t)(q0 + r) * Q_DIM + 128 * h + c);
    }
    float mrow[4], lrow[4], acc[4][8];
    #pragma unroll
    for (int i = 0; i < 4; i++) {
        mrow[i] = -INFINITY; lrow[i] = 0.f;
        #pragma unroll
        for (int d = 0; d < 8; d++) acc[i][d] = 0.f;
    }
    const int last = min(pos0 + q0 + kAttBlock - 1, SEQ_LEN - 1);   // the block's last query position
    const uint16_t* kb = kc_l + (size_t)hk * SEQ_LEN * HEAD_DIM;
    const uint16_t* vb = vc_l + (size_t)hk * SEQ_LEN * HEAD_DIM;
    for (int k0 = 0; k0 <= last; k0 += kAttBlock) {
        __syncthreads();   // the previous tile's k, v and p are consumed
        for (int i = tid; i < kAttBlock * HEAD_DIM / 8; i += kAttThreads) {
            const int r = i / (HEAD_DIM / 8), c = (i % (HEAD_DIM / 8)) * 8;
            const int kp = min(k0 + r, SEQ_LEN - 1);
            const uint4 kw = *(const uint4*)(kb + (size_t)kp * HEAD_DIM + c);
            const uint4 vw = *(const uint4*)(vb + (size_t)kp * HEAD_DIM + c);
            const uint32_t ka[4] = {kw.x, kw.y, kw.z, kw.w}, va[4] = {vw.x, vw.y, vw.z, vw.w};
            #pragma unroll
            for (int j = 0; j < 4; j++) {
                S.k[r][c + 2 * j] = bf_lo(ka[j]); S.k[r][c + 2 * j + 1] = bf_hi(ka[j]);
                S.v[r][c + 2 * j] = bf_lo(va[j]); S.v[r][c + 2 * j + 1] = bf_hi(va[j]);
            }
        }
        __syncthreads();
        float s[4][4];
        #pragma unroll
        for (int i = 0; i < 4; i++)
            #pragma unroll
            for (int c = 0; c < 4; c++) s[i][c] = 0.f;
        #pragma unroll 4
        for (int d = 0; d < HEAD_DIM; d++) {
            float qv[4], kv[4];
            #pragma unroll
            for (int i = 0; i < 4; i++) qv[i] = S.q[4 * ty + i][d];
            #pragma unroll
            for (int c = 0; c < 4; c++) kv[c] = S.k[tx + 16 * c][d];
            #pragma unroll
            for (int i = 0; i < 4; i++)
                #pragma unroll
                for (int c = 0; c < 4; c++) s[i][c] = fmaf(qv[i], kv[c], s[i][c]);
        }
        #pragma unroll
        for (int i = 0; i < 4; i++) {
            const int qp = pos0 + q0 + 4 * ty + i;
            float mx = -INFINITY;
            #pragma unroll
            for (int c = 0; c < 4; c++) {
                const int kp = k0 + tx + 16 * c;
                s[i][c] = kp <= qp ? s[i][c] / sqrt_hd : -INFINITY;
                mx = fmaxf(mx, s[i][c]);
            }
            #pragma unroll
            for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float mn = fmaxf(mrow[i], mx);   // finite: key 0 <= every query position
            const float sc = expf(mrow[i] - mn);
            float ps = 0.f;
            #pragma unroll
            for (int c = 0; c < 4; c++) {
                const float pr = s[i][c] == -INFINITY ? 0.f : expf(s[i][c] - mn);
                S.p[4 * ty + i][tx + 16 * c] = pr;
                ps += pr;
            }
            #pragma unroll
            for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            lrow[i] = fmaf(lrow[i], sc, ps);
            #pragma unroll
            for (int d = 0; d < 8; d++) acc[i][d] *= sc;
            mrow[i] = mn;
        }
        __syncthreads();
        #pragma unroll 4
        for (int j = 0; j < kAttBlock; j++) {
            const float4 v0 = *(const float4*)&S.v[j][8 * tx], v1 = *(const float4*)&S.v[j][8 * tx + 4];
            #pragma unroll
            for (int i = 0; i < 4; i++) {
                const float pr = S.p[4 * ty + i][j];
                acc[i][0] = fmaf(pr, v0.x, acc[i][0]); acc[i][1] = fmaf(pr, v0.y, acc[i][1]);
                acc[i][2] = fmaf(pr, v0.z, acc[i][2]); acc[i][3] = fmaf(pr, v0.w, acc[i][3]);
                acc[i][4] = fmaf(pr, v1.x, acc[i][4]); acc[i][5] = fmaf(pr, v1.y, acc[i][5]);
                acc[i][6] = fmaf(pr, v1.z, acc[i][6]); acc[i][7] = fmaf(pr, v1.w, acc[i][7]);
            }
        }
    }
    #pragma unroll
    for (int i = 0; i < 4; i++) {
        float* o = O + (size_t)(q0 + 4 * ty + i) * Q_DIM + 128 * h + 8 * tx;
        const float inv = 1.0f / lrow[i];
        *(float4*)o = make_float4(acc[i][0] * inv, acc[i][1] * inv, acc[i][2] * inv, acc[i][3] * inv);
        *(float4*)(o + 4) = make_float4(acc[i][4] * inv, acc[i][5] * inv, acc[i][6] * inv, acc[i][7] * inv);
    }
}

}  // namespace pf
}  // namespace qb
