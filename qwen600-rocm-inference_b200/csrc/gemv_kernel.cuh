// gemv_kernel.cuh — isolated batch-1 bf16 GEMV y = bf16(W x), fp32 accumulate.
//
// Replaces matmul_cublas (qwen_model.cuh:706-757: cublasGemmEx with N = 1).
// One CTA per SM; CTA c owns rows [N*c/G, N*(c+1)/G), which are contiguous in
// memory, and streams them with 1-D bulk async copies through the same
// 6 x 32 KB shared-memory ring as the decode kernel.  Each warp dots one
// 1024-column segment of one row against x held in registers; segments of a
// row are summed in a fixed order (deterministic).
#pragma once
#include "decode_kernel.cuh"

namespace qb {

struct __align__(16) GemvSmem {
    uint64_t full[kSlots];
    uint64_t empty[kSlots];
    float part[2][kNCW];
};
constexpr size_t kGemvSmemBytes = (size_t)kSlots * kSlotBytes + sizeof(GemvSmem);
constexpr int kGemvThreads = kNCT + 32;     // 16 consumer warps + one producer warp

__host__ __device__ __forceinline__ int gemv_segs(int K) { return (K + 1023) / 1024; }
__host__ __device__ __forceinline__ int gemv_rows_per_chunk(int K) {
    const int a = kNCW / gemv_segs(K), b = kSlotBytes / (2 * K);
    return a < b ? a : b;
}

__global__ void __launch_bounds__(kGemvThreads, 1)
gemv_bf16_kernel(const uint16_t* __restrict__ W, const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int N, int K,
                 uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    GemvSmem* S = reinterpret_cast<GemvSmem*>(smem + (size_t)kSlots * kSlotBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < kSlots; s++) { mbar_init(&S->full[s], 1); mbar_init(&S->empty[s], kNCW); }
        fence_barrier_init();
    }
    __syncthreads();
    const int G = gridDim.x, c = blockIdx.x;
    const int a = span_lo(N, G, c), b = span_lo(N, G, c + 1);
    const int rpc = gemv_rows_per_chunk(K), nseg = gemv_segs(K);
    const size_t row_bytes = (size_t)K * 2;

    if (warp == kNCW) {
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            uint32_t k = 0;
            for (int r = a; r < b; r += rpc, k++) {
                const int n = min(rpc, b - r);
                const uint32_t s = k % kSlots, ph = (k / kSlots) & 1u;
                if (!mbar_wait(&S->empty[s], ph ^ 1u, 2 * kWaitNs)) atomicOr(err, 2u);
                mbar_arrive_expect_tx(&S->full[s], (uint32_t)(n * row_bytes));
                bulk_g2s(ring + (size_t)s * kSlotBytes, (const uint8_t*)W + (size_t)r * row_bytes, (uint32_t)(n * row_bytes),
                         &S->full[s], pol);
            }
        }
        return;
    }
    // consumer: warp -> (row in chunk, 1024-column segment)
    const int row = warp / nseg, seg = warp % nseg;
    const int c0 = seg * 1024, c1 = min(K, c0 + 1024);
    const int nvec = (c1 - c0) / 256;   // uint4 steps per lane (<= 4)
    float xr[32];
    #pragma unroll
    for (int i = 0; i < 4; i++) {
        if (i < nvec) {
            const uint4 v = __ldg((const uint4*)(x + c0 + 256 * i + 8 * lane));
            xr[8 * i + 0] = bf_lo(v.x); xr[8 * i + 1] = bf_hi(v.x); xr[8 * i + 2] = bf_lo(v.y); xr[8 * i + 3] = bf_hi(v.y);
            xr[8 * i + 4] = bf_lo(v.z); xr[8 * i + 5] = bf_hi(v.z); xr[8 * i + 6] = bf_lo(v.w); xr[8 * i + 7] = bf_hi(v.w);
        } else {
            #pragma unroll
            for (int e = 0; e < 8; e++) xr[8 * i + e] = 0.f;
        }
    }
    uint32_t k = 0;
    for (int r = a; r < b; r += rpc, k++) {
        const int n = min(rpc, b - r);
        const uint32_t s = k % kSlots, ph = (k / kSlots) & 1u;
        if (!mbar_wait(&S->full[s], ph, 3 * kWaitNs)) atomicOr(err, 4u);
        const uint8_t* ch = ring + (size_t)s * kSlotBytes;
        float* part = S->part[k & 1];
        if (row < n) {
            const uint4* w = (const uint4*)(ch + (size_t)row * row_bytes + (size_t)c0 * 2);
            float acc = 0.f;
            #pragma unroll
            for (int i = 0; i < 4; i++)
                if (i < nvec) acc = dot8(w[32 * i + lane], &xr[8 * i], acc);
            acc = warp_sum(acc);
            if (lane == 0) part[warp] = acc;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S->empty[s]);
        named_bar(1, kNCT);
        if (tid < n) {
            float t = 0.f;
            for (int q = 0; q < nseg; q++) t += part[tid * nseg + q];
            y[r + tid] = f2bf(t);
        }
    }
}

}  // namespace qb
