// gemv_kernel.cuh — isolated batch-1 bf16 GEMV y = bf16(W x), fp32 accumulate.
//
// Replaces matmul_cublas (qwen_model.cuh:706-757: cublasGemmEx with N = 1).
// Two kernels, one contract (row-major W [N][K], K a multiple of 256 up to
// 4096, each row's segments summed in a fixed order: deterministic):
//
//  gemv_direct_kernel  small and mid-size matrices (the decode chain's 4-13 MB
//      projections).  No staging ring and no set-up: x is copied to shared
//      memory once per CTA while the first weight loads are already in flight
//      (the two latencies overlap), and every warp takes (row, 1024-column segment)
//      work items, loading its whole share of both rows of a pair with 16-byte
//      streaming loads before the first FMA, so each SM keeps tens of KB of
//      weight reads in flight.  Small CTAs (up to 8 warps) in a grid sized to
//      the work: every SM is busy from the first microsecond.
//  gemv_bf16_kernel    large matrices (the 311 MB LM head).  One CTA per SM
//      owns a contiguous row range and streams it with 1-D bulk async copies
//      through a 5 x 32 KB shared-memory ring (TMA engine, mbarriers).  Every
//      wait is bounded: on expiry it records a code in the caller's error word
//      and the CTA winds down (the producer issues nothing more, consumers
//      leave at the next block barrier, the producer drains its copies before
//      it exits), so y is then invalid and the host reports QWEN_E_TIMEOUT.
#pragma once
#include "decode_kernel.cuh"

namespace qb {

// ---------------------------------------------------------------------------
// direct-load kernel
// ---------------------------------------------------------------------------
constexpr int kGemvDirectMaxK = 4096;
constexpr int kGemvDirectWarps = 8;

// Work layout for K: segs = K / 1024 rounded up segments of a row, rows_cta =
// rows per CTA (warps = rows_cta x segs <= 8).
__host__ __device__ __forceinline__ int gemv_direct_segs(int K) { return (K + 1023) / 1024; }
__host__ __device__ __forceinline__ int gemv_direct_rows_cta(int K) { return kGemvDirectWarps / gemv_direct_segs(K); }

// 16-byte streaming load (read once: no L1 allocation)
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

// grid.x = number of CTAs; CTA b serves rows [b*rows_cta*? ...] in a grid-stride
// loop over row groups of rows_cta rows.  Warp w: row w / segs of the group,
// segment w % segs.  Two row groups per iteration (pair), so each lane has up
// to 2 x 4 16-byte loads in flight.
__global__ void __launch_bounds__(kGemvDirectWarps * 32)
gemv_direct_kernel(const uint16_t* __restrict__ W, const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int N, int K) {
    __shared__ __align__(16) uint16_t xs[kGemvDirectMaxK];
    __shared__ float part[2][kGemvDirectWarps];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int segs = gemv_direct_segs(K), rows_cta = gemv_direct_rows_cta(K);
    const int nthreads = rows_cta * segs * 32;
    bool staged = false;   // x goes to shared memory while the first weight loads are in flight
    const int r_in = warp / segs, seg = warp % segs;
    const int c0 = seg * 1024, c1 = min(K, c0 + 1024);
    const int nvec = (c1 - c0) / 256;   // 16-byte loads per lane per row (<= 4)
    const int groups = (N + rows_cta - 1) / rows_cta;
    for (int g0 = blockIdx.x; g0 < groups; g0 += 2 * gridDim.x) {
        const int g1 = g0 + gridDim.x;
        const int ra = g0 * rows_cta + r_in, rb = g1 * rows_cta + r_in;
        const bool va = ra < N, vb = g1 < groups && rb < N;
        uint4 wa[4], wb[4];
        #pragma unroll
        for (int i = 0; i < 4; i++) {
            if (i < nvec && va) wa[i] = ld_stream16(W + (size_t)ra * K + c0 + 256 * i + 8 * lane);
            if (i < nvec && vb) wb[i] = ld_stream16(W + (size_t)rb * K + c0 + 256 * i + 8 * lane);
        }
        if (!staged) {   // uniform: the loop bounds depend on the block only
            for (int i = tid; i < K / 8; i += nthreads) *(uint4*)&xs[8 * i] = __ldg((const uint4*)x + i);
            __syncthreads();
            staged = true;
        }
        float sa = 0.f, sb = 0.f;
        #pragma unroll
        for (int i = 0; i < 4; i++) {
            if (i < nvec) {
                const uint4 xv = *(const uint4*)&xs[c0 + 256 * i + 8 * lane];
                float xf[8] = {bf_lo(xv.x), bf_hi(xv.x), bf_lo(xv.y), bf_hi(xv.y), bf_lo(xv.z), bf_hi(xv.z), bf_lo(xv.w), bf_hi(xv.w)};
                if (va) sa = dot8(wa[i], xf, sa);
                if (vb) sb = dot8(wb[i], xf, sb);
            }
        }
        sa = warp_sum(sa);
        sb = warp_sum(sb);
        if (segs == 1) {
            if (lane == 0) {
                if (va) y[ra] = f2bf(sa);
                if (vb) y[rb] = f2bf(sb);
            }
        } else {
            if (lane == 0) { part[0][warp] = sa; part[1][warp] = sb; }
            __syncthreads();
            if (tid < 2 * rows_cta) {   // thread t: pair member t / rows_cta, row t % rows_cta of the group
                const int m = tid / rows_cta, rr = tid % rows_cta;
                const int row = (m == 0 ? g0 : g1) * rows_cta + rr;
                if (row < N && (m == 0 || g1 < groups)) {
                    float t = 0.f;
                    for (int q = 0; q < segs; q++) t += part[m][rr * segs + q];
                    y[row] = f2bf(t);
                }
            }
            __syncthreads();
        }
    }
}

// ---------------------------------------------------------------------------
// ring kernel (large matrices)
// ---------------------------------------------------------------------------
struct __align__(16) GemvSmem {
    uint64_t full[kSlots];
    uint64_t empty[kSlots];
    float part[2][kNCW];
    int dead;      // a consumer's wait expired: every consumer leaves at the next block barrier
};
constexpr size_t kGemvSmemBytes = (size_t)kSlots * kSlotBytes + sizeof(GemvSmem);
constexpr int kGemvThreads = kNCT + 32;     // 16 consumer warps + one producer warp

__host__ __device__ __forceinline__ int gemv_segs(int K) { return (K + 1023) / 1024; }
__host__ __device__ __forceinline__ int gemv_rows_per_chunk(int K) {
    const int a = kNCW / gemv_segs(K), b = kSlotBytes / (2 * K);
    return a < b ? a : b;
}

// err (caller's error word): |= 2 when the producer's wait for a free slot
// expired, |= 4 when a consumer's wait for a filled slot expired.
__global__ void __launch_bounds__(kGemvThreads, 1)
gemv_bf16_kernel(const uint16_t* __restrict__ W, const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int N, int K,
                 uint32_t* err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t* ring = smem;
    GemvSmem* S = reinterpret_cast<GemvSmem*>(smem + (size_t)kSlots * kSlotBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) {
        for (int s = 0; s < kSlots; s++) { mbar_init(&S->full[s], 1); mbar_init(&S->empty[s], kNCW); }
        S->dead = 0;
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
                if (!mbar_wait(&S->empty[s], ph ^ 1u, 2 * kWaitNs)) { atomicOr(err, 2u); break; }   // issue nothing more
                mbar_arrive_expect_tx(&S->full[s], (uint32_t)(n * row_bytes));
                bulk_g2s(ring + (size_t)s * kSlotBytes, (const uint8_t*)W + (size_t)r * row_bytes, (uint32_t)(n * row_bytes),
                         &S->full[s], pol);
            }
            // drain: the copies still in flight land before the CTA exits (bounded)
            for (uint32_t j = k > (uint32_t)kSlots ? k - kSlots : 0u; j < k; j++)
                mbar_wait(&S->full[j % kSlots], (j / kSlots) & 1u, kWaitNs);
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
        const bool ok = mbar_wait(&S->full[s], ph, 3 * kWaitNs);
        if (!ok) {
            if (lane == 0) atomicOr(err, 4u);
            S->dead = 1;
        }
        const uint8_t* ch = ring + (size_t)s * kSlotBytes;
        float* part = S->part[k & 1];
        if (ok && row < n) {
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
        if (*(volatile int*)&S->dead) return;   // every consumer reads the same value after the barrier
        if (tid < n) {
            float t = 0.f;
            for (int q = 0; q < nseg; q++) t += part[tid * nseg + q];
            y[r + tid] = f2bf(t);
        }
    }
}

}  // namespace qb
