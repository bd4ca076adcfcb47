// gemm_tc.cuh — C[M][N] = A[M][K] . B[N][K]^T on the sm_100a tensor cores
// (tcgen05.mma, kind::f16, bf16 in, fp32 accumulate in TMEM).
//
// The dense contractions of prefill (the reference has none: it runs the
// decode chain once per prompt token, main.cu:141-145): the projections of M
// prompt rows against a weight matrix stored row-major [N][K] (nn.Linear
// layout, K contiguous), so both operands are K-major.
//
// Persistent kernel, one CTA per SM (or per tile when there are fewer tiles),
// 192 threads; CTA b takes output tiles b, b + grid, ... (128 x BN each):
//   warp 0, one thread: TMA producer — 2-D tiled bulk tensor loads of a
//           128 x 64 A box and a BN x 64 B box per K step, 128-byte swizzle,
//           into a ring of stages (mbarrier complete_tx) that runs on
//           across tile boundaries; no multicast.  Launched with programmatic
//           stream serialization, the kernel starts while the kernel before it
//           finishes: the producer loads the B (weight) boxes of the ring's
//           first stages, then waits for that kernel (pdl_wait), then loads
//           the A (activation) boxes;
//   warp 1: allocates 2 x BN TMEM columns (two fp32 accumulators, 128 lanes =
//           the tile's rows); one thread issues four 128 x BN x 16 MMAs per K
//           step from shared-memory descriptors, commits each stage back to
//           the producer (tcgen05.commit -> mbarrier) and each finished tile
//           to the epilogue, alternating accumulators;
//   warps 2-5: epilogue — wait for a tile's accumulator, read their 32 TMEM
//           lanes (tcgen05.ld 32x32b), store fp32 or bf16 rows and hand the
//           accumulator back, while the MMA thread fills the other one.
// Every wait is bounded; on expiry the thread sets *err and stops waiting; the
// TMEM allocation is always released.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include "ptx.cuh"
#include "../host/config.h"

namespace qb {
namespace tc {

constexpr int kBM = 128;            // tile rows (TMEM lanes)
constexpr int kBK = 64;             // K per stage: one 128-byte swizzle row
constexpr int kThreads = 192;
constexpr int kPairThreads = 320;   // pair form: producer, MMA, 8 epilogue warps (two per TMEM lane quarter)
constexpr int kUmmaK = 16;          // K of one tcgen05.mma for 16-bit inputs
constexpr uint64_t kWaitNs = 2000000000ull;

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle
// layout that TMA writes: rows of 128 B, 8-row groups 1024 B apart (SBO),
// descriptor version 1 (sm_100), layout type 2 = SWIZZLE_128B.  Advancing the
// start address by 32 B selects the next 16-element K slice inside the row.
__device__ __forceinline__ uint64_t kmajor_sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) | ((uint64_t)(1024u >> 4) << 32) |
           ((uint64_t)1u << 46) | ((uint64_t)2u << 61);
}
// Instruction descriptor, kind::f16: D fp32 (bits 4-5 = 1), A and B bf16
// (bits 7-9, 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bit 17,
// M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (one row per lane).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
    #pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// Epilogue of one row segment: `v` = 32 fp32 results of columns [n, n + 32) of
// row m.  kOutF32: C fp32; else C bf16 (round to nearest even).
template <bool kOutF32>
__device__ __forceinline__ void store32(void* C, int ldc, int m, int n, const float (&v)[32]) {
    if constexpr (kOutF32) {
        float4* d = reinterpret_cast<float4*>(static_cast<float*>(C) + (size_t)m * ldc + n);
        #pragma unroll
        for (int i = 0; i < 8; i++) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
    } else {
        uint4* d = reinterpret_cast<uint4*>(static_cast<uint16_t*>(C) + (size_t)m * ldc + n);
        #pragma unroll
        for (int i = 0; i < 4; i++) {
            uint32_t w[4];
            #pragma unroll
            for (int j = 0; j < 4; j++) w[j] = (uint32_t)f2bf(v[8 * i + 2 * j]) | ((uint32_t)f2bf(v[8 * i + 2 * j + 1]) << 16);
            d[i] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
}

// Persistent form: grid = min(tiles, SMs); CTA b takes tiles b, b + grid, ...
// (tile = (n block, m block), n fastest).  Two TMEM accumulators (2 x BN
// columns): the MMA thread fills one while the epilogue warps drain the other,
// so a tile's epilogue overlaps the next tile's mainloop.  The producer runs
// ahead across tile boundaries through the same stage ring.
//
// B may be up to three matrices side by side along N (a grouped GEMM, e.g.
// the q, k and v projections of one layer, which are not adjacent in memory):
// n blocks [end[s-1], end[s]) read map[s] from its row 0; C's columns stay
// contiguous (n block j writes columns j * BN ..).
//
// Split K: with splits > 1 every tile is `splits` work items, item s taking
// K steps [s, s + 1) * kb_b / splits and writing its partial sum at column
// offset s * c_split_off of C (the caller adds the partials).
//
// Rows m_valid .. M-1 of C are not written (padding rows of a short pass).
//
// ldc in elements.  B's K extent may be a divisor kb_b * 64 of K (K = P kb_b
// 64, P = 1-3, the kernel's kParts): A = [a_1 | .. | a_P] (each kb_b * 64
// wide) against B gives sum_i a_i . B^T — the bf16 parts of fp32 activations
// in one accumulation.  A K step covers 64 columns of B and the same 64
// columns of every a_i (one stage: the P A boxes and the B box once), and
// the MMA thread issues the P products of each 16-wide slice in turn; kb_b is
// a multiple of splits.
struct BMaps {
    CUtensorMap map[3];
    int end[3];   // cumulative n-block counts; end[2] = total n blocks
};
// Outputs of the q|k|v epilogue (pair form, kEpi 2): the GEMM's N columns are
// the 16 q heads, then the 8 k heads, then the 8 v heads (128 each) of rows at
// positions pos0 + m.  q and k heads are RMS-normalised over their 128 values,
// scaled by qn / kn and rotated (RoPE: value j < 64 pairs with j + 64 at angle
// j, the table's row `pos` holding cos in columns 0-63 and sin in 64-127); q
// goes to q (fp32, rows Q_DIM apart), k and v to the layer's caches
// ([kv head][SEQ_LEN][128], bf16) and v also to vt ([kv head][128][SEQ_LEN]).
struct QkvOut {
    float* q;
    uint16_t* kc;
    uint16_t* vc;
    uint16_t* vt;
    const uint16_t* qn;
    const uint16_t* kn;
    const float* rope;
    int pos0;
};
// P = the activation parts of A (see PairLayout): a stage holds the P A boxes
// of one K step and its B box once.
template <int BN, int P>
struct Layout {
    static_assert(P >= 1 && P <= 3, "one to three activation parts");
    static constexpr int kABytes = kBM * kBK * 2;
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kStageBytes = P * kABytes + kBBytes;
    static constexpr int kStages = (192 * 1024 / kStageBytes) < 8 ? (192 * 1024 / kStageBytes) : 8;
    static constexpr int kBarOff = kStages * kStageBytes;   // full[S], empty[S], acc_full[2], acc_empty[2], tmem slot
    static constexpr int kSmem = kBarOff + (2 * kStages + 4) * 8 + 16 + 1024;
};
// kEpi = 1 (BN = 256, no K split): the tile holds the gate and up rows of the
// same 128 hidden units (columns 0-127 gate, 128-255 up: the weights packed so,
// n block j covering units 128 j ..); the epilogue writes h = silu(gate) * up as
// epi_parts (1-3) bf16 parts (C: bf16, rows ldc apart, parts HIDDEN_DIM columns
// apart), the down projection's A operand.
template <int BN, bool kOutF32, int kEpi = 0, int kParts = 1>
__global__ void __launch_bounds__(kThreads, 1)
gemm_bf16_tc_persistent(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ BMaps bm, void* C, int ldc, int K,
                        int kb_b, int m_blocks, int splits, int c_split_off, int m_valid, uint32_t* err, int epi_parts, int a_rows) {
    using L = Layout<BN, kParts>;
    constexpr int kStages = L::kStages;
    static_assert(BN % 16 == 0 && BN >= 32 && BN <= 256 && (BN & (BN - 1)) == 0, "tcgen05 M=128 tile: N a power of two in [32, 256]");
    static_assert(2 * BN <= 512, "two accumulators must fit the 512 TMEM columns");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
    uint64_t* empty = full + kStages;
    uint64_t* acc_full = empty + kStages;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_blocks = bm.end[2];
    const int ntiles = n_blocks * m_blocks, nitems = ntiles * splits;
    const int nkb = K / kParts / kBK / splits;   // K steps per work item, each covering every part
    // A boxes of a_rows rows (the map's box height: 128, or fewer when one m block holds
    // only that many valid rows; the rest of the A slot keeps stale data, which only
    // reaches padding rows of the result, never stored)
    const uint32_t stage_tx = (uint32_t)(kParts * a_rows * kBK * 2 + L::kBBytes);
    pdl_launch_dependents();

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; b++) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], 4); }
        fence_barrier_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(&map_a) : "memory");
        for (int s = 0; s < 3; s++)
            if (s == 0 || bm.end[s] > bm.end[s - 1]) asm volatile("prefetch.tensormap [%0];" ::"l"(&bm.map[s]) : "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, 2 * BN);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            // step `it` of the stage ring: work item blockIdx.x + (it / nkb) * gridDim.x, its K step it % nkb
            auto step = [&](uint32_t it, int& m0, int& n0, int& kb, const CUtensorMap*& mb) {
                const int w = blockIdx.x + (int)(it / (uint32_t)nkb) * (int)gridDim.x;
                if (w >= nitems) return false;
                const int t = w % ntiles, nb = t % n_blocks;
                kb = (w / ntiles) * nkb + (int)(it % (uint32_t)nkb);
                m0 = (t / n_blocks) * kBM;
                const int sg = nb < bm.end[0] ? 0 : (nb < bm.end[1] ? 1 : 2);
                mb = &bm.map[sg];
                n0 = (nb - (sg == 0 ? 0 : bm.end[sg - 1])) * BN;   // row in matrix sg
                return true;
            };
            int m0, n0, kb;
            const CUtensorMap* mb;
            // the ring's first stages: weight boxes while the previous kernel may still run
            // (no kernel writes the weights), activation boxes once it has finished
            uint32_t npre = 0;
            for (; npre < (uint32_t)kStages && step(npre, m0, n0, kb, mb); npre++) {
                mbar_arrive_expect_tx(&full[npre], stage_tx);
                tma_load_2d(smem + npre * L::kStageBytes + kParts * L::kABytes, mb, kb * kBK, n0, &full[npre]);
            }
            pdl_wait();
            for (uint32_t it = 0; it < npre; it++) {
                step(it, m0, n0, kb, mb);
                #pragma unroll
                for (int p = 0; p < kParts; p++)
                    tma_load_2d(smem + it * L::kStageBytes + p * L::kABytes, &map_a, (p * kb_b + kb) * kBK, m0, &full[it]);
            }
            // the rest: coordinates once per work item (a division per step would slow this thread
            // below the MMA rate)
            uint32_t it = 0;
            bool ok = true;
            for (int w = blockIdx.x; w < nitems && ok; w += gridDim.x) {
                const int t = w % ntiles, kb0 = (w / ntiles) * nkb;
                const int nb = t % n_blocks, mi0 = (t / n_blocks) * kBM;
                const int sg = nb < bm.end[0] ? 0 : (nb < bm.end[1] ? 1 : 2);
                const CUtensorMap* mbi = &bm.map[sg];
                const int ni0 = (nb - (sg == 0 ? 0 : bm.end[sg - 1])) * BN;   // row in matrix sg
                for (int k = kb0; k < kb0 + nkb; k++, it++) {
                    if (it < npre) continue;   // loaded above
                    const uint32_t s = it % kStages;
                    if (!mbar_wait(&empty[s], ((it / kStages) - 1) & 1u, kWaitNs)) { atomicOr(err, 1u); ok = false; break; }
                    uint8_t* st = smem + s * L::kStageBytes;
                    mbar_arrive_expect_tx(&full[s], stage_tx);
                    #pragma unroll
                    for (int p = 0; p < kParts; p++) tma_load_2d(st + p * L::kABytes, &map_a, (p * kb_b + k) * kBK, mi0, &full[s]);
                    tma_load_2d(st + kParts * L::kABytes, mbi, k * kBK, ni0, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t id = idesc_bf16_f32(kBM, BN);
            uint32_t it = 0, i = 0;
            bool ok = true;
            for (int w = blockIdx.x; w < nitems; w += gridDim.x, i++) {
                const uint32_t b = i & 1u, use = i >> 1;
                if (ok && use > 0 && !mbar_wait(&acc_empty[b], (use - 1) & 1u, kWaitNs)) { atomicOr(err, 8u); ok = false; }
                tc_fence_after();
                const uint32_t d = tmem + b * BN;
                for (int kb = 0; kb < nkb && ok; kb++, it++) {
                    const uint32_t s = it % kStages;
                    if (!mbar_wait(&full[s], (it / kStages) & 1u, kWaitNs)) { atomicOr(err, 2u); ok = false; break; }
                    tc_fence_after();
                    const uint32_t a = smem_addr(smem + s * L::kStageBytes), bb = a + kParts * L::kABytes;
                    #pragma unroll
                    for (int kk = 0; kk < kBK / kUmmaK; kk++)
                        #pragma unroll
                        for (int p = 0; p < kParts; p++)
                            mma_bf16(d, kmajor_sw128_desc(a + p * L::kABytes + kk * 32), kmajor_sw128_desc(bb + kk * 32), id,
                                     (kb | kk | p) != 0 ? 1u : 0u);
                    mma_commit(&empty[s]);
                }
                mma_commit(&acc_full[b]);   // the accumulator is complete (or abandoned: *err is set)
            }
        }
    } else {
        const int q = warp & 3;
        uint32_t i = 0;
        for (int w = blockIdx.x; w < nitems; w += gridDim.x, i++) {
            const uint32_t b = i & 1u, use = i >> 1;
            if (!mbar_wait(&acc_full[b], use & 1u, 2 * kWaitNs)) atomicOr(err, 4u);
            tc_fence_after();
            const int t = w % ntiles;
            const int n0 = (t % n_blocks) * BN + (w / ntiles) * c_split_off, m_w = (t / n_blocks) * kBM + 32 * q, m = m_w + lane;
            if constexpr (kEpi == 1) {
                static_assert(BN == 256, "the SwiGLU epilogue pairs 128 gate and 128 up columns");
                if (m_w < m_valid) {
                    const int u0 = (t % n_blocks) * 128;
                    #pragma unroll 1
                    for (int c = 0; c < 128; c += 32) {
                        float g[32], u[32];
                        tmem_ld32(tmem + b * BN + ((uint32_t)(32 * q) << 16) + (uint32_t)c, g);
                        tmem_ld32(tmem + b * BN + ((uint32_t)(32 * q) << 16) + (uint32_t)(128 + c), u);
                        if (m < m_valid) {
                            uint16_t* row = static_cast<uint16_t*>(C) + (size_t)m * ldc + u0 + c;
                            #pragma unroll
                            for (int i = 0; i < 32; i += 8) {
                                uint32_t h[4], md[4], lo[4];
                                #pragma unroll
                                for (int j = 0; j < 4; j++) {
                                    const float g0 = g[i + 2 * j], g1 = g[i + 2 * j + 1];
                                    split3x2((g0 / (1.0f + expf(-g0))) * u[i + 2 * j], (g1 / (1.0f + expf(-g1))) * u[i + 2 * j + 1], h[j], md[j],
                                             lo[j]);
                                }
                                *(uint4*)(row + i) = make_uint4(h[0], h[1], h[2], h[3]);
                                if (epi_parts > 1) *(uint4*)(row + HIDDEN_DIM + i) = make_uint4(md[0], md[1], md[2], md[3]);
                                if (epi_parts > 2) *(uint4*)(row + 2 * HIDDEN_DIM + i) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                            }
                        }
                    }
                }
            } else if (m_w < m_valid) {   // rows m_valid.. are padding: neither read back nor stored
                #pragma unroll 1
                for (int c = 0; c < BN; c += 32) {
                    float v[32];
                    tmem_ld32(tmem + b * BN + ((uint32_t)(32 * q) << 16) + (uint32_t)c, v);
                    if (m < m_valid) store32<kOutF32>(C, ldc, m, n0 + c, v);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);   // this warp has read its lanes of accumulator b
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, 2 * BN);
}

// ---------------------------------------------------------------------------
// Pair form: a cluster of two CTAs (on two SMs) computes 256 x BN output tiles
// with tcgen05.mma.cta_group::2.  CTA r of the pair loads rows 128 r .. 128 r +
// 127 of the tile's A and rows (BN / 2) r .. of its B per K step and receives
// its 128 rows of D (all BN columns) in its own tensor memory; the leader CTA
// (rank 0) issues every MMA of the pair, reading both CTAs' shared memory.  Per
// CTA and K step 16 KB of A and BN x 64 bytes of B cross from L2 for 128 x BN
// x 64 of MMA work (at BN = 256: 32 KB, against 48 KB for a single-CTA tile),
// so the L2 -> SM stream that bounds the single-CTA form carries a third less.
// Both CTAs' TMA loads complete on the leader's stage barrier; the leader's MMA
// commits arrive on both CTAs' barriers (multicast commit: stage free, tile's
// accumulator complete); the epilogue warps of both CTAs hand each accumulator
// back on the leader's barrier.  No TMA multicast: each CTA loads its own
// boxes into its own shared memory.  Same work items, split K, row padding and
// epilogues as the single-CTA form, with 256-row m blocks, but eight epilogue
// warps (kPairThreads): two per TMEM lane quarter, each draining half of the
// tile's columns, so the last tile's epilogue, which no MMA work hides, takes
// half as long.
//
// A that holds P bf16 parts of each activation side by side (A = [part 0 |
// part 1 | ..], each Kb = K / P columns wide, against one B of Kb columns): a
// stage holds the P A boxes of one K step and the B box once, and the MMA
// thread issues the P products of each 16-wide K slice against the same B
// slice, so B crosses from L2 once per K step instead of once per part (two
// parts: 48 KB per stage and CTA for 2 x 128 x BN x 64 of MMA work instead of
// 64 KB).
template <int BN, int P>
struct PairLayout {
    static_assert(P >= 1 && P <= 3, "one to three activation parts");
    static constexpr int kABytes = kBM * kBK * 2;          // this CTA's 128 rows of one part of A
    static constexpr int kBBytes = (BN / 2) * kBK * 2;     // this CTA's BN / 2 rows of B
    static constexpr int kStageBytes = P * kABytes + kBBytes;
    static constexpr int kStages = (192 * 1024 / kStageBytes) < 8 ? (192 * 1024 / kStageBytes) : 8;
    static constexpr int kBarOff = kStages * kStageBytes;
    static constexpr int kSmem = kBarOff + (2 * kStages + 4) * 8 + 16 + 1024;
};

// Every layout the host instantiates fits one CTA's shared memory (227 KB).
static_assert(Layout<256, 3>::kSmem <= 227 * 1024 && Layout<256, 2>::kSmem <= 227 * 1024 && Layout<256, 1>::kSmem <= 227 * 1024 &&
                  Layout<128, 3>::kSmem <= 227 * 1024 && Layout<128, 1>::kSmem <= 227 * 1024,
              "single-CTA GEMM stages must fit shared memory");
static_assert(PairLayout<256, 3>::kSmem <= 227 * 1024 && PairLayout<256, 2>::kSmem <= 227 * 1024 && PairLayout<256, 1>::kSmem <= 227 * 1024,
              "pair GEMM stages must fit shared memory");
static_assert(Layout<256, 3>::kStages >= 2 && PairLayout<256, 3>::kStages >= 2, "at least two stages in flight");

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The shared::cluster address of the same shared-memory location in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t d;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(saddr), "r"(rank));
    return d;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// 2-D tile load into this CTA's shared memory whose completion is counted on
// the barrier at shared::cluster address `bar` (the leader's).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_addr(dst)), "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on `bar` (the same offset) in both CTAs of the pair once every MMA
// this thread issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 ::"r"(smem_addr(bar)), "h"((uint16_t)3)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}

// The q|k|v epilogue (QkvOut) of one row m (position qo.pos0 + m) and one
// head: ta addresses the head's 128 fp32 accumulator columns of this warp's
// TMEM lanes; hd is the head's 128-column block of the GEMM (0-15 q, 16-23 k,
// 24-31 v).  row_ok: the row is valid (rows at m_valid and beyond are padding
// and stored nowhere); pair_ok: so is the other row of this lane's pair (lanes
// 2i, 2i + 1) and the pair's first position is even.  Warp-collective (TMEM
// loads; the v^T stores pair adjacent positions by a shuffle).  q and k heads
// are read twice (sum of squares, then 32 + 32 rotation partners at a time) so
// that at most 64 values are live.
template <typename T>
__device__ __forceinline__ void store_row32(T* dst, const float (&v)[32]);
template <>
__device__ __forceinline__ void store_row32<float>(float* dst, const float (&v)[32]) {
    float4* d = reinterpret_cast<float4*>(dst);
    #pragma unroll
    for (int i = 0; i < 8; i++) d[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}
template <>
__device__ __forceinline__ void store_row32<uint16_t>(uint16_t* dst, const float (&v)[32]) {
    uint4* d = reinterpret_cast<uint4*>(dst);
    #pragma unroll
    for (int i = 0; i < 4; i++) {
        uint32_t w[4];
        #pragma unroll
        for (int e = 0; e < 4; e++) w[e] = (uint32_t)f2bf(v[8 * i + 2 * e]) | ((uint32_t)f2bf(v[8 * i + 2 * e + 1]) << 16);
        d[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__device__ __forceinline__ void qkv_head_out(const QkvOut& qo, int hd, int m, bool row_ok, bool pair_ok, uint32_t ta) {
    const int pos = qo.pos0 + m;
    const bool is_q = hd < N_HEADS, is_v = hd >= N_HEADS + N_KV_HEADS;
    const int h = is_q ? hd : hd - N_HEADS - (is_v ? N_KV_HEADS : 0);
    if (!is_v) {   // QK-norm, then RoPE (rotate-half pairs j, j + 64 at angle j)
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
        #pragma unroll 1
        for (int c = 0; c < HEAD_DIM; c += 32) {
            float v[32];
            tmem_ld32(ta + (uint32_t)c, v);
            #pragma unroll
            for (int j = 0; j < 32; j++) s4[j & 3] = fmaf(v[j], v[j], s4[j & 3]);
        }
        const float rs = 1.0f / sqrtf(((s4[0] + s4[1]) + (s4[2] + s4[3])) * (1.0f / HEAD_DIM) + EPS);
        const uint4* g4 = reinterpret_cast<const uint4*>(is_q ? qo.qn : qo.kn);
        const float4* cs = reinterpret_cast<const float4*>(qo.rope + (size_t)(row_ok ? pos : 0) * HEAD_DIM);
        float* qd = qo.q + (size_t)m * Q_DIM + h * HEAD_DIM;
        uint16_t* kd = qo.kc + ((size_t)h * SEQ_LEN + pos) * HEAD_DIM;
        #pragma unroll 1
        for (int c = 0; c < HEAD_DIM / 2; c += 32) {
            float a[32], b[32];
            tmem_ld32(ta + (uint32_t)c, a);
            tmem_ld32(ta + (uint32_t)(c + HEAD_DIM / 2), b);
            #pragma unroll
            for (int i = 0; i < 4; i++) {
                const uint4 ga = __ldg(g4 + c / 8 + i), gb = __ldg(g4 + (c + HEAD_DIM / 2) / 8 + i);
                const uint32_t wa[4] = {ga.x, ga.y, ga.z, ga.w}, wb[4] = {gb.x, gb.y, gb.z, gb.w};
                #pragma unroll
                for (int e = 0; e < 4; e++) {
                    a[8 * i + 2 * e] = (a[8 * i + 2 * e] * rs) * bf_lo(wa[e]);
                    a[8 * i + 2 * e + 1] = (a[8 * i + 2 * e + 1] * rs) * bf_hi(wa[e]);
                    b[8 * i + 2 * e] = (b[8 * i + 2 * e] * rs) * bf_lo(wb[e]);
                    b[8 * i + 2 * e + 1] = (b[8 * i + 2 * e + 1] * rs) * bf_hi(wb[e]);
                }
            }
            #pragma unroll
            for (int i = 0; i < 8; i++) {
                const float4 co = __ldg(cs + c / 4 + i), si = __ldg(cs + (c + HEAD_DIM / 2) / 4 + i);
                const float cj[4] = {co.x, co.y, co.z, co.w}, sj[4] = {si.x, si.y, si.z, si.w};
                #pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float x0 = a[4 * i + e], x1 = b[4 * i + e];
                    a[4 * i + e] = x0 * cj[e] - x1 * sj[e];
                    b[4 * i + e] = x0 * sj[e] + x1 * cj[e];
                }
            }
            if (row_ok) {
                if (is_q) {
                    store_row32(qd + c, a);
                    store_row32(qd + c + HEAD_DIM / 2, b);
                } else {
                    store_row32(kd + c, a);
                    store_row32(kd + c + HEAD_DIM / 2, b);
                }
            }
        }
        return;
    }
    uint16_t* vd = qo.vc + ((size_t)h * SEQ_LEN + pos) * HEAD_DIM;
    uint16_t* t = qo.vt + (size_t)h * HEAD_DIM * SEQ_LEN;
    const bool odd = (threadIdx.x & 1) != 0;
    #pragma unroll 1
    for (int c = 0; c < HEAD_DIM; c += 32) {
        float v[32];
        tmem_ld32(ta + (uint32_t)c, v);
        if (row_ok) store_row32(vd + c, v);
        // v^T: for each dim, consecutive lanes' positions are consecutive
        #pragma unroll
        for (int j = 0; j < 32; j += 2) {
            const float recv = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[j + 1], 1);
            if (pair_ok) {   // even lane: dim c + j of positions pos, pos + 1; odd lane: dim c + j + 1 of pos - 1, pos
                if (!odd)
                    *reinterpret_cast<uint32_t*>(t + (size_t)(c + j) * SEQ_LEN + pos) = (uint32_t)f2bf(v[j]) | ((uint32_t)f2bf(recv) << 16);
                else
                    *reinterpret_cast<uint32_t*>(t + (size_t)(c + j + 1) * SEQ_LEN + pos - 1) =
                        (uint32_t)f2bf(recv) | ((uint32_t)f2bf(v[j + 1]) << 16);
            } else if (row_ok) {
                t[(size_t)(c + j) * SEQ_LEN + pos] = f2bf(v[j]);
                t[(size_t)(c + j + 1) * SEQ_LEN + pos] = f2bf(v[j + 1]);
            }
        }
    }
}

// grid: an even number of CTAs (clusters of two), at most one per SM;
// m_blocks counts 256-row blocks; B's maps have (BN / 2)-row boxes.
template <int BN, bool kOutF32, int kEpi = 0, int kParts = 1>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
gemm_bf16_tc_pair(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ BMaps bm, void* C, int ldc, int K, int kb_b,
                  int m_blocks, int splits, int c_split_off, int m_valid, uint32_t* err, int epi_parts, const QkvOut qo) {
    using L = PairLayout<BN, kParts>;
    constexpr int kSt = L::kStages;
    static_assert(BN == 128 || BN == 256, "pair tiles: 256 x 128 or 256 x 256");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
    uint64_t* empty = full + kSt;
    uint64_t* acc_full = empty + kSt;
    uint64_t* acc_empty = acc_full + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
    const int n_blocks = bm.end[2];
    const int ntiles = n_blocks * m_blocks, nitems = ntiles * splits;
    const int nkb = K / kParts / kBK / splits;   // K steps per work item, each covering every part
    pdl_launch_dependents();

    if (threadIdx.x == 0) {
        for (int s = 0; s < kSt; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int b = 0; b < 2; b++) { mbar_init(&acc_full[b], 1); mbar_init(&acc_empty[b], 16); }   // 8 epilogue warps x 2 CTAs
        fence_barrier_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(&map_a) : "memory");
        for (int s = 0; s < 3; s++)
            if (s == 0 || bm.end[s] > bm.end[s - 1]) asm volatile("prefetch.tensormap [%0];" ::"l"(&bm.map[s]) : "memory");
    }
    if (warp == 1) tmem_alloc_pair(tmem_slot, 2 * BN);
    tc_fence_before();
    cluster_sync_all();   // both CTAs' barriers initialised and tensor memory allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t full0 = map_to_rank(smem_addr(full), 0);          // the leader's stage barriers
    const uint32_t acc_empty0 = map_to_rank(smem_addr(acc_empty), 0);

    if (warp == 0) {
        if (lane == 0) {
            // step `it` of the stage ring: work item pair + (it / nkb) * npairs, its K step it % nkb
            auto step = [&](uint32_t it, int& m0, int& n0, int& kb, const CUtensorMap*& mb) {
                const int w = pair + (int)(it / (uint32_t)nkb) * npairs;
                if (w >= nitems) return false;
                const int t = w % ntiles, nb = t % n_blocks;
                kb = (w / ntiles) * nkb + (int)(it % (uint32_t)nkb);
                m0 = (t / n_blocks) * 2 * kBM + kBM * (int)rank;
                const int sg = nb < bm.end[0] ? 0 : (nb < bm.end[1] ? 1 : 2);
                mb = &bm.map[sg];
                n0 = (nb - (sg == 0 ? 0 : bm.end[sg - 1])) * BN + (BN / 2) * (int)rank;
                return true;
            };
            int m0, n0, kb;
            const CUtensorMap* mb;
            // the ring's first stages: weight boxes while the previous kernel may still run
            // (no kernel writes the weights), activation boxes once it has finished
            uint32_t npre = 0;
            for (; npre < (uint32_t)kSt && step(npre, m0, n0, kb, mb); npre++) {
                if (rank == 0) mbar_arrive_expect_tx(&full[npre], 2 * L::kStageBytes);   // both CTAs' bytes
                tma_load_2d_pair(smem + npre * L::kStageBytes + kParts * L::kABytes, mb, kb * kBK, n0, full0 + 8u * npre);
            }
            pdl_wait();
            for (uint32_t it = 0; it < npre; it++) {
                step(it, m0, n0, kb, mb);
                #pragma unroll
                for (int p = 0; p < kParts; p++)
                    tma_load_2d_pair(smem + it * L::kStageBytes + p * L::kABytes, &map_a, (p * kb_b + kb) * kBK, m0, full0 + 8u * it);
            }
            // the rest: coordinates once per work item (a division per step would slow this thread
            // below the MMA rate)
            uint32_t it = 0;
            bool ok = true;
            for (int w = pair; w < nitems && ok; w += npairs) {
                const int t = w % ntiles, kb0 = (w / ntiles) * nkb;
                const int nb = t % n_blocks, mi0 = (t / n_blocks) * 2 * kBM + kBM * (int)rank;
                const int sg = nb < bm.end[0] ? 0 : (nb < bm.end[1] ? 1 : 2);
                const CUtensorMap* mbi = &bm.map[sg];
                const int ni0 = (nb - (sg == 0 ? 0 : bm.end[sg - 1])) * BN + (BN / 2) * (int)rank;
                for (int k = kb0; k < kb0 + nkb; k++, it++) {
                    if (it < npre) continue;   // loaded above
                    const uint32_t s = it % kSt;
                    if (!mbar_wait(&empty[s], ((it / kSt) - 1) & 1u, kWaitNs)) { atomicOr(err, 1u); ok = false; break; }
                    uint8_t* st = smem + s * L::kStageBytes;
                    if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * L::kStageBytes);   // both CTAs' bytes
                    #pragma unroll
                    for (int p = 0; p < kParts; p++) tma_load_2d_pair(st + p * L::kABytes, &map_a, (p * kb_b + k) * kBK, mi0, full0 + 8u * s);
                    tma_load_2d_pair(st + kParts * L::kABytes, mbi, k * kBK, ni0, full0 + 8u * s);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t id = idesc_bf16_f32(2 * kBM, BN);
            uint32_t it = 0, i = 0;
            bool ok = true;
            for (int w = pair; w < nitems; w += npairs, i++) {
                const uint32_t b = i & 1u, use = i >> 1;
                if (ok && use > 0 && !mbar_wait(&acc_empty[b], (use - 1) & 1u, kWaitNs)) { atomicOr(err, 8u); ok = false; }
                tc_fence_after();
                const uint32_t d = tmem + b * BN;
                for (int kb = 0; kb < nkb && ok; kb++, it++) {
                    const uint32_t s = it % kSt;
                    if (!mbar_wait(&full[s], (it / kSt) & 1u, kWaitNs)) { atomicOr(err, 2u); ok = false; break; }
                    tc_fence_after();
                    const uint32_t a = smem_addr(smem + s * L::kStageBytes), bb = a + kParts * L::kABytes;
                    #pragma unroll
                    for (int kk = 0; kk < kBK / kUmmaK; kk++)
                        #pragma unroll
                        for (int p = 0; p < kParts; p++)
                            mma_bf16_pair(d, kmajor_sw128_desc(a + p * L::kABytes + kk * 32), kmajor_sw128_desc(bb + kk * 32), id,
                                          (kb | kk | p) != 0 ? 1u : 0u);
                    mma_commit_pair(&empty[s]);
                }
                mma_commit_pair(&acc_full[b]);   // complete (or abandoned: *err is set) in both CTAs
            }
        }
    } else {
        // warps 2-9: warp w reads TMEM lanes 32 (w % 4) .. + 31 (the rows it may access) and
        // half eh of the tile's columns (for the q|k|v epilogue: head eh of the tile)
        const int q = warp & 3, eh = (warp - 2) >> 2;
        uint32_t i = 0;
        for (int w = pair; w < nitems; w += npairs, i++) {
            const uint32_t b = i & 1u, use = i >> 1;
            if (!mbar_wait(&acc_full[b], use & 1u, 2 * kWaitNs)) atomicOr(err, 4u);
            tc_fence_after();
            const int t = w % ntiles;
            const int n0 = (t % n_blocks) * BN + (w / ntiles) * c_split_off;
            const int m_w = (t / n_blocks) * 2 * kBM + kBM * (int)rank + 32 * q, m = m_w + lane;
            if constexpr (kEpi == 1) {
                static_assert(kEpi != 1 || BN == 256, "the SwiGLU epilogue pairs 128 gate and 128 up columns");
                if (m_w < m_valid) {
                    const int u0 = (t % n_blocks) * 128;
                    #pragma unroll 1
                    for (int c = 64 * eh; c < 64 * eh + 64; c += 32) {
                        float g[32], u[32];
                        tmem_ld32(tmem + b * BN + ((uint32_t)(32 * q) << 16) + (uint32_t)c, g);
                        tmem_ld32(tmem + b * BN + ((uint32_t)(32 * q) << 16) + (uint32_t)(128 + c), u);
                        if (m < m_valid) {
                            uint16_t* row = static_cast<uint16_t*>(C) + (size_t)m * ldc + u0 + c;
                            #pragma unroll
                            for (int i = 0; i < 32; i += 8) {
                                uint32_t h[4], md[4], lo[4];
                                #pragma unroll
                                for (int j = 0; j < 4; j++) {
                                    const float g0 = g[i + 2 * j], g1 = g[i + 2 * j + 1];
                                    split3x2((g0 / (1.0f + expf(-g0))) * u[i + 2 * j], (g1 / (1.0f + expf(-g1))) * u[i + 2 * j + 1], h[j], md[j],
                                             lo[j]);
                                }
                                *(uint4*)(row + i) = make_uint4(h[0], h[1], h[2], h[3]);
                                if (epi_parts > 1) *(uint4*)(row + HIDDEN_DIM + i) = make_uint4(md[0], md[1], md[2], md[3]);
                                if (epi_parts > 2) *(uint4*)(row + 2 * HIDDEN_DIM + i) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                            }
                        }
                    }
                }
            } else if constexpr (kEpi == 2) {
                static_assert(kEpi != 2 || BN == 256, "the q|k|v epilogue takes two heads per tile");
                if (m_w < m_valid) {
                    const bool row_ok = m < m_valid, pair_ok = (qo.pos0 & 1) == 0 && (m | 1) < m_valid;
                    qkv_head_out(qo, (t % n_blocks) * 2 + eh, m, row_ok, pair_ok,
                                 tmem + b * BN + ((uint32_t)(32 * q) << 16) + (uint32_t)(HEAD_DIM * eh));
                }
            } else if (m_w < m_valid) {
                #pragma unroll 1
                for (int c = eh * BN / 2; c < (eh + 1) * BN / 2; c += 32) {
                    float v[32];
                    tmem_ld32(tmem + b * BN + ((uint32_t)(32 * q) << 16) + (uint32_t)c, v);
                    if (m < m_valid) store32<kOutF32>(C, ldc, m, n0 + c, v);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(acc_empty0 + 8u * b);   // this warp has read its lanes of accumulator b
        }
    }
    tc_fence_before();
    cluster_sync_all();   // every MMA, commit and remote arrival of the pair has landed
    if (warp == 1) tmem_dealloc_pair(tmem, 2 * BN);
}

}  // namespace tc
}  // namespace qb
