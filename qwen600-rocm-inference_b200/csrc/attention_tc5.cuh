// attention_tc5.cuh — causal GQA attention of a prompt pass on the sm_100a
// tensor cores (tcgen05.mma, kind::f16: bf16 operands from shared memory,
// fp32 accumulators in TMEM).  No reference counterpart: the reference runs
// its decode attention once per prompt token (main.cu:141-145 over
// qwen_model.cuh:551-614).
//
// One CTA per (64 query positions, KV head hk): the 128 rows of its tiles are
// the 64 positions of q head 2 hk (rows 0-63) and of q head 2 hk + 1 (rows
// 64-127), so every K/V tile serves both heads.  One pass over the key tiles
// (64 keys each, up to the block's last query; heaviest blocks first) with an
// online softmax: S = Q K^T into TMEM (two buffers); each row keeps a running
// max m and sum l; P = exp2(S c - m c) (the 1/sqrt(d) scale folded into c) is
// written unnormalised into shared memory and O += P V accumulates in TMEM.
// When a tile raises a row's max by more than kA5Rescale (base-2 exponent
// units) the row first scales its O columns and l by exp2((m_old - m_new) c)
// in tensor memory (after the previous P V product has completed) and adopts
// the new max; smaller rises keep the old max, so P stays below 2^kA5Rescale
// and O and l carry the same factor, which the final division by l removes.
// Q enters as two bf16 parts side by side along K (K' = 256 against K read
// twice), P likewise (K' = 128 against V^T read twice): 16 mantissa bits of
// each fp32 operand, relative error <= 2^-16 (K and V are bf16 in the cache).
// Q and P are the MMAs' A operands and live in tensor memory (Q written once
// by the softmax threads, P written over each tile with tcgen05.st), so the
// MMAs read only K and V^T from shared memory: with both operands in shared
// memory the products were bound by its bandwidth (6-8 KB per MMA
// instruction).  P's parts are formed with integer arithmetic (split2x2_int)
// so that the conversion unit only evaluates exp2.  K tiles come by TMA from
// the cache ([head][position][dim]), V tiles by TMA from a transposed copy of
// the layer's V ([head][dim][position], transpose_v_kernel) so that keys are
// contiguous; both K-major SW128 tiles.  Warps: 0 TMA producer (K and V^T
// tiles in the order the MMAs use them: S of tile t + 1 is issued before P V
// of tile t, so the softmax of one tile overlaps the S product of the next),
// 1 TMEM allocator and MMA issuer, 2-9 Q loading, softmax and epilogue: warp w
// reads TMEM lanes 32 (w % 4) .. (the rows it may access), warps 2-5 columns
// 0-31 of each S tile (O columns 0-63) and warps 6-9 columns 32-63 (O columns
// 64-127); the two warps of a row agree on each tile's max through shared
// memory, so both halves use the same m.  Every wait is bounded: on expiry the
// thread sets *err and stops waiting; the TMEM allocation is always released.
#pragma once
#include "gemm_tc.cuh"
#include "prefill_kernels.cuh"

namespace qb {
namespace pf {

constexpr int kA5Keys = 64;                       // keys per tile
constexpr int kA5Threads = 320;                   // warps 0 producer, 1 MMA, 2-9 softmax (two per TMEM lane quarter)
constexpr int kA5KBytes = 2 * kA5Keys * 128;      // a K tile: 2 blocks (dim halves) of 64 rows x 128 B
constexpr int kA5VBytes = HEAD_DIM * 128;         // a V^T tile: 128 rows (dims) x 128 B (64 keys)

// V of one layer, [head][position][dim] -> [head][dim][position] for positions
// [0, n): 64 x 64 tiles through shared memory.  grid (ceil(n / 64), 2, N_KV_HEADS), block (64, 8).
__global__ void transpose_v_kernel(const uint16_t* __restrict__ vc_l, uint16_t* __restrict__ vt, int n) {
    pdl_launch_dependents();
    pdl_wait();
    __shared__ uint16_t t[64][66];
    const int p0 = blockIdx.x * 64, d0 = blockIdx.y * 64, hk = blockIdx.z;
    const uint16_t* src = vc_l + (size_t)hk * SEQ_LEN * HEAD_DIM;
    for (int i = threadIdx.y; i < 64; i += 8) {
        const int p = p0 + i;
        t[i][threadIdx.x] = p < n ? src[(size_t)p * HEAD_DIM + d0 + threadIdx.x] : (uint16_t)0;
    }
    __syncthreads();
    uint16_t* dst = vt + ((size_t)hk * HEAD_DIM + d0) * SEQ_LEN;
    for (int i = threadIdx.y; i < 64; i += 8)
        if (p0 + threadIdx.x < n) dst[(size_t)i * SEQ_LEN + p0 + threadIdx.x] = t[threadIdx.x][i];
}

constexpr float kA5Rescale = 8.0f;                 // base-2 exponent rise of a row's max that rescales O
constexpr int kA5KStages = 4;                      // K tiles in flight
constexpr int kA5VStages = 3;                      // V^T tiles in flight
// Tensor memory (all 512 columns: one CTA per SM).  Q and P are MMA A operands
// read from tensor memory, two bf16 values per 32-bit column (K-consecutive
// pairs, the first in the low half), so the MMAs read only K and V^T from
// shared memory.
constexpr uint32_t kTmQ = 0;     // Q: hi parts of dims 0-127 in columns 0-63, mid parts in 64-127
constexpr uint32_t kTmS = 128;   // S buffers b: columns 128 + 64 b .. (fp32)
constexpr uint32_t kTmO = 256;   // O: columns 256-383 (fp32)
constexpr uint32_t kTmP = 384;   // P buffers b: 384 + 64 b: hi parts of keys 0-63 in 32 columns, then mid parts
struct A5Layout {
    static constexpr int kK = 0;
    static constexpr int kV = kK + kA5KStages * kA5KBytes;
    static constexpr int kBar = kV + kA5VStages * kA5VBytes;
    static constexpr int kXm = kBar + 32 * 8;            // [2 tiles][2 halves][128 rows] half-row maxima
    static constexpr int kLs = kXm + 2 * 2 * 128 * 4;    // [2 halves][128 rows] half-row sums at the end
    static constexpr int kSmem = kLs + 2 * 128 * 4 + 1024;
};
static_assert(A5Layout::kSmem <= 227 * 1024, "attention tiles must fit one CTA's shared memory");
static_assert(2 * A5Layout::kSmem > 228 * 1024, "one CTA per SM: the kernel allocates all of tensor memory");

// Two bf16 parts of the non-negative finite values a and b (< 2^127) with
// integer arithmetic instead of conversion instructions, so the conversion
// unit is left to exp2: hi = the value rounded to 8 significant bits (adding
// half a unit of the 16 dropped bits, then truncating), mid = the remainder
// (exact in fp32) truncated to 8 significant bits; |a - hi - mid| < 2^-15 |a|.
// Packed like cvt_bf16x2 (a in the low half).
__device__ __forceinline__ void split2x2_int(float a, float b, uint32_t& h, uint32_t& m) {
    const uint32_t ra = __float_as_uint(a) + 0x8000u, rb = __float_as_uint(b) + 0x8000u;
    const float ma = a - __uint_as_float(ra & 0xffff0000u), mb = b - __uint_as_float(rb & 0xffff0000u);
    h = __byte_perm(ra, rb, 0x7632);
    m = __byte_perm(__float_as_uint(ma), __float_as_uint(mb), 0x7632);
}
// 2^x by the conversion unit's approximation (ex2.approx, subnormal results
// flushed to zero: a softmax weight below 2^-126 contributes nothing).
__device__ __forceinline__ float ex2_ftz(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

// 16 or 32 consecutive 32-bit columns of this warp's 32 TMEM lanes (one row per
// lane); complete after tmem_wait_st.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
          "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
          "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
          "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
          "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])),
          "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
          "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
          "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])),
          "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// D (TMEM) += A (TMEM, 128 rows x 16, two bf16 per column) . B (shared memory descriptor)^T
__device__ __forceinline__ void mma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate)
        : "memory");
}

// grid: rows / 64 * N_KV_HEADS CTAs, kA5Threads threads, A5Layout::kSmem bytes.
// map_k: the layer's K cache as [N_KV_HEADS * SEQ_LEN rows][128], boxes 64 x 64;
// map_v: the transposed V as [N_KV_HEADS * 128 rows][SEQ_LEN], boxes 128 x 64.
// Output: the O projection's A operand, `parts` (1-3) bf16 parts of each value,
// Q_DIM columns apart, in rows of As (ld_as apart).
__global__ void __launch_bounds__(kA5Threads, 1)
attention_tc5_kernel(const __grid_constant__ CUtensorMap map_k, const __grid_constant__ CUtensorMap map_v, const float* __restrict__ Q,
                     int pos0, uint16_t* __restrict__ As, int ld_as, int parts, uint32_t* err) {
    using namespace qb::tc;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + A5Layout::kBar);
    uint64_t* kfull = bars;                          // [kA5KStages]
    uint64_t* kempty = bars + kA5KStages;            // [kA5KStages]
    uint64_t* vfull = bars + 2 * kA5KStages;         // [kA5VStages]
    uint64_t* vempty = vfull + kA5VStages;           // [kA5VStages]
    uint64_t* sfull = vempty + kA5VStages;           // [2] S buffer written (MMA -> softmax)
    uint64_t* sempty = sfull + 2;                    // [2] S buffer read (softmax -> MMA), 8 arrivals
    uint64_t* pfull = sfull + 4;                     // [2] P buffer written and O rescaled (softmax -> MMA), 8 arrivals
    uint64_t* pempty = sfull + 6;                    // [2] P V product of the buffer complete (MMA -> softmax)
    uint64_t* ofull = sfull + 8;                     // O complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sfull + 9);
    static_assert((2 * kA5KStages + 2 * kA5VStages + 10) * 8 <= 32 * 8, "barriers fit their 256 bytes");
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int nqb = gridDim.x / N_KV_HEADS;
    const int qb = nqb - 1 - (int)blockIdx.x / N_KV_HEADS, hk = (int)blockIdx.x % N_KV_HEADS;
    const int q0 = qb * kAttBlock;
    const int last = min(pos0 + q0 + kAttBlock - 1, SEQ_LEN - 1);
    const int T = last / kA5Keys + 1;   // key tiles
    pdl_launch_dependents();

    if (tid == 0) {
        for (int s = 0; s < kA5KStages; s++) { mbar_init(&kfull[s], 1); mbar_init(&kempty[s], 1); }
        for (int s = 0; s < kA5VStages; s++) { mbar_init(&vfull[s], 1); mbar_init(&vempty[s], 1); }
        for (int b = 0; b < 2; b++) { mbar_init(&sfull[b], 1); mbar_init(&sempty[b], 8); mbar_init(&pfull[b], 8); mbar_init(&pempty[b], 1); }
        mbar_init(ofull, 1);
        fence_barrier_init();
        asm volatile("prefetch.tensormap [%0];" ::"l"(&map_k) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&map_v) : "memory");
    }
    if (warp == 1) tmem_alloc(tmem_slot, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();   // Q, K and V come from the kernels before this one

    if (warp == 0) {
        if (lane == 0) {
            // K(0), K(1), V(0), K(2), V(1), ...: the order the MMAs consume them
            bool ok = true;
            auto load_v = [&](int t) {
                const uint32_t sv = (uint32_t)t % kA5VStages;
                if (t >= kA5VStages && !mbar_wait(&vempty[sv], ((t / kA5VStages) - 1) & 1u, tc::kWaitNs)) { atomicOr(err, 16u); return false; }
                mbar_arrive_expect_tx(&vfull[sv], kA5VBytes);
                tma_load_2d(smem + A5Layout::kV + sv * kA5VBytes, &map_v, t * kA5Keys, hk * HEAD_DIM, &vfull[sv]);
                return true;
            };
            for (int t = 0; t < T && ok; t++) {
                const uint32_t s = (uint32_t)t % kA5KStages;
                if (t >= kA5KStages && !mbar_wait(&kempty[s], ((t / kA5KStages) - 1) & 1u, tc::kWaitNs)) { atomicOr(err, 16u); ok = false; break; }
                uint8_t* kd = smem + A5Layout::kK + s * kA5KBytes;
                mbar_arrive_expect_tx(&kfull[s], kA5KBytes);
                tma_load_2d(kd, &map_k, 0, hk * SEQ_LEN + t * kA5Keys, &kfull[s]);
                tma_load_2d(kd + kA5Keys * 128, &map_k, 64, hk * SEQ_LEN + t * kA5Keys, &kfull[s]);
                if (t >= 1) ok = load_v(t - 1);
            }
            if (ok && T > 0) load_v(T - 1);
        }
    } else if (warp == 1) {
        named_bar(3, 288);   // Q is in tensor memory
        tc_fence_after();
        if (lane == 0) {
            constexpr uint32_t id_s = idesc_bf16_f32(128, kA5Keys), id_o = idesc_bf16_f32(128, HEAD_DIM);
            bool ok = true;
            // O += P V for tile t: A = P buffer t & 1 (hi parts of the 64 keys, then mid parts), B = V^T stage
            auto pv = [&](int t) {
                const uint32_t pb = (uint32_t)t & 1u, puse = (uint32_t)t >> 1, sv = (uint32_t)t % kA5VStages;
                if (!mbar_wait(&pfull[pb], puse & 1u, tc::kWaitNs) || !mbar_wait(&vfull[sv], (t / kA5VStages) & 1u, tc::kWaitNs)) {
                    atomicOr(err, 32u);
                    return false;
                }
                tc_fence_after();
                const uint32_t vb = smem_addr(smem + A5Layout::kV + sv * kA5VBytes);
                #pragma unroll
                for (int j = 0; j < 2; j++)
                    #pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        mma_bf16_ts(tmem + kTmO, tmem + kTmP + 64 * pb + 32 * j + 8 * kk, kmajor_sw128_desc(vb + kk * 32), id_o,
                                    (t | j | kk) != 0 ? 1u : 0u);
                mma_commit(&vempty[sv]);
                mma_commit(&pempty[pb]);
                return true;
            };
            for (int t = 0; t < T && ok; t++) {
                const uint32_t b = (uint32_t)t & 1u, use = (uint32_t)t >> 1, s = (uint32_t)t % kA5KStages;
                if (use > 0 && !mbar_wait(&sempty[b], (use - 1) & 1u, tc::kWaitNs)) { atomicOr(err, 32u); ok = false; break; }
                if (!mbar_wait(&kfull[s], (t / kA5KStages) & 1u, tc::kWaitNs)) { atomicOr(err, 32u); ok = false; break; }
                tc_fence_after();
                // S[b] = Q K^T: K' = 256 (Q hi | mid, from tensor memory) against the K tile read twice
                const uint32_t kb = smem_addr(smem + A5Layout::kK + s * kA5KBytes);
                #pragma unroll
                for (int j = 0; j < 4; j++)
                    #pragma unroll
                    for (int kk = 0; kk < 4; kk++)
                        mma_bf16_ts(tmem + kTmS + b * kA5Keys, tmem + kTmQ + 32 * j + 8 * kk,
                                    kmajor_sw128_desc(kb + (j & 1) * (kA5Keys * 128) + kk * 32), id_s, (j | kk) != 0 ? 1u : 0u);
                mma_commit(&kempty[s]);
                mma_commit(&sfull[b]);
                if (t >= 1) ok = pv(t - 1);
            }
            if (ok && T > 0) pv(T - 1);
            mma_commit(ofull);
        }
    } else {
        const int q = warp & 3, half = (warp - 2) >> 2, m = 32 * q + lane;
        const int qp = pos0 + q0 + (m & 63);
        const uint32_t lane_off = (uint32_t)(32 * q) << 16;
        float* xm = reinterpret_cast<float*>(smem + A5Layout::kXm);
        float* ls = reinterpret_cast<float*>(smem + A5Layout::kLs);
        // Q row m, dims 64 half .. +63, as two bf16 parts -> tensor memory (hi, mid)
        {
            const float4* src = reinterpret_cast<const float4*>(Q + (size_t)(q0 + (m & 63)) * Q_DIM + 128 * (2 * hk + (m >> 6)) + 64 * half);
            #pragma unroll 1
            for (int c = 0; c < 2; c++) {
                uint32_t hw[16], mw[16], lw;
                #pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float4 a = src[8 * c + i];
                    split3x2(a.x, a.y, hw[2 * i], mw[2 * i], lw);
                    split3x2(a.z, a.w, hw[2 * i + 1], mw[2 * i + 1], lw);
                }
                tmem_st16(tmem + lane_off + kTmQ + 32 * half + 16 * c, hw);
                tmem_st16(tmem + lane_off + kTmQ + 64 + 32 * half + 16 * c, mw);
            }
            tmem_wait_st();
        }
        tc_fence_before();
        named_bar(3, 288);
        const float c2 = 1.4426950408889634f / sqrtf((float)HEAD_DIM);
        float mrun = -INFINITY, l = 0.f;
        bool ok = true;
        for (int t = 0; t < T; t++) {
            const uint32_t b = (uint32_t)t & 1u, use = (uint32_t)t >> 1;
            if (ok && !mbar_wait(&sfull[b], use & 1u, 2 * tc::kWaitNs)) { atomicOr(err, 64u); ok = false; }
            tc_fence_after();
            float v[32];
            tmem_ld32(tmem + lane_off + kTmS + b * kA5Keys + 32 * half, v);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&sempty[b]);
            const int k0 = t * kA5Keys + 32 * half;
            if (k0 + 31 > qp) {   // causal mask (also past the block's last key): the diagonal tiles only
                #pragma unroll
                for (int i = 0; i < 32; i++) if (k0 + i > qp) v[i] = -INFINITY;
            }
            float mh = -INFINITY;
            #pragma unroll
            for (int i = 0; i < 32; i += 2) mh = max3f(mh, v[i], v[i + 1]);
            xm[((t & 1) * 2 + half) * 128 + m] = mh;
            named_bar(2, 256);
            const float mnew = fmaxf(mrun, fmaxf(mh, xm[((t & 1) * 2 + (half ^ 1)) * 128 + m]));   // finite: key 0 is in tile 0
            const bool need = (mnew - mrun) * c2 > kA5Rescale;   // always on tile 0 (mrun = -inf)
            float f = 1.0f;
            if (need) { f = exp2f((mrun - mnew) * c2); mrun = mnew; l *= f; }   // f = 0 on tile 0
            const float mc = mrun * c2;
            // P (unnormalised), two bf16 parts, into P buffer t & 1 once P V of tile t - 2 is complete
            if (ok && use > 0 && !mbar_wait(&pempty[b], (use - 1) & 1u, 2 * tc::kWaitNs)) { atomicOr(err, 64u); ok = false; }
            tc_fence_after();
            {
                uint32_t h[16], md[16];
                float ps = 0.f;
                #pragma unroll
                for (int j = 0; j < 16; j++) {
                    const float p0 = ex2_ftz(fmaf(v[2 * j], c2, -mc)), p1 = ex2_ftz(fmaf(v[2 * j + 1], c2, -mc));
                    ps += p0 + p1;
                    split2x2_int(p0, p1, h[j], md[j]);
                }
                l += ps;
                tmem_st16(tmem + lane_off + kTmP + 64 * b + 16 * half, h);
                tmem_st16(tmem + lane_off + kTmP + 64 * b + 32 + 16 * half, md);
            }
            // rows whose max moved: scale their O columns (this half's 64) once P V of tile t - 1 is complete
            if (t > 0 && __any_sync(0xffffffffu, need)) {
                const uint32_t pb1 = (uint32_t)(t - 1) & 1u, use1 = (uint32_t)(t - 1) >> 1;
                if (ok && !mbar_wait(&pempty[pb1], use1 & 1u, 2 * tc::kWaitNs)) { atomicOr(err, 64u); ok = false; }
                tc_fence_after();
                #pragma unroll 1
                for (int c = 64 * half; c < 64 * half + 64; c += 32) {
                    float o[32];
                    tmem_ld32(tmem + lane_off + kTmO + c, o);
                    #pragma unroll
                    for (int i = 0; i < 32; i++) o[i] *= f;
                    tmem_st32(tmem + lane_off + kTmO + c, o);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&pfull[b]);
        }
        // epilogue: O row m / l, this half's 64 dims -> the O projection's operand, split
        if (ok && !mbar_wait(ofull, 0, 2 * tc::kWaitNs)) atomicOr(err, 64u);
        tc_fence_after();
        ls[half * 128 + m] = l;
        named_bar(2, 256);
        const float inv = 1.0f / (l + ls[(half ^ 1) * 128 + m]);
        uint16_t* arow = As + (size_t)(q0 + (m & 63)) * ld_as + 128 * (2 * hk + (m >> 6));
        #pragma unroll 1
        for (int c = 64 * half; c < 64 * half + 64; c += 32) {
            float o[32];
            tmem_ld32(tmem + lane_off + kTmO + c, o);
            uint32_t h[16], md[16], lo[16];
            #pragma unroll
            for (int i = 0; i < 16; i++) split3x2(o[2 * i] * inv, o[2 * i + 1] * inv, h[i], md[i], lo[i]);
            // the parts the O projection reads, 16 bytes per store (parts Q_DIM columns apart)
            #pragma unroll
            for (int j = 0; j < 4; j++) {
                reinterpret_cast<uint4*>(arow + c)[j] = make_uint4(h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
                if (parts > 1) reinterpret_cast<uint4*>(arow + Q_DIM + c)[j] = make_uint4(md[4 * j], md[4 * j + 1], md[4 * j + 2], md[4 * j + 3]);
                if (parts > 2) reinterpret_cast<uint4*>(arow + 2 * Q_DIM + c)[j] = make_uint4(lo[4 * j], lo[4 * j + 1], lo[4 * j + 2], lo[4 * j + 3]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, 512);
}

}  // namespace pf
}  // namespace qb
