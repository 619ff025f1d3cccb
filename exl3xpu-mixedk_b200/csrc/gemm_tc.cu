// gemm_tc.cu -- LDLQ feedback-cache update on tcgen05 tensor cores, fed by TMA.
//
// Reference: quantize/quantize.py:742-744 -- after each buffer of the
// right-to-left sweep,  prod += Lfac[16lo:16cur, :]^T @ (W - hatW)[16lo:16cur, :].
// (The block LDL's trailing updates use the same kernels: linalg.cu.)
// Only rows < 16lo of prod are ever read again, so the update is
//   C[M][N] += A[M][K] . B[K][N],   M = 16 lo, N = n, K = 16 (cur - lo),
// with A = Lfac[buf rows, :M]^T and B = E[buf rows, :] -- both stored with the
// M / N index contiguous, C = prod row-major fp32.
//
// Two implementations.  The per-tile split kernel (feedback_gemm_tc_kernel,
// used without split scratch): one CTA (128 threads) owns a 128 x 128 tile of
// C and walks K in 32-deep chunks through a two-stage pipeline:
//   * TMA loads 32 x 32 fp32 boxes of A and B (128-byte swizzle) into a staging
//     buffer, while the previous chunk is being converted / multiplied.
//   * Each thread takes one M (N) row of the chunk out of staging, splits every
//     value x (times the sign sa for A) into x_hi = tf32(x) and
//     x_lo = tf32(x - x_hi), and writes both
//     into K-major operand tiles in the UMMA 128-byte-swizzle canonical layout
//     (128-byte rows of 32 k values, 8-row atoms of 1 KB).  The tf32 MMA reads
//     K-major operands only; the transpose rides on this split pass.
//   * One thread issues, per 8-deep k step, tcgen05.mma kind::tf32 for
//     A_hi.B_hi + A_hi.B_lo + A_lo.B_hi ("3xTF32"; the dropped A_lo.B_lo term is
//     ~2^-22 relative), accumulating in fp32 in tensor memory.
//   * The 128 x 128 fp32 accumulator (128 TMEM columns) is read back with
//     tcgen05.ld and added to C (the reference adds the GEMM result to prod).
// Every wait on an mbarrier is bounded; on time-out the CTA records an error,
// waits (bounded) for its outstanding copies and MMAs, frees its tensor memory
// and returns.
#include <cuda.h>
#include <string.h>

#include "exl3b_internal.h"

namespace exl3b {

constexpr int kTM = 128, kTN = 128, kTK = 32;
constexpr int kBox = 32 * 32 * 4;                 // one 32x32 fp32 box: 4 KB
constexpr int kOpBytes = 128 * kTK * 4;           // one 128 x 32 operand tile: 16 KB
constexpr int kStageBytes = 8 * kBox;             // staging: 4 boxes of A, 4 of B
constexpr int kOpSetBytes = 4 * kOpBytes;         // A_hi | A_lo | B_hi | B_lo
// shared memory (1024-aligned): staging[2] | operands[2] | barriers
constexpr int kGemmSmem = 2 * kStageBytes + 2 * kOpSetBytes + 64 + 1024;
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at <= 2 GHz

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// Wait for an mbarrier phase, bounded by ~2 s of SM clock.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok) : "r"(bar), "r"(parity), "r"(20000u) : "memory");
        if (ok) return true;
        if (clock64() - t0 > kWaitCycles) return false;
    }
}

// UMMA shared-memory descriptor, K-major, 128-byte swizzle (sm100 version 1).
// Rows of 128 bytes, 8-row atoms 1 KB apart (SBO); LBO is unused for this
// layout.  A k step inside the atom advances the start address by 32 bytes.
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)(16 >> 4) << 16;               // LBO (ignored)
    d |= (uint64_t)(1024 >> 4) << 32;             // SBO: next 8-row atom
    d |= (uint64_t)1 << 46;                       // descriptor version (Blackwell)
    d |= (uint64_t)2 << 61;                       // SWIZZLE_128B
    return d;
}

// instruction descriptor: D f32, A/B tf32, both K-major, M = 128, N = 128
constexpr uint32_t kIdesc = (1u << 4)             // c_format F32
                          | (2u << 7)             // a_format TF32
                          | (2u << 10)            // b_format TF32
                          | ((uint32_t)(kTN >> 3) << 17)
                          | ((uint32_t)(kTM >> 4) << 24);

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(tmem_d), "l"(da), "l"(db), "r"(kIdesc), "r"(accumulate) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x,
                                            int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        :: "r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar) : "memory");
}

__device__ __forceinline__ float tf32_round(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Row r (an M or N index inside the tile) of one staged operand chunk -> the
// K-major swizzled hi / lo operand tiles.  Staging holds four TMA boxes side by
// side, box c = rows 32c..32c+31, each box 32 k-rows of 128 bytes with the
// 16-byte chunk index XOR-ed by (k mod 8).  Reads are one 128-byte staging row
// per warp (conflict-free); writes are 16-byte chunks whose swizzle spreads 8
// consecutive rows over all 32 banks.
__device__ __forceinline__ void split_row(const float* __restrict__ stg, float* __restrict__ hi,
                                          float* __restrict__ lo, int r, float sign) {
    const float* box = stg + (r >> 5) * (kBox / 4);
    const int ml = r & 31;
#pragma unroll
    for (int j = 0; j < kTK / 4; ++j) {
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int k = 4 * j + e;
            v[e] = sign * box[k * 32 + ((((ml >> 2) ^ (k & 7))) << 2) + (ml & 3)];
        }
        float4 h, l;
        h.x = tf32_round(v[0]); l.x = tf32_round(v[0] - h.x);
        h.y = tf32_round(v[1]); l.y = tf32_round(v[1] - h.y);
        h.z = tf32_round(v[2]); l.z = tf32_round(v[2] - h.z);
        h.w = tf32_round(v[3]); l.w = tf32_round(v[3] - h.w);
        const int off = r * kTK + ((j ^ (r & 7)) << 2);
        *reinterpret_cast<float4*>(hi + off) = h;
        *reinterpret_cast<float4*>(lo + off) = l;
    }
}

__global__ void __launch_bounds__(128, 1)
feedback_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB,
                        float* __restrict__ C, int ldc, int M, int N, int K,
                        float sa, int lower, int* __restrict__ err) {
    extern __shared__ __align__(1024) uint8_t gsm_raw[];
    // 1024-byte alignment for the swizzle atoms
    uint8_t* gsm = (uint8_t*)(((uintptr_t)gsm_raw + 1023) & ~(uintptr_t)1023);
    uint8_t* stage = gsm;                                   // 2 x 32 KB
    uint8_t* ops = gsm + 2 * kStageBytes;                   // 2 x 64 KB
    uint64_t* bars = reinterpret_cast<uint64_t*>(ops + 2 * kOpSetBytes);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 4);

    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int m0 = blockIdx.y * kTM, n0 = blockIdx.x * kTN;
    // lower: only tiles that reach the lower triangle (C symmetric update)
    if (lower && n0 > m0 + kTM - 1) return;
    // bars[0..1]: staging s filled (TMA); bars[2..3]: MMAs reading operand set s done
    const uint32_t bar_full0 = smem_u32(&bars[0]);
    const uint32_t bar_mma0 = smem_u32(&bars[2]);
    const int nchunks = (K + kTK - 1) / kTK;

    auto issue_loads = [&](int kc) {
        const int s = kc & 1;
        const uint32_t bar = bar_full0 + 8 * s;
        const uint32_t dst = smem_u32(stage + s * kStageBytes);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                     :: "r"(bar), "r"(kStageBytes) : "memory");
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            tma_load_2d(dst + c * kBox, &tmA, m0 + 32 * c, kc * kTK, bar);
            tma_load_2d(dst + 4 * kBox + c * kBox, &tmB, n0 + 32 * c, kc * kTK, bar);
        }
    };

    if (t == 0) {
        for (int i = 0; i < 4; ++i)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(smem_u32(&bars[i])) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        issue_loads(0);
        if (nchunks > 1) issue_loads(1);
    }
    __syncwarp();
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(kTN) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    // counts of loads issued / consumed and MMA commits issued / waited for
    int loads_issued = nchunks > 1 ? 2 : 1, loads_done = 0;
    int commits = 0, commits_done = 0;
    bool fail = false;
    for (int kc = 0; kc < nchunks; ++kc) {
        const int s = kc & 1;
        bool ok = mbar_wait(bar_full0 + 8 * s, (kc >> 1) & 1);
        // the operand set s was last read by the MMAs of chunk kc - 2
        if (ok && kc >= 2) ok = mbar_wait(bar_mma0 + 8 * s, ((kc - 2) >> 1) & 1);
        if (__syncthreads_or(!ok)) { fail = true; break; }
        loads_done = kc + 1;
        if (kc >= 2) commits_done = kc - 1;
        const float* stg = reinterpret_cast<const float*>(stage + s * kStageBytes);
        float* opset = reinterpret_cast<float*>(ops + s * kOpSetBytes);
        split_row(stg, opset, opset + kOpBytes / 4, t, sa);                     // A rows
        split_row(stg + kStageBytes / 8, opset + kOpBytes / 2, opset + 3 * kOpBytes / 4, t,
                  1.0f);                                                         // B rows
        // generic-proxy shared writes (and the staging reads) before the async
        // proxy (tensor core reads, next TMA write) touches the same memory
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (t == 0) {
            if (kc + 2 < nchunks) issue_loads(kc + 2);
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t aH = smem_u32(opset), aL = aH + kOpBytes;
            const uint32_t bH = aH + 2 * kOpBytes, bL = aH + 3 * kOpBytes;
#pragma unroll
            for (int kk = 0; kk < kTK / 8; ++kk) {
                const uint32_t off = kk * 32;        // 8 tf32 values = 32 bytes of the row
                const uint64_t dAh = umma_desc_k_sw128(aH + off);
                const uint64_t dAl = umma_desc_k_sw128(aL + off);
                const uint64_t dBh = umma_desc_k_sw128(bH + off);
                const uint64_t dBl = umma_desc_k_sw128(bL + off);
                umma_tf32(tmem, dAl, dBh, (kc > 0 || kk > 0) ? 1u : 0u);
                umma_tf32(tmem, dAh, dBl, 1u);
                umma_tf32(tmem, dAh, dBh, 1u);
            }
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         :: "r"(bar_mma0 + 8 * s) : "memory");
        }
        commits = kc + 1;
        if (kc + 2 < nchunks) loads_issued = kc + 3;
    }
    if (!fail) {
        // tcgen05.commit tracks every earlier MMA of this thread: the last
        // commit covers them all
        const int kl = nchunks - 1;
        const bool ok = mbar_wait(bar_mma0 + 8 * (kl & 1), (kl >> 1) & 1);
        if (__syncthreads_or(!ok)) fail = true;
        else commits_done = commits;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!fail) {
        // epilogue: warp w holds accumulator rows 32w..32w+31 (TMEM lanes)
        const int row = m0 + 32 * warp + lane;
        const bool vec = ((ldc & 3) == 0) && ((((uintptr_t)C) & 15) == 0);
#pragma unroll 1
        for (int cc = 0; cc < kTN / 32; ++cc) {
            uint32_t r[32];
            const uint32_t taddr = tmem + ((uint32_t)(32 * warp) << 16) + 32 * cc;
            asm volatile(
                "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
                "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
                "[%32];"
                : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                  "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                  "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
                  "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                  "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]),
                  "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                : "r"(taddr));
            asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
            if (row < M) {
                float* crow = C + (size_t)row * ldc + n0 + 32 * cc;
                const int lim = N - (n0 + 32 * cc);
                if (vec && lim >= 32) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float4 c4 = *reinterpret_cast<float4*>(crow + j);
                        c4.x += __uint_as_float(r[j]);
                        c4.y += __uint_as_float(r[j + 1]);
                        c4.z += __uint_as_float(r[j + 2]);
                        c4.w += __uint_as_float(r[j + 3]);
                        *reinterpret_cast<float4*>(crow + j) = c4;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < lim) crow[j] = crow[j] + __uint_as_float(r[j]);
                }
            }
        }
    } else if (t == 0) {
        atomicCAS(err, 0, 4);
        // let every copy and MMA still in flight land before the memory is freed
        for (int i = loads_done; i < loads_issued; ++i) mbar_wait(bar_full0 + 8 * (i & 1), (i >> 1) & 1);
        for (int i = commits_done; i < commits; ++i) mbar_wait(bar_mma0 + 8 * (i & 1), (i >> 1) & 1);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     :: "r"(tmem), "r"(kTN) : "memory");
}

// ------------------------------------------------- pre-split operand path
// For updates with many output tiles the hi/lo split is done once per operand
// instead of once per output tile: tf32_split_kernel writes X (stored [K][R],
// R contiguous, row pitch ld) as hi / lo arrays [R][kp] (K contiguous, kp =
// K rounded up to 32, zero padded), each value x (times `sign`) as
// hi = tf32(x), lo = tf32(x - hi) -- the same split as split_row.  Then
// gemm_tf32x3_kernel: persistent, warp-specialised 3xTF32 GEMM over pre-split
// operands.  One CTA per SM walks the 128 x BN tiles of C (row-major tile
// order, CTA b takes tiles b, b + grid, ...):
//   * warp 0 (one thread) streams 128 x 32 / BN x 32 boxes of the four arrays with TMA
//     (128-byte swizzle: the boxes land in the UMMA K-major canonical layout
//     as they are) through a kStages ring of full / empty mbarriers;
//   * warp 1 (one thread) issues the MMAs (lo.hi, hi.lo, hi.hi per 8-deep k
//     step, as above) into one of two BN-column TMEM accumulators, tile by
//     tile in turn, and commits each stage back to the loader and each
//     finished tile to the epilogue;
//   * warps 2-5 (warp w reads TMEM lanes 32 (w mod 4) ..) run the epilogue,
//     C += sa * acc (sa = +-1: exact, and the same bits as splitting sa * A),
//     and hand the accumulator back -- so tile i's read-modify-write of C
//     overlaps tile i+1's MMAs, and the TMEM allocation and pipeline fill are
//     paid once per SM instead of once per tile.
// Every wait is bounded; on a time-out the CTA records the error, stops
// issuing, waits (bounded) for its outstanding copies and MMAs, frees its
// tensor memory and returns.
// Tile width BN: 128 x 256 tiles (general updates) stream a quarter fewer
// operand bytes per FLOP than 128 x 128 (the kernel is bound by the hi and lo
// boxes it reads out of L2, about 10 TB/s at 128 x 128): two 96 KB stages and
// two 256-column accumulators (all 512 TMEM columns).  128 x 128 tiles (three
// 64 KB stages) stay for the lower-triangle updates, whose narrow trailing
// blocks give too few wide tiles and whose wide tiles waste more work above
// the diagonal.
constexpr int kSplitK = 512;                        // K per pre-split piece
constexpr int kOpBox = 128 * kTK * 4;               // one 128 x 32 tf32 tile: 16 KB

template <int BN>
struct GemmCfg {
    static constexpr int kStages = BN == 256 ? 2 : 3;
    static constexpr int kBBox = BN * kTK * 4;                 // one BN x 32 tf32 box
    static constexpr int kStage = 2 * kOpBox + 2 * kBBox;      // Ah | Al | Bh | Bl
    static constexpr int kSmem = kStages * kStage + 128 + 1024;   // ring | barriers | align
    // instruction descriptor: D f32, A/B tf32, both K-major, M = 128, N = BN
    static constexpr uint32_t kIdesc = (1u << 4) | (2u << 7) | (2u << 10)
                                     | ((uint32_t)(BN >> 3) << 17)
                                     | ((uint32_t)(kTM >> 4) << 24);
    static_assert(kSmem <= 227 * 1024, "shared memory of one CTA");
    static_assert(2 * BN <= 512, "two accumulators in the TMEM of one SM");
};

template <int BN>
__device__ __forceinline__ void umma_tf32_n(uint32_t tmem_d, uint64_t da, uint64_t db,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(tmem_d), "l"(da), "l"(db), "r"(GemmCfg<BN>::kIdesc), "r"(accumulate)
        : "memory");
}

__global__ void __launch_bounds__(256)
tf32_split_kernel(const float* __restrict__ X, int ld, int K, int R, float sign,
                  float* __restrict__ hi, float* __restrict__ lo, int kp) {
    __shared__ float tile[32][33];
    const int r0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8
    for (int i = ty; i < 32; i += 8) {
        const int k = k0 + i, r = r0 + tx;
        tile[i][tx] = (k < K && r < R) ? sign * X[(size_t)k * ld + r] : 0.0f;
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int r = r0 + i, k = k0 + tx;
        if (r < R && k < kp) {
            const float v = tile[tx][i];
            const float h = tf32_round(v);
            hi[(size_t)r * kp + k] = h;
            lo[(size_t)r * kp + k] = tf32_round(v - h);
        }
    }
}

constexpr int kGemmThreads = 192;                   // loader, MMA, 4 epilogue warps

// 128 x BN tile t of the row-major tile grid (tn tiles per row); false when
// `lower` skips it (entirely above the diagonal)
__device__ __forceinline__ bool gemm_tile(int t, int tn, int bn, int lower, int& m0, int& n0) {
    m0 = (t / tn) * kTM;
    n0 = (t % tn) * bn;
    return !(lower && n0 > m0 + kTM - 1);
}

template <int BN>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap tmAh,
                   const __grid_constant__ CUtensorMap tmAl,
                   const __grid_constant__ CUtensorMap tmBh,
                   const __grid_constant__ CUtensorMap tmBl,
                   float* __restrict__ C, int ldc, int M, int N, int kp, float sa,
                   int lower, int* __restrict__ err) {
    using Cfg = GemmCfg<BN>;
    constexpr int kStages = Cfg::kStages, kStage2 = Cfg::kStage, kBBox = Cfg::kBBox;
    extern __shared__ __align__(1024) uint8_t gsm_raw[];
    uint8_t* gsm = (uint8_t*)(((uintptr_t)gsm_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(gsm + kStages * kStage2);
    // bars[0..S): stage full (TMA);  bars[S..2S): stage empty (MMA commit);
    // bars[2S], [2S+1]: accumulator a full (MMA commit);  bars[2S+2], [2S+3]:
    // accumulator a empty (128 epilogue arrivals);  bars[2S+4]: all MMAs done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);
    __shared__ int fail_s;
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int tm = (M + kTM - 1) / kTM, tn = (N + BN - 1) / BN;
    const int ntiles = tm * tn;
    const uint32_t full0 = smem_u32(&bars[0]);
    const uint32_t empty0 = smem_u32(&bars[kStages]);
    const uint32_t afull0 = smem_u32(&bars[2 * kStages]);
    const uint32_t aempty0 = smem_u32(&bars[2 * kStages + 2]);
    const uint32_t done = smem_u32(&bars[2 * kStages + 4]);
    const int nchunks = kp / kTK;
    if (t == 0) {
        for (int i = 0; i < 2 * kStages + 5; ++i) {
            const uint32_t cnt = (i == 2 * kStages + 2 || i == 2 * kStages + 3) ? 128u : 1u;
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;"
                         :: "r"(smem_u32(&bars[i])), "r"(cnt) : "memory");
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fail_s = 0;
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     :: "r"(smem_u32(tmem_slot)), "r"(2 * BN) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_slot;

    if (t == 0) {
        // loader: global chunk it into stage it % S once the MMAs of chunk it - S
        // have read it
        int it = 0, issued = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            int m0, n0;
            if (!gemm_tile(tile, tn, BN, lower, m0, n0)) continue;
            for (int kc = 0; kc < nchunks; ++kc, ++it) {
                const int s = it % kStages, r = it / kStages;
                if (r > 0) ok = mbar_wait(empty0 + 8 * s, (r - 1) & 1);
                if (!ok || *(volatile int*)&fail_s) { ok = false; break; }
                const uint32_t bar = full0 + 8 * s;
                const uint32_t dst = smem_u32(gsm + s * kStage2);
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                             :: "r"(bar), "r"(kStage2) : "memory");
                tma_load_2d(dst, &tmAh, kc * kTK, m0, bar);
                tma_load_2d(dst + kOpBox, &tmAl, kc * kTK, m0, bar);
                tma_load_2d(dst + 2 * kOpBox, &tmBh, kc * kTK, n0, bar);
                tma_load_2d(dst + 2 * kOpBox + kBBox, &tmBl, kc * kTK, n0, bar);
                issued = it + 1;
            }
        }
        if (!ok) {
            atomicExch(&fail_s, 1);
            // every issued load lands before the shared memory is released
            for (int i = 0; i < issued; ++i)
                mbar_wait(full0 + 8 * (i % kStages), (i / kStages) & 1);
        }
    } else if (t == 32) {
        // MMA issuer: tile lt of this CTA into accumulator lt & 1
        int it = 0, lt = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
            int m0, n0;
            if (!gemm_tile(tile, tn, BN, lower, m0, n0)) continue;
            const int a = lt & 1, u = lt >> 1;
            if (u > 0) ok = mbar_wait(aempty0 + 8 * a, (u - 1) & 1);
            if (!ok || *(volatile int*)&fail_s) { ok = false; break; }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t acc = tmem + (uint32_t)(a * BN);
            for (int kc = 0; kc < nchunks; ++kc, ++it) {
                const int s = it % kStages, r = it / kStages;
                ok = mbar_wait(full0 + 8 * s, r & 1);
                if (!ok || *(volatile int*)&fail_s) { ok = false; break; }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t aH = smem_u32(gsm + s * kStage2), aL = aH + kOpBox;
                const uint32_t bH = aH + 2 * kOpBox, bL = bH + kBBox;
#pragma unroll
                for (int kk = 0; kk < kTK / 8; ++kk) {
                    const uint32_t off = kk * 32;
                    umma_tf32_n<BN>(acc, umma_desc_k_sw128(aL + off), umma_desc_k_sw128(bH + off),
                                (kc > 0 || kk > 0) ? 1u : 0u);
                    umma_tf32_n<BN>(acc, umma_desc_k_sw128(aH + off), umma_desc_k_sw128(bL + off), 1u);
                    umma_tf32_n<BN>(acc, umma_desc_k_sw128(aH + off), umma_desc_k_sw128(bH + off), 1u);
                }
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                             :: "r"(empty0 + 8 * s) : "memory");
            }
            if (!ok) break;
            asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                         :: "r"(afull0 + 8 * a) : "memory");
            ++lt;
        }
        if (!ok) atomicExch(&fail_s, 1);
        // the last commit tracks every earlier MMA of this thread
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                     :: "r"(done) : "memory");
    } else if (warp >= 2) {
        // epilogue: TMEM lanes 32 (warp mod 4) .. + 31 = rows of the tile
        const int q = warp & 3;
        const bool vec = ((ldc & 3) == 0) && ((((uintptr_t)C) & 15) == 0);
        int lt = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
            int m0, n0;
            if (!gemm_tile(tile, tn, BN, lower, m0, n0)) continue;
            const int a = lt & 1, u = lt >> 1;
            bool ok = mbar_wait(afull0 + 8 * a, u & 1);
            // one decision per warp: the TMEM loads below are warp-collective
            ok = __all_sync(0xffffffffu, ok && !*(volatile int*)&fail_s);
            if (!ok) {
                if (lane == 0) atomicExch(&fail_s, 1);
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int row = m0 + 32 * q + lane;
#pragma unroll 1
            for (int cc = 0; cc < BN / 32; ++cc) {
                uint32_t r[32];
                const uint32_t taddr = tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(a * BN + 32 * cc);
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
                    "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
                    "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
                    "[%32];"
                    : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                      "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                      "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
                      "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                      "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]),
                      "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                if (cc == BN / 32 - 1) {
                    // the accumulator is read out: hand it back to the MMA issuer
                    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];"
                                 :: "r"(aempty0 + 8 * a) : "memory");
                }
                if (row < M) {
                    float* crow = C + (size_t)row * ldc + n0 + 32 * cc;
                    const int lim = N - (n0 + 32 * cc);
                    if (vec && lim >= 32) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            float4 c4 = *reinterpret_cast<float4*>(crow + j);
                            c4.x += sa * __uint_as_float(r[j]);
                            c4.y += sa * __uint_as_float(r[j + 1]);
                            c4.z += sa * __uint_as_float(r[j + 2]);
                            c4.w += sa * __uint_as_float(r[j + 3]);
                            *reinterpret_cast<float4*>(crow + j) = c4;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < lim) crow[j] = crow[j] + sa * __uint_as_float(r[j]);
                    }
                }
            }
            ++lt;
        }
    }
    // everyone: all MMAs complete (or abandoned)
    const bool ok = mbar_wait(done, 0);
    if (__syncthreads_or(!ok || fail_s)) {
        if (t == 0) atomicCAS(err, 0, 4);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     :: "r"(tmem), "r"(2 * BN) : "memory");
}

// ---------------------------------------------------------------- host side
// cuTensorMapEncodeTiled is a driver-API entry point; it is resolved at run
// time through the runtime (no link dependency on libcuda, so the library also
// loads on machines without a GPU driver).
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

static int encode_operand(CUtensorMap* map, const float* base, int inner, int outer,
                           int ld) {
    cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
    cuuint32_t box[2] = {32, 32};
    cuuint32_t estr[2] = {1, 1};
    EncodeTiledFn enc = encode_fn();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return RC_DEVICE_ERROR;
    }
    const CUresult r = enc(
        map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
        CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return RC_DEVICE_ERROR;
    }
    return RC_OK;
}

static int encode_split(CUtensorMap* map, const float* base, int kp, int rows,
                        int box_rows = 128) {
    cuuint64_t dims[2] = {(cuuint64_t)kp, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)kp * 4};
    cuuint32_t box[2] = {(cuuint32_t)kTK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    EncodeTiledFn enc = encode_fn();
    if (!enc) {
        set_error("cuTensorMapEncodeTiled unavailable from the driver");
        return RC_DEVICE_ERROR;
    }
    const CUresult r = enc(
        map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_error("cuTensorMapEncodeTiled failed (%d)", (int)r);
        return RC_DEVICE_ERROR;
    }
    return RC_OK;
}

static int kp_of(int K) {
    const int k = K < kSplitK ? K : kSplitK;
    return (k + kTK - 1) / kTK * kTK;
}

size_t gemm_split_bytes(int M, int N, int K) {
    return ((size_t)M + (size_t)N) * kp_of(K) * 8 + 1024;
}

int gemm_split(const float* X, int ld, int K, int R, float* hi, float* lo, int kp,
               cudaStream_t stream) {
    dim3 g((R + 31) / 32, kp / 32);
    tf32_split_kernel<<<g, 256, 0, stream>>>(X, ld, K, R, 1.0f, hi, lo, kp);
    note_launch();
    return check_cuda(cudaGetLastError(), "tf32_split launch") ? RC_DEVICE_ERROR : RC_OK;
}

template <int BN>
static int presplit_launch(int M, int N, int kp, const float* Ah, const float* Al,
                           const float* Bh, const float* Bl, float* C, int ldc, float sa,
                           int lower, int* err, cudaStream_t stream) {
    using Cfg = GemmCfg<BN>;
    static bool attr[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev]) {
        if (check_cuda(cudaFuncSetAttribute(gemm_tf32x3_kernel<BN>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            Cfg::kSmem),
                       "cudaFuncSetAttribute(gemm_tf32x3)"))
            return RC_DEVICE_ERROR;
        attr[dev] = true;
    }
    CUtensorMap tAh, tAl, tBh, tBl;
    int rc = encode_split(&tAh, Ah, kp, M);
    if (!rc) rc = encode_split(&tAl, Al, kp, M);
    if (!rc) rc = encode_split(&tBh, Bh, kp, N, BN);
    if (!rc) rc = encode_split(&tBl, Bl, kp, N, BN);
    if (rc) return rc;
    const int tiles = ((N + BN - 1) / BN) * ((M + kTM - 1) / kTM);
    const int sms = device_sms();
    const unsigned grid = (unsigned)(tiles < sms ? tiles : sms);     // persistent CTAs
    gemm_tf32x3_kernel<BN><<<grid, kGemmThreads, Cfg::kSmem, stream>>>(
        tAh, tAl, tBh, tBl, C, ldc, M, N, kp, sa, lower, err);
    note_launch();
    return check_cuda(cudaGetLastError(), "gemm_tf32x3 launch") ? RC_DEVICE_ERROR : RC_OK;
}

int gemm_presplit_run(int M, int N, int kp, const float* Ah, const float* Al, const float* Bh,
                      const float* Bl, float* C, int ldc, float sa, int lower, int* err,
                      cudaStream_t stream) {
    if (M <= 0 || N <= 0) return RC_OK;
    return lower ? presplit_launch<128>(M, N, kp, Ah, Al, Bh, Bl, C, ldc, sa, lower, err, stream)
                 : presplit_launch<256>(M, N, kp, Ah, Al, Bh, Bl, C, ldc, sa, lower, err, stream);
}

// C[M][N] += sa * A_T^T . B on tcgen05 (A_T [K][M], B [K][N], both row-major
// with leading dimensions lda / ldb; all pointers 16-byte aligned, lda / ldb
// multiples of 4; sa = +-1, applied exactly).  lower: skip the 128 x 128 tiles
// entirely above the diagonal (symmetric updates that only need C's lower
// triangle).  err: device word set to 4 on a barrier time-out.  split_ws (>=
// gemm_split_bytes(M, N, K) bytes): the pre-split operand path; without it
// the per-tile split kernel above.
int launch_gemm_tn_acc_tc(int M, int N, int K, const float* A_T, int lda, const float* B,
                          int ldb, float* C, int ldc, int* err, cudaStream_t stream,
                          float sa, int lower, void* split_ws, size_t split_bytes) {
    if (M <= 0 || N <= 0 || K <= 0) return RC_OK;
    if (((uintptr_t)A_T & 15) || ((uintptr_t)B & 15) || (lda & 3) || (ldb & 3)) {
        set_error("tcgen05 GEMM operands must be 16-byte aligned");
        return RC_BAD_REQUEST;
    }
    if (split_ws != nullptr && split_bytes >= gemm_split_bytes(M, N, K)) {
        // pre-split path, K in pieces of kSplitK
        // B the first N rows of A (the same matrix): B's split is A's first rows
        const bool same = A_T == B && lda == ldb && N <= M;
        float* base = reinterpret_cast<float*>(((uintptr_t)split_ws + 1023) & ~(uintptr_t)1023);
        for (int k0 = 0; k0 < K; k0 += kSplitK) {
            const int kk = (K - k0) < kSplitK ? (K - k0) : kSplitK;
            const int kp = (kk + kTK - 1) / kTK * kTK;
            float* Ah = base;
            float* Al = Ah + (size_t)M * kp;
            float* Bh = same ? Ah : Al + (size_t)M * kp;
            float* Bl = same ? Al : Bh + (size_t)N * kp;
            int rc = gemm_split(A_T + (size_t)k0 * lda, lda, kk, M, Ah, Al, kp, stream);
            if (!rc && !same) rc = gemm_split(B + (size_t)k0 * ldb, ldb, kk, N, Bh, Bl, kp, stream);
            if (!rc) rc = gemm_presplit_run(M, N, kp, Ah, Al, Bh, Bl, C, ldc, sa, lower, err, stream);
            if (rc) return rc;
        }
        return RC_OK;
    }
    CUtensorMap tmA, tmB;
    int rc = encode_operand(&tmA, A_T, M, K, lda);
    if (!rc) rc = encode_operand(&tmB, B, N, K, ldb);
    if (rc) return rc;
    static bool attr[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev]) {
        if (check_cuda(cudaFuncSetAttribute(feedback_gemm_tc_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            kGemmSmem),
                       "cudaFuncSetAttribute(feedback_gemm_tc)"))
            return RC_DEVICE_ERROR;
        attr[dev] = true;
    }
    dim3 grid((N + kTN - 1) / kTN, (M + kTM - 1) / kTM);
    feedback_gemm_tc_kernel<<<grid, 128, kGemmSmem, stream>>>(tmA, tmB, C, ldc, M, N, K, sa,
                                                                lower, err);
    note_launch();
    return check_cuda(cudaGetLastError(), "feedback_gemm_tc launch") ? RC_DEVICE_ERROR : RC_OK;
}

}  // namespace exl3b
