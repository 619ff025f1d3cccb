// linalg.cu -- Hessian factorisation for BlockLDLQ (fp32 with tensor-core
// updates, fp64 on CUDA cores).
//
// Reference: quantize/quantize.py:419-437 block_LDL (Cholesky, 16x16 diagonal
// block inverses, L <- L . blockdiag(DL^-1), identity diagonal blocks) with
// the fp32 path of quantize_linear (:816) and the fp64 paths of its fallback
// (:817-835) and of quantize()'s U -> G conversion (:944-950).
//
// Cholesky: blocked right-looking, 64-column steps: (1) one CTA factors the
// 64x64 diagonal block in shared memory and records a LAPACK-style info
// (1-based column of the first non-positive / non-finite pivot) in a device
// status word; (2) rows below solve against it; (3) the trailing lower
// triangle is updated -- fp32: on tcgen05 tensor cores (gemm_tc.cu) in two
// levels of blocking with a lookahead stream (cholesky_lower); fp64: SIMT
// GEMM.  Later launches skip work once the status is set; the host reads the
// status once at the end.
#include "exl3b_internal.h"

namespace exl3b {

constexpr int kNB = 64;   // Cholesky panel

// ------------------------------------------------------------------ GEMM
// C = alpha * A.B + beta * C.  A logical [M][K]: A_KMAJ -> A[m*lda + k],
// else A[k*lda + m].  B logical [K][N]: B_KMAJ -> B[n*ldb + k], else
// B[k*ldb + n].  LOWER: skip output tiles strictly above the diagonal.
template <typename T, bool A_KMAJ, bool B_KMAJ, bool LOWER, int BM, int BN, int TM, int TN>
__global__ void __launch_bounds__((BM / TM) * (BN / TN))
gemm_kernel(int M, int N, int K, const T* __restrict__ A, int lda,
            const T* __restrict__ B, int ldb, T* __restrict__ C, int ldc,
            T alpha, T beta, const int* __restrict__ status) {
    constexpr int BK = 16;
    constexpr int NT = (BM / TM) * (BN / TN);
    __shared__ T As[BK][BM + 4];
    __shared__ T Bs[BK][BN + 4];
    if (status && *status) return;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    if (LOWER && m0 + BM <= n0) return;
    const int t = threadIdx.x;
    const int tm = (t / (BN / TN)) * TM, tn = (t % (BN / TN)) * TN;
    T acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = T(0);
    for (int k0 = 0; k0 < K; k0 += BK) {
        for (int idx = t; idx < BK * BM; idx += NT) {
            int kk, mm;
            if (A_KMAJ) { mm = idx / BK; kk = idx % BK; } else { kk = idx / BM; mm = idx % BM; }
            const int gm = m0 + mm, gk = k0 + kk;
            T v = T(0);
            if (gm < M && gk < K) v = A_KMAJ ? A[(size_t)gm * lda + gk] : A[(size_t)gk * lda + gm];
            As[kk][mm] = v;
        }
        for (int idx = t; idx < BK * BN; idx += NT) {
            int kk, nn;
            if (B_KMAJ) { nn = idx / BK; kk = idx % BK; } else { kk = idx / BN; nn = idx % BN; }
            const int gn = n0 + nn, gk = k0 + kk;
            T v = T(0);
            if (gn < N && gk < K) v = B_KMAJ ? B[(size_t)gn * ldb + gk] : B[(size_t)gk * ldb + gn];
            Bs[kk][nn] = v;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            T a[TM], b[TN];
#pragma unroll
            for (int i = 0; i < TM; ++i) a[i] = As[kk][tm + i];
#pragma unroll
            for (int j = 0; j < TN; ++j) b[j] = Bs[kk][tn + j];
#pragma unroll
            for (int i = 0; i < TM; ++i)
#pragma unroll
                for (int j = 0; j < TN; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
        const int gm = m0 + tm + i;
        if (gm >= M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
            const int gn = n0 + tn + j;
            if (gn >= N || (LOWER && gn > gm)) continue;
            T* c = &C[(size_t)gm * ldc + gn];
            *c = (beta == T(0)) ? alpha * acc[i][j] : fma(alpha, acc[i][j], beta * *c);
        }
    }
}

template <typename T, bool A_KMAJ, bool B_KMAJ, bool LOWER>
static int gemm_launch(int M, int N, int K, const T* A, int lda, const T* B, int ldb,
                       T* C, int ldc, T alpha, T beta, const int* status,
                       cudaStream_t stream) {
    if (M <= 0 || N <= 0) return RC_OK;
    constexpr int BM = sizeof(T) == 4 ? 128 : 64;
    constexpr int BN = BM;
    constexpr int TM = sizeof(T) == 4 ? 8 : 4;
    constexpr int TN = TM;
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    gemm_kernel<T, A_KMAJ, B_KMAJ, LOWER, BM, BN, TM, TN>
        <<<grid, (BM / TM) * (BN / TN), 0, stream>>>(M, N, K, A, lda, B, ldb, C, ldc,
                                                    alpha, beta, status);
    note_launch();
    return check_cuda(cudaGetLastError(), "gemm launch") ? RC_DEVICE_ERROR : RC_OK;
}

// C[M][N] += A_T^T . B with A_T [K][M] (M contiguous), B [K][N] (N contiguous):
// the LDLQ feedback-cache update prod += Lfac[buf, :M]^T . E[buf, :].
int launch_gemm_tn_acc_f32(int M, int N, int K, const float* A_T, int lda,
                           const float* B, int ldb, float* C, int ldc, cudaStream_t stream) {
    return gemm_launch<float, false, false, false>(M, N, K, A_T, lda, B, ldb, C, ldc,
                                                   1.0f, 1.0f, nullptr, stream);
}

// ------------------------------------------------------------------ Cholesky
template <typename T>
__device__ __forceinline__ T dsqrt(T v);
template <> __device__ __forceinline__ float dsqrt<float>(float v) { return sqrtf(v); }
template <> __device__ __forceinline__ double dsqrt<double>(double v) { return sqrt(v); }

// Factor the kNB x kNB diagonal block at (j0, j0) in place (lower).  1024
// threads as 32 x 32; every thread derives the pivot's square root from
// shared memory itself (the same value everywhere), so a column costs two
// barriers: scale the column, then the rank-1 update of the trailing lower
// triangle, 2-D strided without integer division.  (The fp64 and fp32-SIMT
// path; the fp32 tensor-core path uses potrf_inv_kernel.)
template <typename T>
__global__ void __launch_bounds__(1024)
potrf_diag_kernel(T* __restrict__ A, int n, int j0, int nb, int* __restrict__ status) {
    __shared__ T S[kNB][kNB + 1];
    if (*status) return;
    const int t = threadIdx.x;
    const int tx = t & 31, ty = t >> 5;
    for (int r = ty; r < nb; r += 32)
        for (int c = tx; c < nb; c += 32) S[r][c] = A[(size_t)(j0 + r) * n + (j0 + c)];
    __syncthreads();
    int bad = 0;
    for (int j = 0; j < nb; ++j) {
        const T d = S[j][j];
        if (!(d > T(0)) || !isfinite((double)d)) { bad = j0 + j + 1; break; }
        const T djj = dsqrt<T>(d);
        if (t < nb - j - 1) S[j + 1 + t][j] = S[j + 1 + t][j] / djj;
        __syncthreads();
        if (t == 0) S[j][j] = djj;
        for (int i = j + 1 + ty; i < nb; i += 32) {
            const T lij = S[i][j];
            for (int c = j + 1 + tx; c <= i; c += 32) S[i][c] = S[i][c] - lij * S[c][j];
        }
        __syncthreads();
    }
    if (bad) {
        if (t == 0) *status = bad;
        return;
    }
    for (int r = ty; r < nb; r += 32)
        for (int c = tx; c <= r; c += 32) A[(size_t)(j0 + r) * n + (j0 + c)] = S[r][c];
}


// fp32, tensor-core path: factor the nb x nb diagonal block at (j0, j0) (nb a
// multiple of 16, <= kNB) in place and write its inverse (lower triangular,
// zero above the diagonal and outside nb x nb) to Linv [kNB][kNB].  Blocked by
// 16 so that the serial work is warp-local: for each 16-column block K,
//   (1) warp 0 factors the 16 x 16 diagonal block in registers (lane l holds
//       row l; each column's values are broadcast with shuffles) and inverts
//       it (lane c forward-substitutes column c in registers, multiplying by
//       the diagonal's reciprocals);
//   (2) the CTA solves the rows below against it: S[r, K] <- S[r, K] inv^T;
//   (3) the CTA applies the rank-16 update to the trailing lower triangle.
// Then the off-diagonal blocks of the inverse, row block by row block:
//   V[I][J] = -inv(L_II) . sum_{K=J}^{I-1} L[I][K] V[K][J].
// Records a LAPACK-style info (1-based column of the first non-positive /
// non-finite pivot) in *status, like potrf_diag_kernel.  512 threads.
__global__ void __launch_bounds__(512)
potrf_inv_kernel(float* __restrict__ A, int n, int j0, int nb, int* __restrict__ status,
                 float* __restrict__ Linv) {
    __shared__ float S[kNB][kNB + 1];     // the block; becomes L (lower)
    __shared__ float V[kNB][kNB + 1];     // the inverse
    __shared__ float Tm[16][kNB + 1];     // one row block of partial products
    __shared__ int bad_s;
    if (*status) return;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    {
        // all eight loads of a thread in flight at once (the block is one
        // dependent step of the factorisation's serial chain)
        float v[kNB * kNB / 512];
#pragma unroll
        for (int q = 0; q < kNB * kNB / 512; ++q) {
            const int idx = t + 512 * q, r = idx / kNB, c = idx % kNB;
            v[q] = (r < nb && c <= r) ? A[(size_t)(j0 + r) * n + (j0 + c)] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < kNB * kNB / 512; ++q) {
            const int idx = t + 512 * q, r = idx / kNB, c = idx % kNB;
            S[r][c] = v[q];
            V[r][c] = 0.0f;
        }
    }
    if (t == 0) bad_s = 0;
    __syncthreads();
    const int nblk = nb / 16;
    for (int K = 0; K < nblk; ++K) {
        const int k0 = 16 * K;
        if (warp == 0) {
            // lane l < 16 holds row l of the 16 x 16 diagonal block in registers
            float a[16];
            float rdg[16];                           // 1 / L[j][j], the same in every lane
#pragma unroll
            for (int m = 0; m < 16; ++m) a[m] = (lane < 16) ? S[k0 + lane][k0 + m] : 0.0f;
            int badj = -1;                           // the same in every lane
#pragma unroll 16   // fully: a[] must stay in registers
            for (int j = 0; j < 16; ++j) {
                const float d = __shfl_sync(0xffffffffu, a[j], j);
                const bool good = (d > 0.0f) && isfinite(d);
                if (!good && badj < 0) badj = j;
                // 1 / sqrt(d) once per column, warp-uniform (one MUFU operation,
                // ~2 ulp), then multiplies: the per-lane IEEE divisions were the
                // serial chain's longest links.  The factor is needed to fp32
                // accuracy, not to the last bit.
                const float dd = good ? d : 1.0f;
                rdg[j] = rsqrtf(dd);
                const float djj = dd * rdg[j];
                a[j] = (lane == j) ? djj : (lane > j ? a[j] * rdg[j] : a[j]);
                // rank-1 update: a[c] -= a[j] * L[c][j] for j < c <= lane
#pragma unroll
                for (int c = 0; c < 16; ++c) {
                    if (c > j) {
                        const float lcj = __shfl_sync(0xffffffffu, a[j], c);
                        if (lane >= c) a[c] = fmaf(-a[j], lcj, a[c]);
                    }
                }
            }
            if (badj >= 0 && lane == 0) bad_s = j0 + k0 + badj + 1;
            if (badj < 0) {
                if (lane < 16) {
#pragma unroll
                    for (int m = 0; m < 16; ++m)
                        if (m <= lane) S[k0 + lane][k0 + m] = a[m];
                }
                __syncwarp();
                if (lane < 16) {     // column `lane` of the block's inverse
                    const int c = lane;
                    const float (&rd)[16] = rdg;
                    float x[16];
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        float sacc = (j == c) ? 1.0f : 0.0f;
#pragma unroll
                        for (int m = 0; m < j; ++m) sacc = fmaf(-S[k0 + j][k0 + m], x[m], sacc);
                        x[j] = (j < c) ? 0.0f : sacc * rd[j];
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) V[k0 + j][k0 + c] = x[j];
                }
            }
        }
        __syncthreads();
        if (bad_s) break;
        const int rb = nb - k0 - 16;          // rows below the block
        if (rb > 0) {
            float val[2];
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int idx = t + 512 * q;
                val[q] = 0.0f;
                if (idx < rb * 16) {
                    const int r = k0 + 16 + (idx >> 4), c = idx & 15;
                    float acc = 0.0f;
#pragma unroll
                    for (int m = 0; m < 16; ++m) acc = fmaf(S[r][k0 + m], V[k0 + c][k0 + m], acc);
                    val[q] = acc;
                }
            }
            __syncthreads();
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                const int idx = t + 512 * q;
                if (idx < rb * 16) S[k0 + 16 + (idx >> 4)][k0 + (idx & 15)] = val[q];
            }
            __syncthreads();
            for (int idx = t; idx < rb * rb; idx += 512) {
                const int i = k0 + 16 + idx / rb, c = k0 + 16 + idx % rb;
                if (c <= i) {
                    float acc = S[i][c];
#pragma unroll
                    for (int m = 0; m < 16; ++m) acc = fmaf(-S[i][k0 + m], S[c][k0 + m], acc);
                    S[i][c] = acc;
                }
            }
            __syncthreads();
        }
    }
    if (bad_s) {
        if (t == 0) *status = bad_s;
        return;
    }
    for (int I = 1; I < nblk; ++I) {
        const int i0 = 16 * I;
        // Tm[r][c] = sum_{m = c_blk .. i0-1} L[i0 + r][m] V[m][c], c < i0
        for (int idx = t; idx < 16 * i0; idx += 512) {
            const int r = idx / i0, c = idx % i0;
            float acc = 0.0f;
            for (int m = 16 * (c / 16); m < i0; ++m) acc = fmaf(S[i0 + r][m], V[m][c], acc);
            Tm[r][c] = acc;
        }
        __syncthreads();
        for (int idx = t; idx < 16 * i0; idx += 512) {
            const int r = idx / i0, c = idx % i0;
            float acc = 0.0f;
#pragma unroll
            for (int m = 0; m <= 15; ++m) acc = fmaf(V[i0 + r][i0 + m], Tm[m][c], acc);
            V[i0 + r][c] = -acc;
        }
        __syncthreads();
    }
    for (int idx = t; idx < kNB * kNB; idx += 512) {
        const int r = idx / kNB, c = idx % kNB;
        if (r < nb && c <= r) A[(size_t)(j0 + r) * n + (j0 + c)] = S[r][c];
        Linv[idx] = (r < nb && c < nb) ? V[r][c] : 0.0f;
    }
}

// fp32 panel solve for the tensor-core path: rows i >= j0+nb of the panel,
// A[i, j0:j0+nb] <- A[i, j0:j0+nb] . Linv^T (Linv from potrf_diag_kernel), in
// 64-row tiles through shared memory (4 x 4 outputs per thread, ascending
// sum over the panel columns); writes the solved rows back in place and
// transposed into PT (PT[c][i - (j0+nb)], row pitch ldt) for the update GEMM.
__global__ void __launch_bounds__(256)
panel_apply_kernel(float* __restrict__ A, int n, int j0, int nb,
                   const float* __restrict__ Linv, float* __restrict__ PT, int ldt,
                   const int* __restrict__ status) {
    __shared__ float LI[kNB][kNB + 1];
    __shared__ float B[kNB][kNB + 1];
    if (*status) return;
    const int t = threadIdx.x;
    const int rest = n - j0 - nb;
    const int r0 = blockIdx.x * kNB;
    {
        // the tile's loads all in flight at once (this kernel is a step of the
        // factorisation's serial chain)
        constexpr int Q = kNB * kNB / 256;
        float li[Q], bv[Q];
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            const int idx = t + 256 * q, r = idx / kNB, c = idx % kNB;
            li[q] = (r < nb && c < nb) ? Linv[idx] : 0.0f;
            bv[q] = (r0 + r < rest && c < nb) ? A[(size_t)(j0 + nb + r0 + r) * n + j0 + c] : 0.0f;
        }
#pragma unroll
        for (int q = 0; q < Q; ++q) {
            const int idx = t + 256 * q, r = idx / kNB, c = idx % kNB;
            LI[r][c] = li[q];
            B[r][c] = bv[q];
        }
    }
    __syncthreads();
    const int rb = 4 * (t >> 4), cb = t & 15;   // rows rb..rb+3, columns cb + 16 j
    float acc[4][4] = {};
    for (int m = 0; m < kNB; ++m) {
        float bv[4], lv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) bv[i] = B[rb + i][m];
#pragma unroll
        for (int j = 0; j < 4; ++j) lv[j] = LI[cb + 16 * j][m];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(bv[i], lv[j], acc[i][j]);
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) B[rb + i][cb + 16 * j] = acc[i][j];
    __syncthreads();
    for (int idx = t; idx < kNB * kNB; idx += 256) {
        const int r = idx / kNB, c = idx % kNB;              // row-major, coalesced
        if (r0 + r < rest && c < nb) A[(size_t)(j0 + nb + r0 + r) * n + j0 + c] = B[r][c];
        const int c2 = idx / kNB, r2 = idx % kNB;            // transposed, coalesced
        if (r0 + r2 < rest && c2 < nb) PT[(size_t)c2 * ldt + r0 + r2] = B[r2][c2];
    }
}

// Rows i >= j0+nb: A[i, j0:j0+nb] <- A[i, j0:j0+nb] . L_jj^-T (forward
// substitution against the factored diagonal block), one thread per row.
template <typename T>
__global__ void __launch_bounds__(128)
trsm_panel_kernel(T* __restrict__ A, int n, int j0, int nb, const int* __restrict__ status) {
    __shared__ T L[kNB][kNB + 1];
    if (*status) return;
    for (int idx = threadIdx.x; idx < nb * nb; idx += blockDim.x) {
        const int r = idx / nb, c = idx % nb;
        L[r][c] = (c <= r) ? A[(size_t)(j0 + r) * n + (j0 + c)] : T(0);
    }
    __syncthreads();
    const int i = j0 + nb + blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    T* row = &A[(size_t)i * n + j0];
    T x[kNB];
#pragma unroll
    for (int j = 0; j < kNB; ++j) x[j] = (j < nb) ? row[j] : T(0);
#pragma unroll
    for (int j = 0; j < kNB; ++j) {
        if (j >= nb) break;
        T s = x[j];
#pragma unroll
        for (int m = 0; m < j; ++m) s = s - x[m] * L[j][m];
        x[j] = s / L[j][j];
    }
#pragma unroll
    for (int j = 0; j < kNB; ++j)
        if (j < nb) row[j] = x[j];
}

template <typename T>
__global__ void zero_upper_kernel(T* __restrict__ A, int n) {
    const size_t total = (size_t)n * n;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(idx / n), c = (int)(idx % n);
        if (c > r) A[idx] = T(0);
    }
}

// Outer panel of the two-level blocking (fp32 tensor-core path).
constexpr int kOuterNB = 512;

// panel_ws: the transposed outer panel [kOuterNB][ldt], Linv [kNB][kNB], the
// outer update's pre-split panel (one matrix: both operands), then the inner
// updates' pre-split operands
static size_t ldl_panel_floats(int n) {
    return (size_t)kOuterNB * ((n + 3) & ~3) + (size_t)kNB * kNB;
}
static size_t ldl_outer_split_bytes(int n) { return (size_t)n * kOuterNB * 8 + 1024; }
size_t ldl_panel_bytes(int n) {
    return ldl_panel_floats(n) * sizeof(float) + ldl_outer_split_bytes(n) +
           gemm_split_bytes(n, kOuterNB, kNB);
}

// Blocked right-looking Cholesky: diagonal block (kNB), panel solve, update.
// fp32 with panel_ws (tcgen05 tensor cores, 3xTF32, gemm_tc.cu) blocks on two
// levels, because a rank-64 update of the whole trailing matrix reads and
// writes all of it for 64 columns of work (memory-bound: ~220 GB of traffic at
// n = 17408):
//  * inner steps of kNB columns inside an outer panel of kOuterNB columns:
//    potrf, trsm of the rows below, and the rank-kNB update of the outer
//    panel's remaining columns only;
//  * one rank-kOuterNB update of the trailing matrix per outer panel
//    (compute-bound; 8x less traffic).
// Every inner panel P (rows below its diagonal block) is transposed once into
// panel_ws [kOuterNB][ldt] (row = column within the outer panel, column =
// global row - J); the inner updates and the outer update both read it.  The
// outer update runs in two parts: the next outer panel's columns first, then
// the rest.  With a helper stream `side` (high priority) the serial chain runs
// there and the rest-updates on the caller's stream, so a rest-update overlaps
// the next panel's diagonal steps; the update after it waits for it.  The
// GEMM covers the 128 x 128 tiles that reach the lower triangle -- the
// entries above the diagonal that the diagonal tiles also write are never read
// and are zeroed at the end.  fp64 (and fp32 without panel_ws): one level, SIMT
// update of the lower triangle.
template <typename T>
int cholesky_lower(T* A, int n, int* dstatus, cudaStream_t stream, float* panel_ws,
                   int* gemm_err, cudaStream_t side, cudaEvent_t ev_fork,
                   cudaEvent_t ev_join) {
    const bool tc = sizeof(T) == 4 && panel_ws != nullptr;
    const int outer = tc ? kOuterNB : n;
    const int ldt = (n + 3) & ~3;
    float* linv = tc ? panel_ws + (size_t)kOuterNB * ldt : nullptr;
    float* osplit = nullptr;
    void* isplit = nullptr;
    size_t isplit_bytes = 0;
    if (tc) {
        uint8_t* p = reinterpret_cast<uint8_t*>(panel_ws + ldl_panel_floats(n));
        osplit = reinterpret_cast<float*>(((uintptr_t)p + 1023) & ~(uintptr_t)1023);
        isplit = p + ldl_outer_split_bytes(n);
        isplit_bytes = gemm_split_bytes(n, kOuterNB, kNB);
    }
    // lookahead: the serial chain (diagonal steps, splits, next-panel updates)
    // runs on the high-priority helper stream `side`, the rest-updates on the
    // caller's stream, so that freed SMs go to the chain first
    const bool ahead = tc && side && ev_fork && ev_join;
    cudaStream_t cs = ahead ? side : stream;
    bool pending = false;                     // a rest-update is in flight on `stream`
    if (ahead && (check_cuda(cudaEventRecord(ev_join, stream), "lookahead start") ||
                  check_cuda(cudaStreamWaitEvent(cs, ev_join, 0), "lookahead start")))
        return RC_DEVICE_ERROR;
    for (int J = 0; J < n; J += outer) {
        const int W = (n - J) < outer ? (n - J) : outer;
        for (int j0 = J; j0 < J + W; j0 += kNB) {
            const int nb = (J + W - j0) < kNB ? (J + W - j0) : kNB;
            const int rest = n - j0 - nb;
            if (tc)
                potrf_inv_kernel<<<1, 512, 0, cs>>>(reinterpret_cast<float*>(A), n, j0, nb,
                                                    dstatus, linv);
            else
                potrf_diag_kernel<T><<<1, 1024, 0, cs>>>(A, n, j0, nb, dstatus);
            note_launch();
            if (rest <= 0) continue;
            const int wi = J + W - (j0 + nb);     // outer-panel columns right of this panel
            T* P = A + (size_t)(j0 + nb) * n + j0;
            T* C = A + (size_t)(j0 + nb) * n + (j0 + nb);
            int rc = RC_OK;
            if (tc) {
                // solve and transpose in one pass (the diagonal block's inverse)
                float* PT = panel_ws + (size_t)(j0 - J) * ldt + (j0 + nb - J);
                panel_apply_kernel<<<(rest + kNB - 1) / kNB, 256, 0, cs>>>(
                    reinterpret_cast<float*>(A), n, j0, nb, linv, PT, ldt, dstatus);
                note_launch();
                if (wi > 0)
                    rc = launch_gemm_tn_acc_tc(rest, wi, nb, PT, ldt, PT, ldt,
                                               reinterpret_cast<float*>(C), n, gemm_err,
                                               cs, -1.0f, 1, isplit, isplit_bytes);
            } else {
                trsm_panel_kernel<T><<<(rest + 127) / 128, 128, 0, stream>>>(A, n, j0, nb,
                                                                           dstatus);
                note_launch();
                if (wi > 0)
                    rc = gemm_launch<T, true, true, true>(rest, wi, nb, P, n, P, n, C, n,
                                                          T(-1), T(1), dstatus, stream);
            }
            if (rc) return rc;
            if (check_cuda(cudaGetLastError(), "cholesky launch")) return RC_DEVICE_ERROR;
        }
        const int R = n - (J + W);
        if (tc && R > 0) {
            // A[J+W:, J+W:] -= Q Q^T, Q = A[J+W:, J:J+W] (transposed: panel_ws rows
            // 0..W-1 from column W on), split once into osplit.  The previous
            // rest-update reads osplit and writes the columns this one does:
            // wait for it first.
            if (pending && check_cuda(cudaStreamWaitEvent(cs, ev_join, 0), "lookahead join"))
                return RC_DEVICE_ERROR;
            pending = false;
            const int kp = (W + 31) / 32 * 32;
            float* Qh = osplit;
            float* Ql = osplit + (size_t)R * kp;
            int rc = gemm_split(panel_ws + W, ldt, W, R, Qh, Ql, kp, cs);
            if (rc) return rc;
            float* Cf = reinterpret_cast<float*>(A);
            // (a) the next outer panel's columns, rows J+W.. (its diagonal block
            //     lower triangle + everything below), on the caller's stream
            const int W2 = R < outer ? R : outer;
            rc = gemm_presplit_run(R, W2, kp, Qh, Ql, Qh, Ql, Cf + (size_t)(J + W) * n + (J + W),
                                   n, -1.0f, 1, gemm_err, cs);
            if (rc) return rc;
            // (b) the rest of the trailing matrix (columns >= J+W+W2), on the
            //     caller's stream: it overlaps the next outer panel's diagonal
            //     steps, which touch columns < J+W+W2 only
            const int R2 = R - W2;
            if (R2 > 0) {
                if (ahead && (check_cuda(cudaEventRecord(ev_fork, cs), "lookahead fork") ||
                              check_cuda(cudaStreamWaitEvent(stream, ev_fork, 0),
                                         "lookahead fork")))
                    return RC_DEVICE_ERROR;
                const size_t o = (size_t)W2 * kp;
                rc = gemm_presplit_run(R2, R2, kp, Qh + o, Ql + o, Qh + o, Ql + o,
                                       Cf + (size_t)(J + W + W2) * n + (J + W + W2), n, -1.0f,
                                       1, gemm_err, stream);
                if (rc) return rc;
                if (ahead) {
                    if (check_cuda(cudaEventRecord(ev_join, stream), "lookahead join"))
                        return RC_DEVICE_ERROR;
                    pending = true;
                }
            }
        }
    }
    // the caller's stream continues after the chain's last work
    if (ahead && (check_cuda(cudaEventRecord(ev_fork, cs), "lookahead end") ||
                  check_cuda(cudaStreamWaitEvent(stream, ev_fork, 0), "lookahead end")))
        return RC_DEVICE_ERROR;
    zero_upper_kernel<T><<<1024, 256, 0, stream>>>(A, n);
    note_launch();
    return check_cuda(cudaGetLastError(), "zero_upper launch") ? RC_DEVICE_ERROR : RC_OK;
}

// ------------------------------------------------------------ block LDL post
// DLi[b] = inverse of the lower-triangular 16x16 diagonal block b of L
// (forward substitution, exact zeros above the diagonal); D[b] = DL DL^T.
template <typename T>
__global__ void __launch_bounds__(256)
dl_inverse_kernel(const T* __restrict__ L, int n, T* __restrict__ DLi, T* __restrict__ D) {
    __shared__ T S[16][17];
    __shared__ T I[16][17];
    const int b = blockIdx.x, t = threadIdx.x;
    const int r = t / 16, c = t % 16;
    S[r][c] = (c <= r) ? L[(size_t)(16 * b + r) * n + (16 * b + c)] : T(0);
    __syncthreads();
    if (D) {
        T s = T(0);
        for (int m = 0; m < 16; ++m) s += S[r][m] * S[c][m];
        D[(size_t)b * 256 + t] = s;
    }
    if (t < 16) {   // column t of the inverse: solve S x = e_t
        const int col = t;
        T x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            T s = (i == col) ? T(1) : T(0);
#pragma unroll
            for (int m = 0; m < i; ++m) s -= S[i][m] * x[m];
            x[i] = (i < col) ? T(0) : s / S[i][i];
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) I[i][col] = x[i];
    }
    __syncthreads();
    DLi[(size_t)b * 256 + t] = I[r][c];
}

// Lout[r, 16b:16b+16] = L[r, 16b:16b+16] . DLi[b] for r below block b,
// identity on the diagonal blocks, zero above.  Out-of-place (Lout fp32).
template <typename T>
__global__ void __launch_bounds__(256)
dl_apply_kernel(const T* __restrict__ L, int n, const T* __restrict__ DLi,
                float* __restrict__ Lout) {
    __shared__ T M[16][17];
    const int b = blockIdx.y;
    const int t = threadIdx.x;
    M[t / 16][t % 16] = DLi[(size_t)b * 256 + t];
    __syncthreads();
    const int r = blockIdx.x * 256 + t;
    if (r >= n) return;
    float* o = &Lout[(size_t)r * n + 16 * b];
    if (r < 16 * b) {
#pragma unroll
        for (int c = 0; c < 16; ++c) o[c] = 0.0f;
        return;
    }
    if (r < 16 * b + 16) {
#pragma unroll
        for (int c = 0; c < 16; ++c) o[c] = (c == r - 16 * b) ? 1.0f : 0.0f;
        return;
    }
    const T* a = &L[(size_t)r * n + 16 * b];
    T x[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) x[m] = a[m];
#pragma unroll
    for (int c = 0; c < 16; ++c) {
        T s = T(0);
#pragma unroll
        for (int m = 0; m < 16; ++m) s = fma(x[m], M[m][c], s);
        o[c] = (float)s;
    }
}

template <typename T>
int block_ldl(T* A, int n, float* Lout, T* dD, T* dDLi, int* dstatus, cudaStream_t stream,
              float* panel_ws, int* gemm_err, cudaStream_t side, cudaEvent_t ev_fork,
              cudaEvent_t ev_join) {
    int rc = cholesky_lower<T>(A, n, dstatus, stream, panel_ws, gemm_err, side, ev_fork,
                               ev_join);
    if (rc) return rc;
    dl_inverse_kernel<T><<<n / 16, 256, 0, stream>>>(A, n, dDLi, dD);
    dim3 g((n + 255) / 256, n / 16);
    dl_apply_kernel<T><<<g, 256, 0, stream>>>(A, n, dDLi, Lout);
    note_launch(2);
    return check_cuda(cudaGetLastError(), "block_ldl launch") ? RC_DEVICE_ERROR : RC_OK;
}

template int block_ldl<float>(float*, int, float*, float*, float*, int*, cudaStream_t, float*,
                              int*, cudaStream_t, cudaEvent_t, cudaEvent_t);
template int block_ldl<double>(double*, int, float*, double*, double*, int*, cudaStream_t,
                               float*, int*, cudaStream_t, cudaEvent_t, cudaEvent_t);

// ------------------------------------------------------------ quantize() U path
// Ui = U^-1 for upper-triangular U (fp64), column by column (one thread per
// column solving U x = e_c by back substitution over the upper triangle).
__global__ void trtri_upper_kernel(const double* __restrict__ U, int n, double* __restrict__ Ui) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= n) return;
    // x_i = 0 for i > c; back-substitute i = c .. 0
    for (int i = n - 1; i > c; --i) Ui[(size_t)i * n + c] = 0.0;
    for (int i = c; i >= 0; --i) {
        double s = (i == c) ? 1.0 : 0.0;
        for (int m = i + 1; m <= c; ++m) s -= U[(size_t)i * n + m] * Ui[(size_t)m * n + c];
        Ui[(size_t)i * n + c] = s / U[(size_t)i * n + i];
    }
}

__global__ void f32_to_f64_kernel(const float* __restrict__ a, double* __restrict__ b, size_t n) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        b[i] = (double)a[i];
}

// G = U^-1 U^-T in fp64 from an fp32 upper-triangular U (quantize.py:946-949).
int u_to_gram_f64(const float* U, int n, double* Ud, double* Ui, double* G, cudaStream_t stream) {
    f32_to_f64_kernel<<<1024, 256, 0, stream>>>(U, Ud, (size_t)n * n);
    trtri_upper_kernel<<<(n + 127) / 128, 128, 0, stream>>>(Ud, n, Ui);
    // G = Ui . Ui^T : A = Ui [M][K] K-major, B[k][j] = Ui[j][k] -> K-major
    int rc = gemm_launch<double, true, true, false>(n, n, n, Ui, n, Ui, n, G, n, 1.0, 0.0,
                                                    nullptr, stream);
    if (rc) return rc;
    note_launch(2);
    return check_cuda(cudaGetLastError(), "u_to_gram launch") ? RC_DEVICE_ERROR : RC_OK;
}

int launch_f32_to_f64(const float* a, double* b, size_t n, cudaStream_t stream) {
    f32_to_f64_kernel<<<1024, 256, 0, stream>>>(a, b, n);
    note_launch();
    return check_cuda(cudaGetLastError(), "f32_to_f64 launch") ? RC_DEVICE_ERROR : RC_OK;
}

}  // namespace exl3b
