// linalg.cu -- Hessian factorisation for BlockLDLQ on fp32/fp64 CUDA cores.
//
// Reference: quantize/quantize.py:419-437 block_LDL (Cholesky, 16x16 diagonal
// block inverses, L <- L . blockdiag(DL^-1), identity diagonal blocks) with
// the fp32 path of quantize_linear (:816) and the fp64 paths of its fallback
// (:817-835) and of quantize()'s U -> G conversion (:944-950).
//
// Cholesky: blocked right-looking, panel 64: (1) one CTA factors the 64x64
// diagonal block in shared memory and records a LAPACK-style info (1-based
// column of the first non-positive / non-finite pivot) in a device status
// word; (2) rows below solve against the panel (triangular solve); (3) SIMT
// GEMM updates the trailing lower triangle.  Later launches skip work once the
// status is set; the host reads the status once at the end.
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
// triangle, 2-D strided without integer division.
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

// PT[c][r] = P[r][c] for the rows x cols panel P (row pitch ldp); PT row pitch
// ldt.  32 x 32 tiles through shared memory (coalesced both ways).
__global__ void __launch_bounds__(256)
transpose_panel_kernel(const float* __restrict__ P, int ldp, int rows, int cols,
                       float* __restrict__ PT, int ldt) {
    __shared__ float tile[32][33];
    const int r0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8
    for (int k = ty; k < 32; k += 8) {
        const int r = r0 + k, c = c0 + tx;
        tile[k][tx] = (r < rows && c < cols) ? P[(size_t)r * ldp + c] : 0.0f;
    }
    __syncthreads();
    for (int k = ty; k < 32; k += 8) {
        const int c = c0 + k, r = r0 + tx;
        if (c < cols && r < rows) PT[(size_t)c * ldt + r] = tile[tx][k];
    }
}

// Outer panel of the two-level blocking (fp32 tensor-core path).
constexpr int kOuterNB = 512;

size_t ldl_panel_bytes(int n) { return (size_t)kOuterNB * ((n + 3) & ~3) * sizeof(float); }

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
// GEMM covers the 128 x 128 tiles that reach the lower triangle -- the
// entries above the diagonal that the diagonal tiles also write are never read
// and are zeroed at the end.  fp64 (and fp32 without panel_ws): one level, SIMT
// update of the lower triangle.
template <typename T>
int cholesky_lower(T* A, int n, int* dstatus, cudaStream_t stream, float* panel_ws,
                   int* gemm_err) {
    const bool tc = sizeof(T) == 4 && panel_ws != nullptr;
    const int outer = tc ? kOuterNB : n;
    const int ldt = (n + 3) & ~3;
    for (int J = 0; J < n; J += outer) {
        const int W = (n - J) < outer ? (n - J) : outer;
        for (int j0 = J; j0 < J + W; j0 += kNB) {
            const int nb = (J + W - j0) < kNB ? (J + W - j0) : kNB;
            potrf_diag_kernel<T><<<1, 1024, 0, stream>>>(A, n, j0, nb, dstatus);
            note_launch();
            const int rest = n - j0 - nb;
            if (rest <= 0) continue;
            trsm_panel_kernel<T><<<(rest + 127) / 128, 128, 0, stream>>>(A, n, j0, nb, dstatus);
            note_launch();
            const int wi = J + W - (j0 + nb);     // outer-panel columns right of this panel
            T* P = A + (size_t)(j0 + nb) * n + j0;
            T* C = A + (size_t)(j0 + nb) * n + (j0 + nb);
            int rc = RC_OK;
            if (tc) {
                float* PT = panel_ws + (size_t)(j0 - J) * ldt + (j0 + nb - J);
                dim3 g((rest + 31) / 32, (nb + 31) / 32);
                transpose_panel_kernel<<<g, 256, 0, stream>>>(
                    reinterpret_cast<const float*>(P), n, rest, nb, PT, ldt);
                note_launch();
                if (wi > 0)
                    rc = launch_gemm_tn_acc_tc(rest, wi, nb, PT, ldt, PT, ldt,
                                               reinterpret_cast<float*>(C), n, gemm_err,
                                               stream, -1.0f, 1);
            } else if (wi > 0) {
                rc = gemm_launch<T, true, true, true>(rest, wi, nb, P, n, P, n, C, n, T(-1),
                                                      T(1), dstatus, stream);
            }
            if (rc) return rc;
            if (check_cuda(cudaGetLastError(), "cholesky launch")) return RC_DEVICE_ERROR;
        }
        const int R = n - (J + W);
        if (tc && R > 0) {
            // A[J+W:, J+W:] -= Q Q^T, Q = A[J+W:, J:J+W] (transposed: panel_ws
            // rows 0..W-1 from column W on)
            const float* QT = panel_ws + W;
            float* C = reinterpret_cast<float*>(A) + (size_t)(J + W) * n + (J + W);
            const int rc = launch_gemm_tn_acc_tc(R, R, W, QT, ldt, QT, ldt, C, n, gemm_err,
                                                 stream, -1.0f, 1);
            if (rc) return rc;
        }
    }
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
              float* panel_ws, int* gemm_err) {
    int rc = cholesky_lower<T>(A, n, dstatus, stream, panel_ws, gemm_err);
    if (rc) return rc;
    dl_inverse_kernel<T><<<n / 16, 256, 0, stream>>>(A, n, dDLi, dD);
    dim3 g((n + 255) / 256, n / 16);
    dl_apply_kernel<T><<<g, 256, 0, stream>>>(A, n, dDLi, Lout);
    note_launch(2);
    return check_cuda(cudaGetLastError(), "block_ldl launch") ? RC_DEVICE_ERROR : RC_OK;
}

template int block_ldl<float>(float*, int, float*, float*, float*, int*, cudaStream_t, float*,
                              int*);
template int block_ldl<double>(double*, int, float*, double*, double*, int*, cudaStream_t,
                               float*, int*);

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
