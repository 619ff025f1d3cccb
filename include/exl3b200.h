/* exl3b200.h -- C ABI of libexl3b200.so, the B200 EXL3 trellis quantizer.
 *
 * Plain pointers and sizes; no framework types.  Every function returns an
 * int status (0 = success; codes below) and never aborts the process;
 * exl3b_last_error() returns a text description of the calling thread's last
 * failure.  "d" pointers are CUDA device pointers on the current device;
 * `stream` is a cudaStream_t (NULL = legacy default stream).  Entry points
 * that take a stream are asynchronous with respect to the host.
 *
 * Reference interfaces replaced (SergiioB/exl3xpu-mixedk):
 *   quantize/viterbi_esimd.cpp:935-968   xtq_vit_init
 *   quantize/viterbi_esimd.cpp:970-1005  xtq_vit_run
 *   quantize/quantize.py:611-628         _esimd_tailbite  (exl3b_tailbite)
 *   quantize/quantize.py:323-354         quantize_seq_tailbite
 *   quantize/quantize.py:218-320         viterbi          (exl3b_viterbi)
 *   quantize/quantize.py:135-146         had_left / had_right (exl3b_hadamard_axis)
 *   quantize/quantize.py:849-853, 958-963  the per-tensor self-check asserts
 *                                        (exl3b_verify_trellis)
 * and the pipeline entry points below, each with its reference lines.
 */
#ifndef EXL3B200_H
#define EXL3B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EXL3B_ABI_VERSION 1

/* Status codes.  1..7 keep the meanings of the reference's xtq_vit_* codes. */
#define EXL3B_OK              0
#define EXL3B_NO_DEVICE       1   /* no CUDA device / init failure            */
#define EXL3B_ALLOC           2   /* device allocation failed                 */
#define EXL3B_BAD_DEVICE      3   /* device index out of range                */
#define EXL3B_DEVICE_ERROR    4   /* CUDA error in a launch or copy           */
#define EXL3B_TOO_MANY_BYTES  5   /* over XTQ_VIT_MAXBYTES                    */
#define EXL3B_BAD_NSEQ        6   /* sequence count out of range              */
#define EXL3B_BAD_REQUEST     7   /* malformed request / unsupported code     */
#define EXL3B_BAD_K           8   /* K outside 2..7                           */
#define EXL3B_NOT_SPD         9   /* factorisation met a non-positive pivot   */
#define EXL3B_NONFINITE      10   /* non-finite input                         */
#define EXL3B_WORKSPACE      11   /* caller workspace too small / misaligned  */

/* Code ids of the V=1 decode tables (quantize.py:56-87). */
#define EXL3B_CODE_MUL1   0       /* "exl3_mul1"  */
#define EXL3B_CODE_3INST  1       /* "exl3_3inst" */
#define EXL3B_CODE_MCG    2       /* "exl3_mcg"   */

/* Text of the calling thread's last error ("" if none). */
const char* exl3b_last_error(void);

/* EXL3B_ABI_VERSION of the loaded library. */
int exl3b_abi_version(void);

/* Host-only: fp32 [65536] decode table of a code id (quantize.py:90-97
 * get_lut).  Needs no GPU. */
int exl3b_code_lut(int code, float* out65536);

/* Number of CUDA kernels this library has launched (all devices, all
 * threads) since it was loaded. */
long long exl3b_launch_count(void);

/* Per-launch CUDA-event timing of the dominant kernels, on the stream each
 * is launched on.  exl3b_profile_begin() starts recording; exl3b_profile_end
 * stops, synchronises the recorded events and returns, for `kind`
 * (0 = fused LDLQ tile kernel, 1 = feedback GEMM, 2 = standalone encoder,
 * 3 = Hadamard rotations of W / W_hat / H, 4 = block LDL factorisation),
 * the summed duration, the launch count and the summed work units
 * (0, 2: weights encoded; 1: useful FLOP; 3: algorithmic bytes; 4: k^3/3
 * FLOP). */
void exl3b_profile_begin(void);
int exl3b_profile_end(int kind, double* ms_total, long long* launches, double* units);

/* Select `device` and build its decode tables (optional; first use of any
 * entry point initialises the current device). */
int exl3b_device_init(int device);

/* Bound, in milliseconds, of every device-side wait of the LDLQ sweep (a tile
 * waiting for the tile below it in its column, a backpointer-slot claim); 0
 * restores the default of 4000 ms.  A wait that runs out ends its kernel with
 * an error block, and exl3b_ldlq_sweep returns EXL3B_DEVICE_ERROR with the
 * cause in exl3b_last_error(); the context stays usable.  Applies to sweeps
 * started afterwards, in every thread.  No counterpart in the reference (its
 * native encoder has no cross-CTA waits). */
int exl3b_set_wait_limit_ms(double ms);

/* Workspace bytes exl3b_tailbite needs for (nseq, K) on the current device
 * (0 for invalid arguments). */
size_t exl3b_tailbite_workspace_bytes(int nseq, int K);

/* Tail-biting Viterbi encode (quantize_seq_tailbite, quantize.py:323-354,
 * bit-exact with its fp32 "sq" emit), K = 2..7, V = 1.
 *   dX       [nseq][256] fp32 targets, 16-byte aligned (one tile per row,
 *            element t = tile position perm[t])
 *   pivot    pass-1 boundary step, 0 <= pivot < 256
 *   margin   0 = full pass 1; > 0 = pass 1 runs pivot+margin steps
 *   dStates  [nseq][256] int32 full 16-bit states
 *   workspace/workspace_bytes: caller scratch (256-byte aligned, at least
 *            exl3b_tailbite_workspace_bytes) or NULL for library scratch. */
int exl3b_tailbite(const float* dX, int nseq, int K, int code, int pivot,
                   int margin, int32_t* dStates, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Single Viterbi pass (viterbi, quantize.py:218-320), bit-exact with its fp32
 * "sq" emit; the building block of the tail-biting encode.
 *   dX        [nseq][T] fp32 targets, 1 <= T <= 256
 *   dOverlap  [nseq] int32 or NULL: pins s_0 >> K and s_{T-1} mod 2^(16-K)
 *             to overlap[b] (values taken mod 2^(16-K))
 *   back_from -1: dStates [nseq][T] receives every state; >= 0: backpointers
 *             are kept only for steps after back_from and dStates [nseq]
 *             receives the state at step back_from (the state at T-1 when
 *             back_from >= T-1), as the reference's back_from argument
 *   workspace/workspace_bytes: exl3b_viterbi_workspace_bytes(nseq, K) bytes,
 *             256-byte aligned, or NULL for library scratch. */
size_t exl3b_viterbi_workspace_bytes(int nseq, int K);
int exl3b_viterbi(const float* dX, int nseq, int T, int K, int code,
                  const int32_t* dOverlap, int back_from, int32_t* dStates,
                  void* workspace, size_t workspace_bytes, void* stream);

/* Tail-biting encode that allocates no device memory.  No counterpart in the
 * reference: it is for callers that must not allocate device memory while
 * they run -- a process whose GPU memory belongs to another allocator (for
 * example an inference server that reserves the device's memory at start-up
 * and treats later cudaMalloc calls as failures), or a loop that cannot take
 * the device-wide synchronisation cudaMalloc / cudaFree can cause.  Same
 * arguments and results as exl3b_tailbite, minus the workspace: the
 * backpointer scratch is a fixed 64 MiB device array inside the library and
 * the decode values are computed from the code formulas.  The array is
 * created when the CUDA runtime loads the library's device code on a GPU and
 * kept until the process exits: under lazy module loading (the default since
 * CUDA 12.2) that is during the first call on each device, which therefore
 * does take 64 MiB; under eager loading, every context that loads the library
 * takes it at start-up.  Make one warm-up call per device before reserving
 * the device's memory and before any stream capture; later calls allocate
 * nothing.  At most 64 (K = 2, 3), 128 (K = 4, 5), 256 (K = 6) or 512 (K = 7)
 * sequences per call; more returns EXL3B_BAD_NSEQ.  All calls on a device
 * share the scratch: calls that overlap on the GPU race, so issue them in
 * order on one stream. */
int exl3b_tailbite_noalloc(const float* dX, int nseq, int K, int code, int pivot,
                           int margin, int32_t* dStates, void* stream);

/* Drop-in for the reference's native Viterbi (viterbi_esimd.cpp:935-1005):
 * same signatures, argument meaning and return codes.  Host X [nseq][256]
 * fp32 in, host int32 states [nseq][256] out, synchronous, mul1 code at
 * K = 4 ("mul1p", "mul1", "mul1t").  Env: XTQ_VIT_DEVIDX, XTQ_VIT_MAXSEQ,
 * XTQ_VIT_MAXBYTES. */
int xtq_vit_init(void);
int xtq_vit_run(const float* X, int nseq, const char* code, int margin,
                int pivot, int32_t* out);


/* ===================================================================
 * Quantizer pipeline (quantize/quantize.py:749-966).  Device pointers,
 * asynchronous on `stream` unless stated.  Matrices are row-major;
 * "[k][n]" is the reference's inner orientation (k = in, n = out).
 * =================================================================== */

/* Incoherence, forward (to_inner, quantize.py:149-155):
 *   Wi[k][n] = B_128 . diag(row_mul) . W^T . diag(col_mul) . B_128
 * W [m_out][k_in] of dtype 0 = fp32, 1 = bf16, 2 = fp16; row_mul [k_in] and
 * col_mul [m_out] multipliers (1/suh, 1/svh) or NULL; both dims multiples of
 * 128.  sumsq_parts (nullable, [(k/128)*(n/128)] fp64) receives per-block
 * sums of squares of Wi (deterministic rms). */
int exl3b_incoherence_fwd(const void* dW, int dtype, int m_out, int k_in,
                          const float* d_row_mul, const float* d_col_mul,
                          float* dWi, double* d_sumsq_parts, void* stream);

/* Incoherence, inverse (from_inner, quantize.py:158-164), output transposed:
 *   W[n][k] = ((B . (s * Wi) ) * su[:,None] . B * sv[None,:])^T
 * with s = *d_pre_scale (device scalar, nullable = 1). */
int exl3b_incoherence_inv(const float* dWi, int k, int n, const float* d_pre_scale,
                          const float* d_su, const float* d_sv, float* dW,
                          void* stream);

/* EXL3 per-channel magnitude folds (quantize_linear channel_scales=True,
 * quantize.py:785-800; prepare_incoherence :1025-1041):
 *   sv_mag = rms_in(W) / mean(rms_in(W)), 0.1 where ~0 (sv_store: 0 there)
 *   w = had_right(W^T / (sv * sv_mag));  su_mag = rms_out(w) (0.1 where ~0)
 *   Wi[k][n] = had_left(w / (su * su_mag))
 * su/sv are the sign vectors (fp32 +-1).  Outputs su_mag [k], sv_mag [n],
 * sv_store [n]; sumsq_parts as in exl3b_incoherence_fwd. */
size_t exl3b_channel_scale_workspace_bytes(int m_out, int k_in);
int exl3b_channel_scale_fwd(const void* dW, int dtype, int m_out, int k_in,
                            const float* d_su, const float* d_sv, float* dWi,
                            float* d_su_mag, float* d_sv_mag, float* d_sv_store,
                            double* d_sumsq_parts, void* ws, size_t ws_bytes,
                            void* stream);

/* Stored EXL3 fields (quantize.py:857-858): suh = fp16(su * su_mag * Wscale)
 * (d_wscale nullable = 1), svh = fp16(sv * sv_store). */
int exl3b_channel_scale_store(const float* d_su, const float* d_su_mag,
                              const float* d_wscale, const float* d_sv,
                              const float* d_sv_store, int k, int n,
                              void* d_suh_f16, void* d_svh_f16, void* stream);

/* Hessian rotation (rotate_hessian, quantize.py:167-176):
 *   G = B . diag(su) . H . diag(su) . B,  H, G fp32 [k][k]. */
int exl3b_rotate_hessian(const float* dH, int k, const float* d_su, float* dG,
                         void* stream);

/* Damping (quantize.py:810-814): dead diagonal entries -> 1, then
 * diag += percdamp * mean(diag).  d_nonfinite (nullable) receives the count
 * of non-finite entries of the damped G. */
int exl3b_damp_hessian(float* dG, int k, float percdamp, int* d_nonfinite,
                       void* stream);

/* Fallback escalation (quantize.py:823-829): G64 = fp64 copy of G, then
 * diag(G64) += extra * mean(diag(G64)). */
int exl3b_convert_f32_f64(const float* dA, double* dB, size_t n, void* stream);
int exl3b_damp_hessian_f64(double* dG, int k, double extra, void* stream);

/* quantize() harness transposes (quantize.py:933-942, 961-965):
 *   inverse = 0: Y[k][n] = X[n][k] / (row_mag[n] * col_mag[k])
 *   inverse = 1: Y[n][k] = (X[k][n] * (*d_scale)) * (row_mag[n] * col_mag[k])
 * mags nullable (= 1); X is [rows_x][cols_x]; sumsq_parts as above
 * ([ceil(rows_x/32) * ceil(cols_x/32)] fp64, nullable). */
int exl3b_transpose_scale(int inverse, const float* dX, int rows_x, int cols_x,
                          const float* d_row_mag, const float* d_col_mag,
                          const float* d_scale, float* dY,
                          double* d_sumsq_parts, void* stream);

/* *d_scale = fl32(sqrt(fl32(sum(parts) / count))) / lut_rms
 * (quantize.py:803 / :941, fixed summation order). d_tmp: 1 fp64 scratch. */
int exl3b_rms_scale(const double* d_parts, int nparts, double count,
                    float lut_rms, double* d_tmp, float* d_scale, void* stream);

/* y = x / *d_s elementwise (IEEE fp32 division), n a multiple of 4. */
int exl3b_div_scalar(const float* dx, const float* d_s, float* dy, size_t n,
                     void* stream);

/* Block LDL (block_LDL, quantize.py:419-437): Cholesky of the SPD matrix A
 * (fp32, or fp64 if f64; destroyed), 16x16 diagonal-block inverses,
 * Lfac = L . blockdiag(DL^-1) with identity diagonal blocks, written as fp32
 * [k][k] (the fp64 path's Lfac.float()).  dD (nullable) receives D blocks
 * [k/16][16][16] in A's precision.  Synchronises `stream`; returns
 * EXL3B_NOT_SPD if a pivot is not positive (quantize.py:815-835 fallback is
 * the caller's). */
size_t exl3b_block_ldl_workspace_bytes(int k, int f64);
int exl3b_block_ldl(void* dA, int k, int f64, float* dLfac, void* dD, void* ws,
                    size_t ws_bytes, void* stream);

/* quantize() U path (quantize.py:944-949): G = U^-1 U^-T in fp64 from an
 * fp32 upper-triangular U [k][k]. */
size_t exl3b_u_to_gram_workspace_bytes(int k);
int exl3b_u_to_gram(const float* dU, int k, double* dG, void* ws,
                    size_t ws_bytes, void* stream);

/* BlockLDLQ sweep with fused tail-biting trellis encode (ldlq_viterbi,
 * quantize.py:631-746, pack_states :360-378).
 *   dWq   [k][n] fp32 unit-scaled inner weights
 *   dLfac [k][k] fp32 block-LDL factor, or NULL (plain trellis encode)
 *   segments: column tiles [seg_c0[s], seg_c0[s+1]) use K = seg_K[s] and write
 *         trellis int16 [k/16][(seg_c0[s+1]-seg_c0[s])][16 K] at seg_trellis[s]
 *         (seg_c0 has nseg+1 entries, seg_c0[0] = 0, seg_c0[nseg] = n/16;
 *         up to 8 segments: one fused module with per-member K)
 *   dHatW [k][n] fp32 decoded weights (output)
 *   dStates [k/16][n/16][256] int32 (nullable), dXout [k/16][n/16][256]
 *         fp32 encoder targets (nullable; for per-launch checks)
 *   buf_cols: the reference's LDLQ buffer (rows of k between feedback-cache
 *         updates); launches cover max(buf_cols, 512) rows, the fastest
 *         blocking here (the LDLQ targets are the same sums in another fp32
 *         order)
 *   block_lo/block_hi: process k-blocks [block_lo, block_hi) (full sweep:
 *         0, k/16); successive calls must walk downwards with the same ws
 *   ws: exl3b_ldlq_workspace_bytes(k, n, min K, dLfac != NULL) bytes,
 *         256-byte aligned; holds E = Wq - hatW, the feedback cache and the
 *         encoder backpointers. */
size_t exl3b_ldlq_workspace_bytes(int k, int n, int kmin, int use_ldlq);
int exl3b_ldlq_sweep(const float* dWq, const float* dLfac, int k, int n, int nseg,
                     const int* seg_c0, const int* seg_K, int16_t* const* seg_trellis,
                     int code, int pivot, int margin, int buf_cols, float* dHatW,
                     int32_t* dStates, float* dXout, int block_lo, int block_hi,
                     void* ws, size_t ws_bytes, void* stream);

/* LDLQ feedback-cache update (quantize.py:742-744) on tcgen05 tensor cores:
 *   C[M][N] += A_T^T . B,   A_T [K][M] (row pitch lda), B [K][N] (pitch ldb)
 * 3xTF32 (fp32-grade) products, TMA-fed, fp32 accumulation.  Pointers 16-byte
 * aligned, lda / ldb multiples of 4.  ws: >= 256 bytes of device scratch (a
 * status word).  With exl3b_feedback_gemm_workspace_bytes(M, N, K) bytes the
 * operands are split into tf32 hi / lo once per call (K in pieces of 512)
 * instead of once per output tile: the same products, faster when there are
 * many output tiles.  Synchronises `stream`. */
size_t exl3b_feedback_gemm_workspace_bytes(int M, int N, int K);
int exl3b_feedback_gemm(int M, int N, int K, const float* dA_T, int lda, const float* dB,
                        int ldb, float* dC, int ldc, void* ws, size_t ws_bytes,
                        void* stream);

/* Per-tensor self-check of an encoded column segment (the reference's
 * asserts at quantize.py:849-853 and :958-963: pack/unpack round trip and
 * decode == encoder output).  Adds to *dMismatch (device int, caller-zeroed)
 * the number of weights whose value decoded from dTrellis [tk][tn][16K]
 * through `code` differs (bit pattern) from dHatW [16 tk][ldw] (the
 * segment's first column; ldw >= 16 tn) and, when dStates [tk][ld_states]
 * [256] (int32, the segment's first tile; nullable) is given, the number of
 * states unpacked from the trellis that differ from the encoder's. */
int exl3b_verify_trellis(const int16_t* dTrellis, int tk, int tn, int K, int code,
                         const float* dHatW, int ldw, const int32_t* dStates, int ld_states,
                         int* dMismatch, void* stream);

/* One-sided block-128 Hadamard (had_left / had_right, quantize.py:135-146) of
 * X [rows][cols] fp32: axis 0 along rows (rows % 128 == 0, any cols), axis 1
 * along columns (cols % 128 == 0, any rows); normalised by 1/sqrt(128).
 * dY may equal dX. */
int exl3b_hadamard_axis(const float* dX, int rows, int cols, int axis, float* dY,
                        void* stream);

/* Bitstream (quantize.py:360-415): pack int32 states [ntiles][256] into
 * int16 [ntiles][16K]; unpack back to full 16-bit states; decode a trellis
 * [tk][tn][16K] to W_inner fp32 [16 tk][16 tn] through code `code`. */
int exl3b_pack_states(const int32_t* dStates, int ntiles, int K, int16_t* dOut,
                      void* stream);
int exl3b_unpack_states(const int16_t* dTrellis, int ntiles, int K,
                        int32_t* dStates, void* stream);
int exl3b_decode_trellis(const int16_t* dTrellis, int tk, int tn, int K, int code,
                         float* dW, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* EXL3B200_H */
