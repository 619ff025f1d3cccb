// exl3b_internal.h -- host-side declarations shared by the .cu files.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "exl3b_common.cuh"

namespace exl3b {

constexpr int kMaxDevices = 64;

// Per-device state owned by the library (decode tables, grow-only scratch).
struct DeviceState {
    bool ready = false;
    int sms = 0;
    __half* lut16[3] = {nullptr, nullptr, nullptr};   // per CodeId, [65536]
    float* lut32[3] = {nullptr, nullptr, nullptr};
    uint4* f2tab[3][8] = {};          // per (CodeId, K): pre-paired decode words
    uint8_t* scratch = nullptr;       // library-owned workspace (grow-only)
    size_t scratch_bytes = 0;
    float* stageX = nullptr;          // xtq_vit_run staging (grow-only)
    int32_t* stageS = nullptr;
    size_t stage_seqs = 0;
    // block LDL lookahead: a high-priority helper stream and fork / join events
    cudaStream_t side = nullptr;
    cudaEvent_t ev_fork = nullptr, ev_join = nullptr;
};

// Kernel-launch accounting (exl3b_launch_count) and optional per-launch
// CUDA-event timing of the dominant kernels (exl3b_profile_*).
void note_launch(int n = 1);
enum ProfKernel : int { PROF_TILE = 0, PROF_GEMM = 1, PROF_TAILBITE = 2, PROF_ROTATE = 3,
                        PROF_LDL = 4, PROF_N = 5 };
bool prof_on();
void prof_begin_launch(cudaStream_t s, int kind, double units);
void prof_end_launch(cudaStream_t s);

// Current device's state, initialised on first use (rc != 0 on failure).
int device_state(DeviceState** out);
int device_sms();

// Host-side decode table (fp32, fp16-exact values) for a code id.
int build_code_lut(int code, float* out65536);

// Bytes of one CTA's backpointer slot for K.
size_t bp_slot_bytes(int K);

// Pre-paired decode-word table ([16][512] uint4) of code/K, built on first use.
int f2tab_get(DeviceState* st, int code, int K, const uint4** out);
int build_f2tab(int K, const __half* lut16, uint4* tab, cudaStream_t stream);

// Tail-biting encode of nseq sequences X [nseq][256] -> states [nseq][256].
// Standalone encoder plan for (nseq, K) on a device with `sms` SMs: the
// lazy-argmin pipeline (K >= kLazyMinK, at least two sequences per SM; grid =
// SMs, two row regions per CTA) or the traced encoder (grid = min(nseq, SMs),
// one backpointer slot per CTA); bytes = workspace needed.  The same rule
// picks the LDLQ sweep's tile kernel per launch.
constexpr int kLazyMinK = 2;
inline bool lazy_pipeline(int K, long long units, int sms) {
    return K >= kLazyMinK && sms > 0 && units >= 2LL * sms;
}
struct TailbitePlan { bool lazy; int grid; size_t bytes; };
TailbitePlan tailbite_plan(int nseq, int K, int sms);
size_t lazy_region_bytes(int K);
int launch_tailbite(const float* dX, int nseq, int K, int pivot, int margin,
                    int32_t* dStates, uint8_t* ws, const TailbitePlan& plan,
                    const uint4* f2tab, const float* lut32, cudaStream_t stream);
// Single Viterbi pass over nseq sequences of T <= 256 targets (X [nseq][T]):
// optional per-sequence overlap pin, back_from < 0 for all states
// ([nseq][T]) else the state at back_from ([nseq]).  Waves of `grid` CTAs,
// one backpointer slot (bp_slot_bytes(K)) per CTA of a wave.
int launch_viterbi(const float* dX, int nseq, int T, int K, const int32_t* dOverlap,
                   int back_from, int32_t* dStates, uint8_t* ws, int grid,
                   const uint4* f2tab, cudaStream_t stream);

// ------------------------------------------------------------ incoherence
struct HadParams {
    const void* X;      // input matrix
    int in_dtype;       // 0 fp32, 1 bf16, 2 fp16
    int ldx;            // input row stride (elements)
    bool trans_in;      // block element (r, c) = X[c][r] instead of X[r][c]
    float* Y;           // output fp32
    int ldy;
    bool trans_out;     // write Y[c][r]
    int rows, cols;     // logical matrix (after trans_in), multiples of 128
    float pre_scale;    // scalar multiply on load
    const float* pre_scale_dev;  // device scalar multiply on load (nullable)
    const float* pre_r; // per-row multiplier on load (nullable)
    const float* pre_c; // per-col multiplier on load (nullable)
    const float* mid_r; // per-row multiplier between the transforms
    const float* post_c;// per-col multiplier after both transforms
    double* sumsq;      // per-block sum of squares of Y (nullable), [nblocks]
    const float* pre_r_div;  // per-row divisor on load (nullable)
    const float* pre_c_div;  // per-col divisor on load (nullable)
    bool skip_left;     // no transform along rows (r)
    bool skip_right;    // no transform along cols (c)
    double* row_sumsq;  // per-row partial sums of squares [rows][cols/128]
};

int launch_had2(const HadParams& p, cudaStream_t stream);
int launch_transpose_scale(bool inv, const float* X, int rows_x, int cols_x,
                           const float* rmag, const float* cmag, const float* s,
                           float* Y, double* sumsq, cudaStream_t stream);
int launch_rms_scale(const double* partials, int nparts, double count, float lut_rms,
                     double* tmp1, float* scale, cudaStream_t stream);
int launch_div_scalar(const float* x, const float* s, float* y, size_t n, cudaStream_t stream);
int launch_damp(float* G, int k, float percdamp, cudaStream_t stream);
int launch_count_nonfinite(const float* G, size_t n, int* cnt, cudaStream_t stream);
int launch_damp_f64(double* G, int k, double extra, cudaStream_t stream);
int launch_row_rms(const void* X, int dtype, int rows, int cols, float* rms, cudaStream_t stream);
int launch_chan_out(float* r_out, const float* sv, int n, float* div_c, float* store_c,
                    cudaStream_t stream);
int launch_chan_in(const double* row_parts, int k, int nparts, const float* su, float* r_in,
                   float* div_r, cudaStream_t stream);
int launch_chan_store(const float* su, const float* r_in, const float* wscale,
                      const float* sv, const float* store_c, int k, int n,
                      __half* suh, __half* svh, cudaStream_t stream);
int launch_f32_to_f64(const float* a, double* b, size_t n, cudaStream_t stream);

// ------------------------------------------------------------ factorisation
// side / ev_fork / ev_join (optional, fp32 tensor-core path): a helper stream
// and two events for the lookahead that overlaps each outer panel's trailing
// update with the next panel's factorisation
template <typename T>
int block_ldl(T* A, int n, float* Lout, T* dD, T* dDLi, int* dstatus, cudaStream_t stream,
              float* panel_ws = nullptr, int* gemm_err = nullptr, cudaStream_t side = nullptr,
              cudaEvent_t ev_fork = nullptr, cudaEvent_t ev_join = nullptr);
// fp32 scratch a block_ldl<float> on tensor cores needs (transposed outer panel
// 512 x n, the diagonal block's inverse, the update GEMMs' pre-split operands)
size_t ldl_panel_bytes(int n);
int u_to_gram_f64(const float* U, int n, double* Ud, double* Ui, double* G, cudaStream_t stream);
int launch_gemm_tn_acc_f32(int M, int N, int K, const float* A_T, int lda,
                           const float* B, int ldb, float* C, int ldc, cudaStream_t stream);
int launch_gemm_tn_acc_tc(int M, int N, int K, const float* A_T, int lda, const float* B,
                          int ldb, float* C, int ldc, int* err, cudaStream_t stream,
                          float sa = 1.0f, int lower = 0, void* split_ws = nullptr,
                          size_t split_bytes = 0);
// scratch of the pre-split operand path of launch_gemm_tn_acc_tc
size_t gemm_split_bytes(int M, int N, int K);
// the pre-split path in two steps: X [K][R] (pitch ld, K <= 512) -> tf32 hi / lo
// [R][kp] (kp = K rounded up to 32; arrays 16-byte aligned), then
// C[M][N] += sa * A.B^T over such arrays (rows of A and B: M and N)
int gemm_split(const float* X, int ld, int K, int R, float* hi, float* lo, int kp,
               cudaStream_t stream);
int gemm_presplit_run(int M, int N, int kp, const float* Ah, const float* Al, const float* Bh,
                      const float* Bl, float* C, int ldc, float sa, int lower, int* err,
                      cudaStream_t stream);

// ------------------------------------------------------------ LDLQ sweep
struct SweepArgs {
    const float* Wq;
    const float* Lfac;
    int k, n;
    int nseg;
    const int* seg_c0;       // [nseg + 1] column tiles
    const int* seg_K;
    int16_t* const* seg_trellis;
    int pivot, margin, buf_cols;
    float* hatW;
    float* E;
    float* prod;
    int32_t* states;
    float* xout;
    uint8_t* bp_ws;
    size_t bp_slot;
    float* lazy_ws;          // lazy pipeline: SMs x 2 row regions (lazy_pipeline launches)
    void* split_ws;          // feedback GEMM pre-split operands (null: per-tile split)
    size_t split_bytes;
    int* tickets2;           // ticket counter of launches on the helper stream
    cudaStream_t side;       // helper stream (null: every launch on the caller's)
    cudaEvent_t ev_fork, ev_join;
    int nslots;              // backpointer slots (> SM count)
    int* slots;              // [nslots] ownership flags (zero at sweep start)
    int* colprog;            // [tn] finished k-blocks per column (zero at start)
    int* tickets;            // launch ticket counter (zeroed before each launch)
    int* err;                // error word (zero at sweep start)
    double wait_ns;          // bound of every device-side wait of the sweep
    const uint4* const* f2tab;  // [8] per K
    const float* lut32;
    int block_hi, block_lo;  // sweep blocks [block_lo, block_hi)
};
int ldlq_sweep(const SweepArgs& a, cudaStream_t stream);
int ldlq_tile_max_resident_per_sm();
int launch_pack(const int32_t* st, int nt, int K, int16_t* out, cudaStream_t stream);
int launch_unpack(const int16_t* tr, int nt, int K, int32_t* st, cudaStream_t stream);
int launch_decode(const int16_t* tr, int tk, int tn, int K, const float* lut, float* W,
                  cudaStream_t stream);
// Self-check of an encoded column segment (quantize.py:849-853, :958-963):
// adds to *bad the number of weights whose value decoded from the trellis
// [tk][tn][16K] differs from hatW (row pitch ldw floats) and, with states
// (row pitch ld_states tiles of 256), of states unpacked from the trellis
// that differ from the encoder's.
int launch_verify(const int16_t* tr, int tk, int tn, int K, const float* lut,
                  const float* hatW, int ldw, const int32_t* states, int ld_states, int* bad,
                  cudaStream_t stream);
// Wait bound (ns) of the sweep's device-side waits (exl3b_set_wait_limit_ms).
double sweep_wait_ns();
// One-sided block-128 Hadamard (had_left axis 0, had_right axis 1).
int launch_had_axis(const float* X, int rows, int cols, int axis, float* Y,
                    cudaStream_t stream);

}  // namespace exl3b
