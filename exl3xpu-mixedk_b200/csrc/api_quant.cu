// api_quant.cu -- C ABI of the quantizer pipeline (include/exl3b200.h):
// incoherence transforms, Hessian damping and block-LDL factorisation, the
// fused LDLQ + trellis sweep, and bitstream pack / unpack / decode.
#include <string.h>

#include "exl3b_internal.h"
#include "../../include/exl3b200.h"

using namespace exl3b;

namespace {

inline cudaStream_t S(void* s) { return static_cast<cudaStream_t>(s); }

inline size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

int need_device(DeviceState** st) {
    const int rc = device_state(st);
    if (rc) set_error("no usable CUDA device");
    return rc;
}

bool dims128(int a, int b) { return a > 0 && b > 0 && a % 128 == 0 && b % 128 == 0; }

// One two-sided rotation launch, recorded as PROF_ROTATE with its
// algorithmic bytes (read input + write output once).
int had2_profiled(const HadParams& p, cudaStream_t s, double bytes) {
    prof_begin_launch(s, PROF_ROTATE, bytes);
    const int rc = launch_had2(p, s);
    prof_end_launch(s);
    return rc;
}

}  // namespace

extern "C" {

int exl3b_incoherence_fwd(const void* dW, int dtype, int m_out, int k_in,
                          const float* d_row_mul, const float* d_col_mul, float* dWi,
                          double* d_sumsq_parts, void* stream) {
    if (!dims128(m_out, k_in)) {
        set_error("W [%d, %d]: both dims must be multiples of 128", m_out, k_in);
        return RC_BAD_REQUEST;
    }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    HadParams p;
    memset(&p, 0, sizeof(p));
    p.X = dW; p.in_dtype = dtype; p.ldx = k_in; p.trans_in = true;
    p.Y = dWi; p.ldy = m_out; p.trans_out = false;
    p.rows = k_in; p.cols = m_out; p.pre_scale = 1.0f;
    p.pre_r = d_row_mul; p.pre_c = d_col_mul; p.sumsq = d_sumsq_parts;
    return had2_profiled(p, S(stream), (double)m_out * k_in * ((dtype == 0 ? 4 : 2) + 4));
}

int exl3b_incoherence_inv(const float* dWi, int k, int n, const float* d_pre_scale,
                          const float* d_su, const float* d_sv, float* dW, void* stream) {
    if (!dims128(k, n)) {
        set_error("W_inner [%d, %d]: both dims must be multiples of 128", k, n);
        return RC_BAD_REQUEST;
    }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    HadParams p;
    memset(&p, 0, sizeof(p));
    p.X = dWi; p.in_dtype = 0; p.ldx = n; p.trans_in = false;
    p.Y = dW; p.ldy = k; p.trans_out = true;
    p.rows = k; p.cols = n; p.pre_scale = 1.0f; p.pre_scale_dev = d_pre_scale;
    p.mid_r = d_su; p.post_c = d_sv;
    return had2_profiled(p, S(stream), (double)k * n * 8);
}

int exl3b_rotate_hessian(const float* dH, int k, const float* d_su, float* dG,
                         void* stream) {
    if (!dims128(k, k)) {
        set_error("H [%d, %d]: k must be a multiple of 128", k, k);
        return RC_BAD_REQUEST;
    }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    HadParams p;
    memset(&p, 0, sizeof(p));
    p.X = dH; p.in_dtype = 0; p.ldx = k; p.Y = dG; p.ldy = k;
    p.rows = k; p.cols = k; p.pre_scale = 1.0f; p.pre_r = d_su; p.pre_c = d_su;
    return had2_profiled(p, S(stream), (double)k * k * 8);
}

int exl3b_damp_hessian(float* dG, int k, float percdamp, int* d_nonfinite, void* stream) {
    if (k <= 0) { set_error("k=%d", k); return RC_BAD_REQUEST; }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    int rc = launch_damp(dG, k, percdamp, S(stream));
    if (!rc && d_nonfinite) rc = launch_count_nonfinite(dG, (size_t)k * k, d_nonfinite, S(stream));
    return rc;
}

size_t exl3b_channel_scale_workspace_bytes(int m_out, int k_in) {
    if (!dims128(m_out, k_in)) return 0;
    const size_t k = k_in, n = m_out;
    return align256(k * n * 4) + align256(k * (n / 128) * 8) + align256(k * 4) + align256(n * 4);
}

int exl3b_channel_scale_fwd(const void* dW, int dtype, int m_out, int k_in,
                            const float* d_su, const float* d_sv, float* dWi,
                            float* d_su_mag, float* d_sv_mag, float* d_sv_store,
                            double* d_sumsq_parts, void* ws, size_t ws_bytes,
                            void* stream) {
    if (!dims128(m_out, k_in)) {
        set_error("W [%d, %d]: both dims must be multiples of 128", m_out, k_in);
        return RC_BAD_REQUEST;
    }
    if (!ws || ws_bytes < exl3b_channel_scale_workspace_bytes(m_out, k_in)) {
        set_error("channel_scale workspace too small");
        return RC_WORKSPACE;
    }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    const int k = k_in, n = m_out;
    uint8_t* w = static_cast<uint8_t*>(ws);
    float* W1 = reinterpret_cast<float*>(w);
    w += align256((size_t)k * n * 4);
    double* rparts = reinterpret_cast<double*>(w);
    w += align256((size_t)k * (n / 128) * 8);
    float* div_r = reinterpret_cast<float*>(w);
    w += align256((size_t)k * 4);
    float* div_c = reinterpret_cast<float*>(w);
    cudaStream_t s = S(stream);
    // r_out: per-output-channel RMS (W32.square().mean(0).sqrt(), :787)
    int rc = launch_row_rms(dW, dtype, n, k, d_sv_mag, s);
    if (!rc) rc = launch_chan_out(d_sv_mag, d_sv, n, div_c, d_sv_store, s);
    if (rc) return rc;
    // w = had_right(W32 / (sv * r_out))  (:793-794)
    HadParams p;
    memset(&p, 0, sizeof(p));
    p.X = dW; p.in_dtype = dtype; p.ldx = k; p.trans_in = true;
    p.Y = W1; p.ldy = n; p.rows = k; p.cols = n; p.pre_scale = 1.0f;
    p.pre_c_div = div_c; p.skip_left = true; p.row_sumsq = rparts;
    if ((rc = launch_had2(p, s))) return rc;
    // r_in and W_i = had_left(w / (su * r_in))  (:795-799)
    if ((rc = launch_chan_in(rparts, k, n / 128, d_su, d_su_mag, div_r, s))) return rc;
    memset(&p, 0, sizeof(p));
    p.X = W1; p.in_dtype = 0; p.ldx = n; p.Y = dWi; p.ldy = n; p.rows = k; p.cols = n;
    p.pre_scale = 1.0f; p.pre_r_div = div_r; p.skip_right = true; p.sumsq = d_sumsq_parts;
    return launch_had2(p, s);
}

int exl3b_channel_scale_store(const float* d_su, const float* d_su_mag, const float* d_wscale,
                              const float* d_sv, const float* d_sv_store, int k, int n,
                              void* d_suh_f16, void* d_svh_f16, void* stream) {
    if (k <= 0 || n <= 0) { set_error("dims"); return RC_BAD_REQUEST; }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    return launch_chan_store(d_su, d_su_mag, d_wscale, d_sv, d_sv_store, k, n,
                             static_cast<__half*>(d_suh_f16), static_cast<__half*>(d_svh_f16),
                             S(stream));
}

int exl3b_damp_hessian_f64(double* dG, int k, double extra, void* stream) {
    if (k <= 0) { set_error("k=%d", k); return RC_BAD_REQUEST; }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    return launch_damp_f64(dG, k, extra, S(stream));
}

int exl3b_convert_f32_f64(const float* dA, double* dB, size_t n, void* stream) {
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    return launch_f32_to_f64(dA, dB, n, S(stream));
}

int exl3b_transpose_scale(int inverse, const float* dX, int rows_x, int cols_x,
                          const float* d_row_mag, const float* d_col_mag,
                          const float* d_scale, float* dY, double* d_sumsq_parts,
                          void* stream) {
    if (rows_x <= 0 || cols_x <= 0) { set_error("dims"); return RC_BAD_REQUEST; }
    if (inverse && !d_scale) { set_error("inverse transpose needs a scale"); return RC_BAD_REQUEST; }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    return launch_transpose_scale(inverse != 0, dX, rows_x, cols_x, d_row_mag, d_col_mag,
                                  d_scale, dY, d_sumsq_parts, S(stream));
}

int exl3b_rms_scale(const double* d_parts, int nparts, double count, float lut_rms,
                    double* d_tmp, float* d_scale, void* stream) {
    if (nparts <= 0 || count <= 0) { set_error("nparts=%d", nparts); return RC_BAD_REQUEST; }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    return launch_rms_scale(d_parts, nparts, count, lut_rms, d_tmp, d_scale, S(stream));
}

int exl3b_div_scalar(const float* dx, const float* d_s, float* dy, size_t n, void* stream) {
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    return launch_div_scalar(dx, d_s, dy, n, S(stream));
}

size_t exl3b_block_ldl_workspace_bytes(int k, int f64) {
    if (k <= 0 || k % 16) return 0;
    const size_t es = f64 ? 8 : 4;
    // block inverses | status word | (fp32) transposed panel + GEMM error word
    return align256((size_t)(k / 16) * 256 * es) + 256 +
           (f64 ? 0 : align256(ldl_panel_bytes(k)) + 256);
}

// After a failed launch sequence that may have forked work onto the helper
// stream: outside a stream capture, wait until both streams are idle (the
// caller may release the workspace once the call returns); inside a capture,
// where synchronising is not allowed and would invalidate it, join the helper
// stream back into the caller's with the join event instead.  The results of
// these calls are deliberately not checked: the error already recorded is the
// one reported.
static void drain_after_error(cudaStream_t s, DeviceState* st, bool side_used) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) cs = cudaStreamCaptureStatusNone;
    if (cs != cudaStreamCaptureStatusNone) {
        if (side_used && st->side && st->ev_join) {
            (void)cudaEventRecord(st->ev_join, st->side);
            (void)cudaStreamWaitEvent(s, st->ev_join, 0);
        }
        return;
    }
    if (side_used && st->side) (void)cudaStreamSynchronize(st->side);
    (void)cudaStreamSynchronize(s);
}

// The device's high-priority helper stream and its fork / join events,
// created on first use (the block LDL's lookahead, the sweep's concurrent
// segment launches).
static int side_stream(DeviceState* st) {
    if (st->side) return RC_OK;
    int lo_pri = 0, hi_pri = 0;
    cudaDeviceGetStreamPriorityRange(&lo_pri, &hi_pri);
    if (check_cuda(cudaStreamCreateWithPriority(&st->side, cudaStreamNonBlocking, hi_pri),
                   "helper stream") ||
        check_cuda(cudaEventCreateWithFlags(&st->ev_fork, cudaEventDisableTiming),
                   "helper event") ||
        check_cuda(cudaEventCreateWithFlags(&st->ev_join, cudaEventDisableTiming),
                   "helper event"))
        return RC_DEVICE_ERROR;
    return RC_OK;
}

int exl3b_block_ldl(void* dA, int k, int f64, float* dLfac, void* dD, void* ws,
                    size_t ws_bytes, void* stream) {
    if (k <= 0 || k % 16) { set_error("k=%d must be a positive multiple of 16", k); return RC_BAD_REQUEST; }
    if (!ws || ws_bytes < exl3b_block_ldl_workspace_bytes(k, f64)) {
        set_error("block_ldl workspace too small");
        return RC_WORKSPACE;
    }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    const size_t es = f64 ? 8 : 4;
    uint8_t* w = static_cast<uint8_t*>(ws);
    void* dli = w;
    int* status = reinterpret_cast<int*>(w + align256((size_t)(k / 16) * 256 * es));
    float* panel = nullptr;
    int* gerr = nullptr;
    if (!f64) {
        panel = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(status) + 256);
        gerr = reinterpret_cast<int*>(reinterpret_cast<uint8_t*>(panel) +
                                      align256(ldl_panel_bytes(k)));
    }
    cudaStream_t s = S(stream);
    if (check_cuda(cudaMemsetAsync(status, 0, sizeof(int), s), "memset status") ||
        (gerr && check_cuda(cudaMemsetAsync(gerr, 0, sizeof(int), s), "memset gemm status")))
        return RC_DEVICE_ERROR;
    // the lookahead's helper stream and events
    if (!f64 && side_stream(st)) return RC_DEVICE_ERROR;
    prof_begin_launch(s, PROF_LDL, (double)k * k * k / 3.0);
    int rc = f64 ? block_ldl<double>(static_cast<double*>(dA), k, dLfac, static_cast<double*>(dD),
                                     static_cast<double*>(dli), status, s)
                 : block_ldl<float>(static_cast<float*>(dA), k, dLfac, static_cast<float*>(dD),
                                    static_cast<float*>(dli), status, s, panel, gerr, st->side,
                                    st->ev_fork, st->ev_join);
    prof_end_launch(s);
    if (rc) {
        // the lookahead chain may still run on the helper stream: let it end
        // before the caller can release the workspace
        drain_after_error(s, st, !f64);
        return rc;
    }
    int h = 0, g = 0;
    if (check_cuda(cudaMemcpyAsync(&h, status, sizeof(int), cudaMemcpyDeviceToHost, s),
                   "read status") ||
        (gerr && check_cuda(cudaMemcpyAsync(&g, gerr, sizeof(int), cudaMemcpyDeviceToHost, s),
                            "read gemm status")) ||
        check_cuda(cudaStreamSynchronize(s), "block_ldl sync"))
        return RC_DEVICE_ERROR;
    if (g) {
        set_error("block LDL: tensor-core trailing update timed out (%d)", g);
        return RC_DEVICE_ERROR;
    }
    if (h) {
        set_error("Cholesky: leading minor of order %d is not positive-definite", h);
        return RC_NOT_SPD;
    }
    return RC_OK;
}

size_t exl3b_u_to_gram_workspace_bytes(int k) {
    if (k <= 0) return 0;
    return 2 * align256((size_t)k * k * 8);
}

int exl3b_u_to_gram(const float* dU, int k, double* dG, void* ws, size_t ws_bytes, void* stream) {
    if (k <= 0) { set_error("k=%d", k); return RC_BAD_REQUEST; }
    if (!ws || ws_bytes < exl3b_u_to_gram_workspace_bytes(k)) {
        set_error("u_to_gram workspace too small");
        return RC_WORKSPACE;
    }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    double* Ud = static_cast<double*>(ws);
    double* Ui = reinterpret_cast<double*>(static_cast<uint8_t*>(ws) + align256((size_t)k * k * 8));
    return u_to_gram_f64(dU, k, Ud, Ui, dG, S(stream));
}


// ------------------------------------------------------------------ LDLQ
// Workspace: E [k][n] | prod [k][n] (LDLQ only) | backpointer slots |
// control words (slot flags, per-column progress, ticket, error word) |
// lazy-pipeline row regions (SMs x 2 x Lazy<K>::REGION, largest for the
// smallest K of the sweep) | (LDLQ) the feedback GEMM's pre-split operands.
static int sweep_slots() { return device_sms() * ldlq_tile_max_resident_per_sm() + 16; }

static size_t sweep_slot(const int* seg_K, int nseg) {
    size_t m = 0;
    for (int s = 0; s < nseg; ++s) {
        const size_t b = bp_slot_bytes(seg_K[s]);
        m = b > m ? b : m;
    }
    return m;
}

static size_t sweep_ctrl_bytes(int tn) {
    return align256(((size_t)sweep_slots() + (size_t)tn + 24) * sizeof(int));
}

static size_t sweep_lazy_bytes(int kmin) {
    size_t r = 0;                        // the largest region of any K >= kmin
    for (int K = kmin; K <= 7; ++K) r = lazy_region_bytes(K) > r ? lazy_region_bytes(K) : r;
    return align256((size_t)device_sms() * 2 * r);
}

size_t exl3b_ldlq_workspace_bytes(int k, int n, int kmin, int use_ldlq) {
    if (k <= 0 || n <= 0 || k % 16 || n % 16 || kmin < 2 || kmin > 7) return 0;
    const size_t kn = (size_t)k * n * 4;
    const size_t bp = (size_t)sweep_slots() * bp_slot_bytes(kmin);
    return align256(kn) + (use_ldlq ? align256(kn) : 0) + align256(bp) +
           sweep_ctrl_bytes(n / 16) + sweep_lazy_bytes(kmin) +
           (use_ldlq ? align256(gemm_split_bytes(k, n, k)) : 0);
}

int exl3b_ldlq_sweep(const float* dWq, const float* dLfac, int k, int n, int nseg,
                     const int* seg_c0, const int* seg_K, int16_t* const* seg_trellis,
                     int code, int pivot, int margin, int buf_cols, float* dHatW,
                     int32_t* dStates, float* dXout, int block_lo, int block_hi,
                     void* ws, size_t ws_bytes, void* stream) {
    if (k <= 0 || n <= 0 || k % 16 || n % 16) {
        set_error("Wq [%d, %d]: dims must be positive multiples of 16", k, n);
        return RC_BAD_REQUEST;
    }
    if (nseg < 1 || nseg > 8 || !seg_c0 || !seg_K || !seg_trellis) {
        set_error("nseg=%d (1..8 segments)", nseg);
        return RC_BAD_REQUEST;
    }
    const int tk = k / 16, tn = n / 16;
    if (seg_c0[0] != 0 || seg_c0[nseg] != tn) {
        set_error("segments must cover column tiles [0, %d)", tn);
        return RC_BAD_REQUEST;
    }
    int kmin = 8;
    for (int s = 0; s < nseg; ++s) {
        if (seg_K[s] < 2 || seg_K[s] > 7) { set_error("K=%d outside 2..7", seg_K[s]); return RC_BAD_K; }
        if (seg_c0[s + 1] <= seg_c0[s]) { set_error("empty segment %d", s); return RC_BAD_REQUEST; }
        kmin = seg_K[s] < kmin ? seg_K[s] : kmin;
    }
    if (code < 0 || code > 2 || pivot < 0 || pivot >= kSteps || margin < 0 || buf_cols < 16) {
        set_error("code=%d pivot=%d margin=%d buf_cols=%d", code, pivot, margin, buf_cols);
        return RC_BAD_REQUEST;
    }
    if (block_lo < 0 || block_hi > tk || block_lo >= block_hi) {
        set_error("block range [%d, %d) of %d", block_lo, block_hi, tk);
        return RC_BAD_REQUEST;
    }
    const size_t need = exl3b_ldlq_workspace_bytes(k, n, kmin, dLfac != nullptr);
    if (!ws || ws_bytes < need || ((uintptr_t)ws & 255)) {
        set_error("LDLQ workspace %zu < %zu bytes or misaligned", ws_bytes, need);
        return RC_WORKSPACE;
    }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    SweepArgs a;
    memset(&a, 0, sizeof(a));
    const uint4* tabs[8] = {};
    for (int s = 0; s < nseg; ++s) {
        const uint4* t = nullptr;
        const int rc = f2tab_get(st, code, seg_K[s], &t);
        if (rc) return rc;
        tabs[seg_K[s]] = t;
    }
    uint8_t* w = static_cast<uint8_t*>(ws);
    const size_t kn = align256((size_t)k * n * 4);
    a.E = reinterpret_cast<float*>(w);
    w += kn;
    a.prod = dLfac ? reinterpret_cast<float*>(w) : nullptr;
    if (dLfac) w += kn;
    a.nslots = sweep_slots();
    a.bp_slot = sweep_slot(seg_K, nseg);
    a.bp_ws = w;
    w += align256((size_t)a.nslots * bp_slot_bytes(kmin));
    int* ctrl = reinterpret_cast<int*>(w);
    a.lazy_ws = reinterpret_cast<float*>(w + sweep_ctrl_bytes(tn));
    if (dLfac) {
        a.split_ws = w + sweep_ctrl_bytes(tn) + sweep_lazy_bytes(kmin);
        a.split_bytes = align256(gemm_split_bytes(k, n, k));
    }
    a.slots = ctrl;
    a.colprog = ctrl + a.nslots;
    a.tickets = a.colprog + tn;
    a.err = a.tickets + 1;                 // err[0..4]
    a.tickets2 = a.tickets + 8;
    if (nseg > 1) {                        // segments of different K can run side by side
        if (side_stream(st)) return RC_DEVICE_ERROR;
        a.side = st->side;
        a.ev_fork = st->ev_fork;
        a.ev_join = st->ev_join;
    }
    a.Wq = dWq; a.Lfac = dLfac; a.k = k; a.n = n;
    a.nseg = nseg; a.seg_c0 = seg_c0; a.seg_K = seg_K; a.seg_trellis = seg_trellis;
    a.pivot = pivot; a.margin = margin; a.buf_cols = buf_cols;
    a.hatW = dHatW; a.states = dStates; a.xout = dXout;
    a.f2tab = tabs; a.lut32 = st->lut32[code];
    a.block_lo = block_lo; a.block_hi = block_hi;
    a.wait_ns = sweep_wait_ns();
    cudaStream_t s = S(stream);
    if (block_hi == tk) {   // start of a sweep: feedback cache and control words
        if ((dLfac && check_cuda(cudaMemsetAsync(a.prod, 0, (size_t)k * n * 4, s), "memset prod")) ||
            check_cuda(cudaMemsetAsync(ctrl, 0, sweep_ctrl_bytes(tn), s), "memset control"))
            return RC_DEVICE_ERROR;
    }
    int rc = ldlq_sweep(a, s);
    if (rc) {
        // work may still run on the helper stream: nothing of the workspace
        // may be released before it ends
        drain_after_error(s, st, a.side != nullptr);
        return rc;
    }
    // the tile kernels bound every dependency wait; report a time-out
    int err[14] = {};
    if (check_cuda(cudaMemcpyAsync(err, a.err, sizeof(err), cudaMemcpyDeviceToHost, s),
                   "read sweep status") ||
        check_cuda(cudaStreamSynchronize(s), "sweep sync"))
        return RC_DEVICE_ERROR;
    if (err[0]) {
        set_error("LDLQ sweep: tile scheduling failed (%s) at ticket %d, k-block %d, "
                  "column %d, column progress %d; slots held %d of %d, first holders "
                  "%d %d %d %d %d %d %d %d",
                  err[0] == 1 ? "no free backpointer slot" :
                  err[0] == 2 ? "dependency wait timed out" :
                  err[0] == 4 ? "feedback GEMM barrier timed out" :
                  err[0] == 5 ? "traceback row staging wait timed out" : "aborted", err[1], err[2],
                  err[3], err[4], err[13], a.nslots, err[5], err[6], err[7], err[8], err[9],
                  err[10], err[11], err[12]);
        return RC_DEVICE_ERROR;
    }
    return RC_OK;
}

size_t exl3b_feedback_gemm_workspace_bytes(int M, int N, int K) {
    if (M < 0 || N < 0 || K < 0) return 0;
    return 256 + gemm_split_bytes(M, N, K);
}

int exl3b_feedback_gemm(int M, int N, int K, const float* dA_T, int lda, const float* dB,
                        int ldb, float* dC, int ldc, void* ws, size_t ws_bytes, void* stream) {
    if (M < 0 || N < 0 || K < 0 || lda < M || ldb < N || ldc < N) {
        set_error("feedback GEMM dims M=%d N=%d K=%d lda=%d ldb=%d ldc=%d", M, N, K, lda, ldb, ldc);
        return RC_BAD_REQUEST;
    }
    if (!ws || ws_bytes < 256 || ((uintptr_t)ws & 255)) {
        set_error("feedback GEMM needs a 256-byte status workspace");
        return RC_WORKSPACE;
    }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    cudaStream_t s = S(stream);
    int* err = static_cast<int*>(ws);
    if (check_cuda(cudaMemsetAsync(err, 0, sizeof(int), s), "memset gemm status"))
        return RC_DEVICE_ERROR;
    // beyond the status word: the pre-split operand path when it fits
    uint8_t* split = static_cast<uint8_t*>(ws) + 256;
    const size_t split_bytes = ws_bytes - 256;
    int rc = launch_gemm_tn_acc_tc(M, N, K, dA_T, lda, dB, ldb, dC, ldc, err, s, 1.0f, 0,
                                   split_bytes >= gemm_split_bytes(M, N, K) ? split : nullptr,
                                   split_bytes);
    if (rc) return rc;
    int h = 0;
    if (check_cuda(cudaMemcpyAsync(&h, err, sizeof(int), cudaMemcpyDeviceToHost, s),
                   "read gemm status") ||
        check_cuda(cudaStreamSynchronize(s), "gemm sync"))
        return RC_DEVICE_ERROR;
    if (h) {
        set_error("feedback GEMM: a barrier wait timed out");
        return RC_DEVICE_ERROR;
    }
    return RC_OK;
}

int exl3b_verify_trellis(const int16_t* dTrellis, int tk, int tn, int K, int code,
                         const float* dHatW, int ldw, const int32_t* dStates, int ld_states,
                         int* dMismatch, void* stream) {
    if (K < 2 || K > 7) { set_error("K=%d", K); return RC_BAD_K; }
    if (code < 0 || code > 2 || tk < 0 || tn < 0 || ldw < 16 * tn ||
        (dStates && ld_states < tn) || !dTrellis || !dHatW || !dMismatch) {
        set_error("verify: code %d, [%d x %d] tiles, ldw %d, ld_states %d", code, tk, tn,
                  ldw, ld_states);
        return RC_BAD_REQUEST;
    }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    return launch_verify(dTrellis, tk, tn, K, st->lut32[code], dHatW, ldw, dStates, ld_states,
                         dMismatch, S(stream));
}

int exl3b_hadamard_axis(const float* dX, int rows, int cols, int axis, float* dY,
                        void* stream) {
    if (!dX || !dY) { set_error("null matrix"); return RC_BAD_REQUEST; }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    return launch_had_axis(dX, rows, cols, axis, dY, S(stream));
}

int exl3b_pack_states(const int32_t* dStates, int ntiles, int K, int16_t* dOut, void* stream) {
    if (K < 2 || K > 7) { set_error("K=%d", K); return RC_BAD_K; }
    if (ntiles < 0) { set_error("ntiles=%d", ntiles); return RC_BAD_REQUEST; }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    return launch_pack(dStates, ntiles, K, dOut, S(stream));
}

int exl3b_unpack_states(const int16_t* dTrellis, int ntiles, int K, int32_t* dStates,
                        void* stream) {
    if (K < 1 || K > 8) { set_error("K=%d", K); return RC_BAD_K; }
    if (ntiles < 0) { set_error("ntiles=%d", ntiles); return RC_BAD_REQUEST; }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    return launch_unpack(dTrellis, ntiles, K, dStates, S(stream));
}

int exl3b_decode_trellis(const int16_t* dTrellis, int tk, int tn, int K, int code,
                         float* dW, void* stream) {
    if (K < 1 || K > 8) { set_error("K=%d", K); return RC_BAD_K; }
    if (code < 0 || code > 2 || tk < 0 || tn < 0) { set_error("code/dims"); return RC_BAD_REQUEST; }
    DeviceState* st;
    if (need_device(&st)) return RC_NO_DEVICE;
    return launch_decode(dTrellis, tk, tn, K, st->lut32[code], dW, S(stream));
}

}  // extern "C"
