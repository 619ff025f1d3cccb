// api.cu -- C ABI of libexl3b200.so (declared in include/exl3b200.h).
//
// Plain pointers and sizes only.  Every entry point returns an int rc
// (exl3b::Rc) and never aborts; exl3b_last_error() gives the text of the
// last failure on the calling thread.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>
#include <vector>

#include "exl3b_internal.h"
#include "../../include/exl3b200.h"

namespace exl3b {

static thread_local char g_err[512] = "";
static std::mutex g_mu;
static DeviceState g_dev[kMaxDevices];

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
}

int check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return 0;
    set_error("%s: %s", what, cudaGetErrorString(e));
    return 1;
}

// ---------------------------------------------------------------- wait bound
// Bound of the LDLQ sweep's device-side waits (ns); exl3b_set_wait_limit_ms.
static std::atomic<double> g_wait_ns{4.0e9};
double sweep_wait_ns() { return g_wait_ns.load(std::memory_order_relaxed); }

// ---------------------------------------------------------------- accounting
static std::atomic<long long> g_launches{0};
void note_launch(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

struct ProfRec { cudaEvent_t a, b; int kind; double units; };
static std::atomic<bool> g_prof{false};
static std::mutex g_prof_mu;
static std::vector<ProfRec> g_prof_recs;
static ProfRec g_prof_open;

bool prof_on() { return g_prof.load(std::memory_order_relaxed); }

void prof_begin_launch(cudaStream_t s, int kind, double units) {
    if (!prof_on()) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    g_prof_open.kind = kind;
    g_prof_open.units = units;
    cudaEventCreate(&g_prof_open.a);
    cudaEventCreate(&g_prof_open.b);
    cudaEventRecord(g_prof_open.a, s);
}

void prof_end_launch(cudaStream_t s) {
    if (!prof_on()) return;
    std::lock_guard<std::mutex> lk(g_prof_mu);
    cudaEventRecord(g_prof_open.b, s);
    g_prof_recs.push_back(g_prof_open);
}

// ---------------------------------------------------------------- codebooks
// Decode tables of the reference's V=1 codes (quantize.py:56-87).  Every value
// is an fp16 number, which is what lets the encoder hold them packed.
static float half_round(double v) {
    // v is exactly representable in fp32 for every table below, so the
    // fp32 -> fp16 round-to-nearest-even of cuda_fp16 is the exact rounding.
    return __half2float(__float2half_rn((float)v));
}

static double half_bits_to_double(uint16_t b) {
    __half_raw r;
    r.x = b;
    return (double)__half2float(__half(r));
}

int build_code_lut(int code, float* out) {
    if (!out) return RC_BAD_REQUEST;
    for (uint32_t s = 0; s < 65536u; ++s) {
        if (code == CODE_MUL1) {
            const uint32_t x = s * 0x83DCD12Du;
            const uint32_t bsum = (x & 0xFF) + ((x >> 8) & 0xFF) +
                                  ((x >> 16) & 0xFF) + (x >> 24);
            const double h = 1024.0 + (double)bsum;
            out[s] = half_round(h * half_bits_to_double(0x1EEE) +
                                half_bits_to_double(0xC931));
        } else if (code == CODE_3INST || code == CODE_MCG) {
            uint32_t x = (code == CODE_3INST) ? s * 89226354u + 64248484u
                                              : s * 0xCBAC1FEDu;
            x = (x & 0x8FFF8FFFu) ^ 0x3B603B60u;
            const double lo = half_bits_to_double((uint16_t)(x & 0xFFFF));
            const double hi = half_bits_to_double((uint16_t)(x >> 16));
            out[s] = half_round(lo + hi);
        } else {
            set_error("unknown code id %d", code);
            return RC_BAD_REQUEST;
        }
    }
    return RC_OK;
}

// ---------------------------------------------------------------- devices
static int init_device_locked(int dev, DeviceState* st) {
    if (st->ready) return RC_OK;
    int sms = 0;
    if (check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
                   "cudaDeviceGetAttribute"))
        return RC_NO_DEVICE;
    st->sms = sms;
    static float host_lut[65536];
    static __half host_h[65536];
    for (int c = 0; c < 3; ++c) {
        build_code_lut(c, host_lut);
        for (int s = 0; s < 65536; ++s) host_h[s] = __float2half_rn(host_lut[s]);
        if (check_cuda(cudaMalloc(&st->lut16[c], 65536 * sizeof(__half)), "cudaMalloc(lut16)") ||
            check_cuda(cudaMalloc(&st->lut32[c], 65536 * sizeof(float)), "cudaMalloc(lut32)"))
            return RC_ALLOC;
        if (check_cuda(cudaMemcpy(st->lut16[c], host_h, sizeof(host_h), cudaMemcpyHostToDevice),
                       "cudaMemcpy(lut16)") ||
            check_cuda(cudaMemcpy(st->lut32[c], host_lut, sizeof(host_lut), cudaMemcpyHostToDevice),
                       "cudaMemcpy(lut32)"))
            return RC_DEVICE_ERROR;
    }
    st->ready = true;
    return RC_OK;
}

int device_state(DeviceState** out) {
    int dev = 0;
    if (check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return RC_NO_DEVICE;
    if (dev < 0 || dev >= kMaxDevices) {
        set_error("device %d beyond table", dev);
        return RC_BAD_DEVICE;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    const int rc = init_device_locked(dev, &g_dev[dev]);
    if (rc) return rc;
    *out = &g_dev[dev];
    return RC_OK;
}

int f2tab_get(DeviceState* st, int code, int K, const uint4** out) {
    if (code < 0 || code > 2 || K < 2 || K > 7) {
        set_error("code %d / K %d", code, K);
        return RC_BAD_REQUEST;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if (!st->f2tab[code][K]) {
        uint4* tab = nullptr;
        if (check_cuda(cudaMalloc(&tab, 16 * 512 * sizeof(uint4)), "cudaMalloc(f2tab)"))
            return RC_ALLOC;
        int rc = build_f2tab(K, st->lut16[code], tab, 0);
        if (!rc && check_cuda(cudaDeviceSynchronize(), "build_f2tab")) rc = RC_DEVICE_ERROR;
        if (rc) { cudaFree(tab); return rc; }
        st->f2tab[code][K] = tab;
    }
    *out = st->f2tab[code][K];
    return RC_OK;
}

int device_sms() {
    DeviceState* st = nullptr;
    if (device_state(&st)) return 0;
    return st->sms;
}

static int grow(uint8_t** p, size_t* have, size_t want) {
    if (*have >= want) return RC_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *have = 0;
    if (check_cuda(cudaMalloc(p, want), "cudaMalloc(scratch)")) return RC_ALLOC;
    *have = want;
    return RC_OK;
}

}  // namespace exl3b

using namespace exl3b;

// ====================================================================== ABI
extern "C" {

const char* exl3b_last_error(void) { return g_err; }

long long exl3b_launch_count(void) { return g_launches.load(); }

void exl3b_profile_begin(void) {
    std::lock_guard<std::mutex> lk(g_prof_mu);
    for (auto& r : g_prof_recs) { cudaEventDestroy(r.a); cudaEventDestroy(r.b); }
    g_prof_recs.clear();
    g_prof.store(true);
}

int exl3b_profile_end(int kind, double* ms_total, long long* launches, double* units) {
    g_prof.store(false);
    std::lock_guard<std::mutex> lk(g_prof_mu);
    double ms = 0.0, u = 0.0;
    long long n = 0;
    for (auto& r : g_prof_recs) {
        if (r.kind != kind) continue;
        if (check_cuda(cudaEventSynchronize(r.b), "profile sync")) return RC_DEVICE_ERROR;
        float e = 0.0f;
        if (check_cuda(cudaEventElapsedTime(&e, r.a, r.b), "profile elapsed")) return RC_DEVICE_ERROR;
        ms += e;
        u += r.units;
        ++n;
    }
    if (ms_total) *ms_total = ms;
    if (launches) *launches = n;
    if (units) *units = u;
    return RC_OK;
}

int exl3b_abi_version(void) { return EXL3B_ABI_VERSION; }

int exl3b_set_wait_limit_ms(double ms) {
    if (!(ms >= 0.0) || ms > 60000.0) {
        set_error("wait limit %g ms outside [0, 60000]", ms);
        return RC_BAD_REQUEST;
    }
    g_wait_ns.store(ms == 0.0 ? 4.0e9 : ms * 1.0e6);
    return RC_OK;
}

int exl3b_code_lut(int code, float* out65536) { return build_code_lut(code, out65536); }

int exl3b_device_init(int device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        set_error("no CUDA device");
        return RC_NO_DEVICE;
    }
    if (device < 0 || device >= n) {
        set_error("device %d of %d", device, n);
        return RC_BAD_DEVICE;
    }
    if (check_cuda(cudaSetDevice(device), "cudaSetDevice")) return RC_BAD_DEVICE;
    DeviceState* st = nullptr;
    return device_state(&st);
}

size_t exl3b_tailbite_workspace_bytes(int nseq, int K) {
    if (K < 2 || K > 7 || nseq <= 0) return 0;
    return tailbite_plan(nseq, K, device_sms()).bytes;
}

int exl3b_tailbite(const float* dX, int nseq, int K, int code, int pivot,
                   int margin, int32_t* dStates, void* workspace,
                   size_t workspace_bytes, void* stream) {
    if (K < 2 || K > 7) { set_error("K=%d outside 2..7", K); return RC_BAD_K; }
    if (nseq <= 0) { set_error("nseq=%d", nseq); return RC_BAD_NSEQ; }
    if (code < 0 || code > 2) { set_error("code id %d", code); return RC_BAD_REQUEST; }
    if (pivot < 0 || pivot >= kSteps || margin < 0) {
        set_error("pivot=%d margin=%d", pivot, margin);
        return RC_BAD_REQUEST;
    }
    if (!dX || !dStates || ((uintptr_t)dX & 15)) {
        set_error("X must be a 16-byte aligned device pointer");
        return RC_BAD_REQUEST;
    }
    DeviceState* st = nullptr;
    int rc = device_state(&st);
    if (rc) return rc;
    const TailbitePlan plan = tailbite_plan(nseq, K, st->sms);
    const size_t need = plan.bytes;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    if (ws) {
        if (workspace_bytes < need || ((uintptr_t)ws & 255)) {
            set_error("workspace %zu bytes < %zu or not 256-byte aligned",
                      workspace_bytes, need);
            return RC_WORKSPACE;
        }
    } else {
        std::lock_guard<std::mutex> lk(g_mu);
        rc = grow(&st->scratch, &st->scratch_bytes, need);
        if (rc) return rc;
        ws = st->scratch;
    }
    const uint4* tab = nullptr;
    rc = f2tab_get(st, code, K, &tab);
    if (rc) return rc;
    return launch_tailbite(dX, nseq, K, pivot, margin, dStates, ws, plan, tab,
                           st->lut32[code], static_cast<cudaStream_t>(stream));
}

size_t exl3b_viterbi_workspace_bytes(int nseq, int K) {
    if (K < 2 || K > 7 || nseq <= 0) return 0;
    const int sms = device_sms();
    const int grid = nseq < sms ? nseq : sms;
    return (size_t)grid * bp_slot_bytes(K);
}

int exl3b_viterbi(const float* dX, int nseq, int T, int K, int code,
                  const int32_t* dOverlap, int back_from, int32_t* dStates,
                  void* workspace, size_t workspace_bytes, void* stream) {
    if (K < 2 || K > 7) { set_error("K=%d outside 2..7", K); return RC_BAD_K; }
    if (nseq <= 0) { set_error("nseq=%d", nseq); return RC_BAD_NSEQ; }
    if (T < 1 || T > kSteps) {
        set_error("T=%d: a pass covers 1..%d steps", T, kSteps);
        return RC_BAD_REQUEST;
    }
    if (code < 0 || code > 2) { set_error("code id %d", code); return RC_BAD_REQUEST; }
    if (back_from < -1) { set_error("back_from=%d (-1 = none)", back_from); return RC_BAD_REQUEST; }
    if (!dX || !dStates) { set_error("X and states must be device pointers"); return RC_BAD_REQUEST; }
    DeviceState* st = nullptr;
    int rc = device_state(&st);
    if (rc) return rc;
    const int grid = nseq < st->sms ? nseq : st->sms;
    const size_t need = (size_t)grid * bp_slot_bytes(K);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    if (ws) {
        if (workspace_bytes < need || ((uintptr_t)ws & 255)) {
            set_error("workspace %zu bytes < %zu or not 256-byte aligned",
                      workspace_bytes, need);
            return RC_WORKSPACE;
        }
    } else {
        std::lock_guard<std::mutex> lk(g_mu);
        rc = grow(&st->scratch, &st->scratch_bytes, need);
        if (rc) return rc;
        ws = st->scratch;
    }
    const uint4* tab = nullptr;
    rc = f2tab_get(st, code, K, &tab);
    if (rc) return rc;
    return launch_viterbi(dX, nseq, T, K, dOverlap, back_from, dStates, ws, grid, tab,
                          static_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------------
// Drop-in for the reference's ctypes transport (viterbi_esimd.cpp:935-1005):
// same names, argument meaning and return codes.  Host buffers in and out,
// synchronous.  Codes "mul1p" / "mul1" / "mul1t" are the reference's K=4 mul1
// encoders; "ih2x2" (V=2) has no counterpart here and returns 7.
// Env: XTQ_VIT_DEVIDX (device), XTQ_VIT_MAXSEQ (default 4096),
//      XTQ_VIT_MAXBYTES (device-byte cap, default 6 GiB).
static long long env_ll(const char* name, long long dflt) {
    const char* e = getenv(name);
    return e ? atoll(e) : dflt;
}

int xtq_vit_init(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || n <= 0) {
        set_error("xtq_vit_init: no CUDA device");
        return RC_NO_DEVICE;
    }
    const int idx = (int)env_ll("XTQ_VIT_DEVIDX", -1);
    if (idx >= 0) {
        if (idx >= n) {
            fprintf(stderr, "exl3b xtq_vit_init: XTQ_VIT_DEVIDX=%d but only %d CUDA devices\n", idx, n);
            set_error("XTQ_VIT_DEVIDX=%d of %d devices", idx, n);
            return RC_BAD_DEVICE;
        }
        if (check_cuda(cudaSetDevice(idx), "cudaSetDevice")) return RC_NO_DEVICE;
    }
    DeviceState* st = nullptr;
    return device_state(&st) ? RC_NO_DEVICE : RC_OK;
}

static bool g_xtq_ready = false;

int xtq_vit_run(const float* X, int nseq, const char* code, int margin,
                int pivot, int32_t* out) {
    // first use initialises like the reference (`if (!g_q && xtq_vit_init())`)
    if (!g_xtq_ready) {
        if (xtq_vit_init()) return RC_NO_DEVICE;
        g_xtq_ready = true;
    }
    DeviceState* st = nullptr;
    if (device_state(&st)) return RC_NO_DEVICE;
    if (!code || !(strcmp(code, "mul1p") == 0 || strcmp(code, "mul1") == 0 ||
                   strcmp(code, "mul1t") == 0)) {
        set_error("xtq_vit_run: unsupported code '%s'", code ? code : "(null)");
        return RC_BAD_REQUEST;
    }
    if (nseq <= 0 || nseq > env_ll("XTQ_VIT_MAXSEQ", 4096)) {
        fprintf(stderr, "exl3b xtq_vit_run: %d sequences exceed XTQ_VIT_MAXSEQ\n", nseq);
        set_error("nseq %d out of range", nseq);
        return RC_BAD_NSEQ;
    }
    const int K = 4;
    const TailbitePlan plan = tailbite_plan(nseq, K, st->sms);
    const size_t dev_bytes = (size_t)nseq * kSteps * 8 + plan.bytes;
    if ((long long)dev_bytes > env_ll("XTQ_VIT_MAXBYTES", 6LL << 30)) {
        fprintf(stderr, "exl3b xtq_vit_run: %d sequences need more device bytes than XTQ_VIT_MAXBYTES\n", nseq);
        set_error("nseq %d over XTQ_VIT_MAXBYTES", nseq);
        return RC_TOO_MANY_BYTES;
    }
    if (pivot < 0 || pivot >= kSteps || margin < 0) {
        set_error("pivot=%d margin=%d", pivot, margin);
        return RC_BAD_REQUEST;
    }
    const uint4* tab = nullptr;
    int rc = f2tab_get(st, CODE_MUL1, K, &tab);
    if (rc) return rc;
    std::lock_guard<std::mutex> lk(g_mu);
    if ((size_t)nseq > st->stage_seqs) {
        if (st->stageX) cudaFree(st->stageX);
        if (st->stageS) cudaFree(st->stageS);
        st->stageX = nullptr;
        st->stageS = nullptr;
        st->stage_seqs = 0;
        if (cudaMalloc(&st->stageX, (size_t)nseq * kSteps * 4) != cudaSuccess ||
            cudaMalloc(&st->stageS, (size_t)nseq * kSteps * 4) != cudaSuccess) {
            set_error("xtq_vit_run: staging allocation failed");
            return RC_ALLOC;
        }
        st->stage_seqs = (size_t)nseq;
    }
    rc = grow(&st->scratch, &st->scratch_bytes, plan.bytes);
    if (rc) return rc;
    if (check_cuda(cudaMemcpy(st->stageX, X, (size_t)nseq * kSteps * 4,
                              cudaMemcpyHostToDevice), "xtq_vit_run H2D"))
        return RC_DEVICE_ERROR;
    rc = launch_tailbite(st->stageX, nseq, K, pivot, margin, st->stageS,
                         st->scratch, plan, tab, st->lut32[CODE_MUL1], 0);
    if (rc) return rc;
    if (check_cuda(cudaMemcpy(out, st->stageS, (size_t)nseq * kSteps * 4,
                              cudaMemcpyDeviceToHost), "xtq_vit_run D2H"))
        return RC_DEVICE_ERROR;
    return RC_OK;
}

}  // extern "C"
