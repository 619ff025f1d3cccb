// noalloc.cu -- a tail-biting trellis encoder entry point that allocates no
// device memory (exl3b_tailbite_noalloc).
//
// Who needs it: callers that must not allocate device memory while they run.
// Examples are a process whose GPU memory is owned by another allocator (an
// inference server that reserves the device's memory at start-up and treats
// any later cudaMalloc as a failure), or a tight loop that cannot take the
// device-wide synchronisation that cudaMalloc / cudaFree can cause.
// exl3b_tailbite may allocate: its library-owned workspace grows on demand,
// and first use on a device uploads the decode tables.
//
// How: the encoder's backpointer scratch (one 256-step slot per sequence) lives
// in a fixed file-scope device array of kNoAllocScratchBytes (64 MiB).  The CUDA
// runtime creates that array when it loads this library's device code on a GPU,
// and the GPU keeps it until the process exits.  With lazy module loading (the
// default since CUDA 12.2, CUDA_MODULE_LOADING=LAZY) that load happens inside
// the first call on each device -- the cudaGetSymbolAddress of the set-up --
// so that first call does take 64 MiB of device memory; with eager loading
// every context that loads the library takes it at start-up, whether or not it
// ever calls this entry point.  Callers that reserve the device's memory
// should make one warm-up call per device first.  The decode values
// are computed in the kernel from the code formulas instead of being read from
// device tables, so no table has to be allocated either.  The caller passes the
// targets and the output states, as for exl3b_tailbite.
//
// Limits and rules (also in include/exl3b200.h):
//  * at most kNoAllocScratchBytes / (256 steps x backpointer row) sequences per
//    call: 64 for K = 2, 3; 128 for K = 4, 5; 256 for K = 6; 512 for K = 7.
//    Larger requests are rejected with EXL3B_BAD_NSEQ and a message giving the
//    limit; callers with more sequences make several calls.
//  * every call on a device uses the same scratch array.  Calls whose kernels
//    overlap on the GPU (other streams, other host threads) race on it; issue
//    them one after another on one stream.  No part of the scratch has to start
//    at zero: each backpointer row is written before it is read within a call.
//  * the first call on each device does the set-up: it looks up the device
//    address of the scratch array (cudaGetSymbolAddress, which under lazy
//    loading also loads the module and so creates the 64 MiB array) and raises
//    the kernels' shared-memory limit.  Make that first call before reserving
//    the device's memory and before any stream capture; later calls allocate
//    nothing.
#include <mutex>

#include "exl3b_internal.h"
#include "viterbi.cuh"
#include "../../include/exl3b200.h"

namespace exl3b {

constexpr size_t kNoAllocScratchBytes = (size_t)64 << 20;

// Backpointer scratch shared by every exl3b_tailbite_noalloc call on a device.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Decode value of state s under code id `code` (quantize.py:56-87), computed in
// fp32: each table entry is an exact fp32 value rounded once to fp16, so this
// equals the host-built table entry bit for bit.
__device__ __forceinline__ __half code_value(int code, uint32_t s) {
    if (code == CODE_MUL1) {
        const uint32_t x = s * 0x83DCD12Du;
        const uint32_t bs = (x & 0xFFu) + ((x >> 8) & 0xFFu) + ((x >> 16) & 0xFFu) + (x >> 24);
        // fp16 0x1EEE and 0xC931 as fp32; the product and the sum are exact
        const float v = __fadd_rn(__fmul_rn((float)(1024u + bs), 0.00676727294921875f),
                                  -10.3828125f);
        return __float2half_rn(v);
    }
    uint32_t x = (code == CODE_3INST) ? s * 89226354u + 64248484u : s * 0xCBAC1FEDu;
    x = (x & 0x8FFF8FFFu) ^ 0x3B603B60u;
    const float lo = __half2float(__ushort_as_half((unsigned short)(x & 0xFFFFu)));
    const float hi = __half2float(__ushort_as_half((unsigned short)(x >> 16)));
    return __float2half_rn(lo + hi);   // exact fp32 sum of two fp16 values
}

// This thread's 128 decode values, packed in pairs in the pre-paired table
// layout ([16][kVT] uint4, word r2 in component r2 % 4 of entry (r2/4)*kVT + t),
// written to a shared-memory staging area.  Loading them back like a table
// keeps the step loop exactly as in the table-based encoder (no register
// spills); each thread reads only its own words.
template <int K>
__device__ __forceinline__ void vit_stage_f2(uint4* __restrict__ stage, int code, int t) {
    using G = Geo<K>;
#pragma unroll 1
    for (int q = 0; q < 16; ++q) {
        uint32_t w4[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const int r = 2 * (4 * q + c);                // first state of the pair
            const int e = r / G::NC, w = r % G::NC;
            const uint32_t s0 = (uint32_t)(G::out_j(t, e) + w * G::SPRE);
            const __half2 h = __halves2half2(code_value(code, s0),
                                             code_value(code, s0 + G::SPRE));
            w4[c] = *reinterpret_cast<const uint32_t*>(&h);
        }
        stage[q * kVT + t] = make_uint4(w4[0], w4[1], w4[2], w4[3]);
    }
}

constexpr int kStageBytes = 16 * kVT * 16;   // 128 KB

template <int K>
constexpr int noalloc_smem() {
    return VitSmem<K>::BYTES > kStageBytes ? VitSmem<K>::BYTES : kStageBytes;
}

// One CTA per sequence; CTA b uses scratch slot b.
template <int K>
__global__ void __launch_bounds__(kVT, 1)
tailbite_noalloc_kernel(const float* __restrict__ X, int pivot, int margin, int code,
                        int32_t* __restrict__ states, uint8_t* __restrict__ scratch) {
    extern __shared__ __align__(16) char smem[];
    using SM = VitSmem<K>;
    using G = Geo<K>;
    const int t = threadIdx.x;
    const int seq = blockIdx.x;
    __half2 f2[64];
    vit_stage_f2<K>(reinterpret_cast<uint4*>(smem), code, t);
    vit_load_f2tab(f2, reinterpret_cast<const uint4*>(smem), t);
    __syncthreads();     // the staging area is reused by the encoder below
    float* xs = reinterpret_cast<float*>(smem + SM::OFF_X);
    if (t < 64)
        reinterpret_cast<float4*>(xs)[t] =
            reinterpret_cast<const float4*>(X + (size_t)seq * kSteps)[t];
    __syncthreads();
    uint8_t* bp = scratch + (size_t)blockIdx.x * kSteps * G::BP_ROW;
    vit_tailbite<K>(f2, smem, pivot, margin, bp, t);
    if (t < kSteps)
        states[(size_t)seq * kSteps + t] =
            reinterpret_cast<const int32_t*>(smem + SM::OFF_ST)[t];
}

namespace {

std::mutex g_na_mu;
uint8_t* g_na_ptr[kMaxDevices] = {};

template <int K>
int set_smem_limit() {
    return check_cuda(cudaFuncSetAttribute(tailbite_noalloc_kernel<K>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           noalloc_smem<K>()),
                      "cudaFuncSetAttribute(tailbite_noalloc)");
}

// Once per device, with it current: the scratch array's device address and the
// kernels' shared-memory limit.  Calls no allocating routine itself, but under
// lazy module loading the symbol lookup loads the module, which creates the
// array.
int noalloc_setup(int dev, uint8_t** out) {
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (!g_na_ptr[dev]) {
        void* p = nullptr;
        if (check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch),
                       "cudaGetSymbolAddress(noalloc scratch)"))
            return RC_DEVICE_ERROR;
        if (set_smem_limit<2>() || set_smem_limit<3>() || set_smem_limit<4>() ||
            set_smem_limit<5>() || set_smem_limit<6>() || set_smem_limit<7>())
            return RC_DEVICE_ERROR;
        g_na_ptr[dev] = static_cast<uint8_t*>(p);
    }
    *out = g_na_ptr[dev];
    return RC_OK;
}

template <int K>
void launch_noalloc(const float* dX, int nseq, int pivot, int margin, int code,
                    int32_t* dStates, uint8_t* scratch, cudaStream_t s) {
    tailbite_noalloc_kernel<K><<<nseq, kVT, noalloc_smem<K>(), s>>>(dX, pivot, margin, code,
                                                                    dStates, scratch);
}

}  // namespace
}  // namespace exl3b

using namespace exl3b;

extern "C" int exl3b_tailbite_noalloc(const float* dX, int nseq, int K, int code,
                                      int pivot, int margin, int32_t* dStates,
                                      void* stream) {
    if (K < 2 || K > 7) { set_error("K=%d outside 2..7", K); return RC_BAD_K; }
    if (code < 0 || code > 2) { set_error("code id %d", code); return RC_BAD_REQUEST; }
    if (pivot < 0 || pivot >= kSteps || margin < 0) {
        set_error("pivot=%d margin=%d", pivot, margin);
        return RC_BAD_REQUEST;
    }
    if (!dX || !dStates || ((uintptr_t)dX & 15)) {
        set_error("X must be a 16-byte aligned device pointer");
        return RC_BAD_REQUEST;
    }
    const long long max_seq = (long long)(kNoAllocScratchBytes / bp_slot_bytes(K));
    if (nseq <= 0 || nseq > max_seq) {
        set_error("exl3b_tailbite_noalloc: nseq=%d, but its fixed %zu MiB scratch holds at "
                  "most %lld sequences per call at K=%d; split the batch",
                  nseq, kNoAllocScratchBytes >> 20, max_seq, K);
        return RC_BAD_NSEQ;
    }
    int dev = 0;
    if (check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return RC_NO_DEVICE;
    if (dev < 0 || dev >= kMaxDevices) { set_error("device %d", dev); return RC_BAD_DEVICE; }
    uint8_t* scratch = nullptr;
    int rc = noalloc_setup(dev, &scratch);
    if (rc) return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (K) {
        case 2: launch_noalloc<2>(dX, nseq, pivot, margin, code, dStates, scratch, s); break;
        case 3: launch_noalloc<3>(dX, nseq, pivot, margin, code, dStates, scratch, s); break;
        case 4: launch_noalloc<4>(dX, nseq, pivot, margin, code, dStates, scratch, s); break;
        case 5: launch_noalloc<5>(dX, nseq, pivot, margin, code, dStates, scratch, s); break;
        case 6: launch_noalloc<6>(dX, nseq, pivot, margin, code, dStates, scratch, s); break;
        case 7: launch_noalloc<7>(dX, nseq, pivot, margin, code, dStates, scratch, s); break;
    }
    note_launch();
    return check_cuda(cudaGetLastError(), "tailbite_noalloc_kernel launch") ? RC_DEVICE_ERROR
                                                                            : RC_OK;
}
