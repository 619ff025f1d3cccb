// viterbi.cu -- standalone tail-biting encoder over a batch of sequences.
//
// One 512-thread CTA encodes one sequence (it holds all of the SM's registers,
// so one CTA per SM).  The host launches waves of at most `grid` CTAs
// (grid <= SM count); CTA b of a wave uses backpointer slot b of the
// workspace (256 * BP_ROW bytes), so a workspace of grid slots serves any
// number of sequences.  A persistent per-CTA loop over sequences was
// measured to cost register spills (loop-invariant addresses kept live
// across the sequence loop); one sequence per CTA keeps the encoder
// spill-free.
#include "exl3b_internal.h"
#include "vit_lazy.cuh"
#include "viterbi.cuh"

namespace exl3b {

// Batches of at least two sequences per SM go through the lazy-argmin
// pipeline instead (vit_lazy.cuh): SM-count persistent CTAs, CTA b encoding
// sequences b, b + grid, b + 2 grid, ... two at a time, with two row regions of
// the workspace (Lazy<K>::REGION bytes each).  Its loop state lives in shared
// memory, not in registers.
//
// One CTA of kVT threads writes the pre-paired decode words of every thread.
template <int K>
__global__ void __launch_bounds__(kVT)
build_f2tab_kernel(const __half* __restrict__ lut16, uint4* __restrict__ tab) {
    const int t = threadIdx.x;
    __half2 f2[64];
    vit_load_f<K>(f2, lut16, t);
#pragma unroll
    for (int q = 0; q < 16; ++q) {
        uint4 v;
        v.x = *reinterpret_cast<uint32_t*>(&f2[4 * q + 0]);
        v.y = *reinterpret_cast<uint32_t*>(&f2[4 * q + 1]);
        v.z = *reinterpret_cast<uint32_t*>(&f2[4 * q + 2]);
        v.w = *reinterpret_cast<uint32_t*>(&f2[4 * q + 3]);
        tab[q * kVT + t] = v;
    }
}

int build_f2tab(int K, const __half* lut16, uint4* tab, cudaStream_t stream) {
    switch (K) {
        case 2: build_f2tab_kernel<2><<<1, kVT, 0, stream>>>(lut16, tab); break;
        case 3: build_f2tab_kernel<3><<<1, kVT, 0, stream>>>(lut16, tab); break;
        case 4: build_f2tab_kernel<4><<<1, kVT, 0, stream>>>(lut16, tab); break;
        case 5: build_f2tab_kernel<5><<<1, kVT, 0, stream>>>(lut16, tab); break;
        case 6: build_f2tab_kernel<6><<<1, kVT, 0, stream>>>(lut16, tab); break;
        case 7: build_f2tab_kernel<7><<<1, kVT, 0, stream>>>(lut16, tab); break;
        default: set_error("K=%d outside 2..7", K); return RC_BAD_K;
    }
    note_launch();
    return check_cuda(cudaGetLastError(), "build_f2tab launch") ? RC_DEVICE_ERROR : RC_OK;
}

template <int K>
__global__ void __launch_bounds__(kVT, 1)
tailbite_kernel(const float* __restrict__ X, int pivot, int margin,
                int32_t* __restrict__ states, uint8_t* __restrict__ bp_ws,
                const uint4* __restrict__ f2tab) {
    extern __shared__ __align__(16) char smem[];
    using SM = VitSmem<K>;
    using G = Geo<K>;
    const int t = threadIdx.x;
    const int seq = blockIdx.x;
    __half2 f2[64];
    vit_load_f2tab(f2, f2tab, t);
    float* xs = reinterpret_cast<float*>(smem + SM::OFF_X);
    if (t < 64)
        reinterpret_cast<float4*>(xs)[t] =
            reinterpret_cast<const float4*>(X + (size_t)seq * kSteps)[t];
    __syncthreads();
    uint8_t* bp = bp_ws + (size_t)blockIdx.x * kSteps * G::BP_ROW;
    vit_tailbite<K>(f2, smem, pivot, margin, bp, t);
    if (t < kSteps)
        states[(size_t)seq * kSteps + t] =
            reinterpret_cast<const int32_t*>(smem + SM::OFF_ST)[t];
}

// Single Viterbi pass (quantize.py:218-320 viterbi): T <= 256 targets per
// sequence (row-major X [nseq][T]), optional per-sequence pin `overlap`
// (s_0 >> K and s_{T-1} mod 2^(16-K) both equal to it; values are taken mod
// 2^(16-K)), and optional `back_from` >= 0: backpointers only for steps after
// it, and only the state at step back_from is returned (states [nseq]).
// Otherwise states [nseq][T].  Same trellis step and traceback as the
// tail-biting encoder's passes (vit_pass), one CTA per sequence.
template <int K>
__global__ void __launch_bounds__(kVT, 1)
viterbi_kernel(const float* __restrict__ X, int T, const int32_t* __restrict__ overlap,
               int back_from, int32_t* __restrict__ states, uint8_t* __restrict__ bp_ws,
               const uint4* __restrict__ f2tab) {
    extern __shared__ __align__(16) char smem[];
    using SM = VitSmem<K>;
    using G = Geo<K>;
    const int t = threadIdx.x;
    const int seq = blockIdx.x;
    __half2 f2[64];
    vit_load_f2tab(f2, f2tab, t);
    float* xs = reinterpret_cast<float*>(smem + SM::OFF_X);
    if (t < T) xs[t] = X[(size_t)seq * T + t];
    __syncthreads();
    const int ov = overlap ? (overlap[seq] & (G::SPRE - 1)) : -1;
    uint8_t* bp = bp_ws + (size_t)blockIdx.x * kSteps * G::BP_ROW;
    int32_t* st = reinterpret_cast<int32_t*>(smem + SM::OFF_ST);
    const int s = vit_pass<K>(f2, smem, 0, T, ov, back_from < 0 ? 0 : back_from,
                              back_from < 0 ? st : nullptr, bp, t);
    if (back_from < 0) {
        if (t < T) states[(size_t)seq * T + t] = st[t];
    } else if (t == 0) {
        states[seq] = s;
    }
}


template <int K>
__global__ void __launch_bounds__(kLazyThreads, 1)
tailbite_lazy_kernel(const float* __restrict__ X, int nseq, int pivot, int margin,
                     int32_t* __restrict__ states, float* __restrict__ regions,
                     const uint4* __restrict__ f2tab, const float* __restrict__ lut32) {
    extern __shared__ __align__(16) char smem[];
    using SM = LazySmem<K>;
    using L = Lazy<K>;
    const int t = threadIdx.x;
    __half2 f2[64];
    vit_load_f2tab(f2, f2tab, t < kVT ? t : 0);
    float* xs = reinterpret_cast<float*>(smem + SM::OFF_X);
    int32_t* st = reinterpret_cast<int32_t*>(smem + SM::OFF_ST);
    volatile TbJob* jb = reinterpret_cast<volatile TbJob*>(smem + SM::OFF_JOB);
    // pending pass-2 traceback of the previous pair's B: have, seq, s_pivot, s_255
    volatile int* ctl = reinterpret_cast<volatile int*>(smem + SM::OFF_RED + 224);
    float* reg0 = regions + (size_t)(2 * blockIdx.x) * (L::REGION / 4);
    float* reg1 = reg0 + L::REGION / 4;
    const int n1 = (margin > 0 && pivot + margin < kSteps) ? pivot + margin : kSteps;
    const int nmine = nseq > (int)blockIdx.x ? (nseq - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    if (t == 0) {
        jb->active = 0;
        ctl[0] = 0;
    }
    __syncthreads();
    for (int k = 0; k < nmine; k += 2) {
        const int seqA = blockIdx.x + k * gridDim.x;
        const bool hasB = k + 1 < nmine;
        // ---- phase a: F1(A) | T2(previous B)
        if (t < 64)
            reinterpret_cast<float4*>(xs)[t] =
                reinterpret_cast<const float4*>(X + (size_t)seqA * kSteps)[t];
        if (t == 0 && ctl[0])
            tb_job_start<K>(smem, reg1, 1, 1, 0, ctl[2] >> K, 0, kSteps - 1, ctl[3]);
        __syncthreads();
        const int fA1 = lazy_pass<K>(f2, smem, 0, pivot, n1, -1, pivot, reg0, nullptr, lut32, t);
        tb_job_drain<K>(smem, lut32, t);
        if (ctl[0] && t < kSteps) states[(size_t)ctl[1] * kSteps + t] = st[kSteps + t];
        __syncthreads();
        // ---- phase b: F1(B) | T1(A)
        if (hasB && t < 64)
            reinterpret_cast<float4*>(xs + kSteps)[t] =
                reinterpret_cast<const float4*>(X + (size_t)(seqA + gridDim.x) * kSteps)[t];
        if (t == 0) tb_job_start<K>(smem, reg0, 0, 0, pivot, -1, pivot, n1 - 1, fA1);
        __syncthreads();
        int fB1 = 0;
        if (hasB) fB1 = lazy_pass<K>(f2, smem, 1, pivot, n1, -1, pivot, reg1, nullptr, lut32, t);
        tb_job_drain<K>(smem, lut32, t);
        const int spA = jb->result;
        __syncthreads();
        // ---- phase c: F2(A) | T1(B)
        if (hasB && t == 0) tb_job_start<K>(smem, reg1, 1, 0, pivot, -1, pivot, n1 - 1, fB1);
        __syncthreads();
        const int fA2 = lazy_pass<K>(f2, smem, 0, 0, kSteps, spA >> K, 0, reg0, &st[kSteps - 1],
                                     lut32, t);
        tb_job_drain<K>(smem, lut32, t);
        const int spB = hasB ? jb->result : 0;
        __syncthreads();
        // ---- phase d: F2(B) | T2(A)
        if (t == 0) tb_job_start<K>(smem, reg0, 0, 1, 0, spA >> K, 0, kSteps - 1, fA2);
        __syncthreads();
        int fB2 = 0;
        if (hasB)
            fB2 = lazy_pass<K>(f2, smem, 1, 0, kSteps, spB >> K, 0, reg1, &st[2 * kSteps - 1],
                               lut32, t);
        tb_job_drain<K>(smem, lut32, t);
        if (t < kSteps) states[(size_t)seqA * kSteps + t] = st[t];
        if (t == 0) {
            ctl[0] = hasB ? 1 : 0;
            ctl[1] = seqA + gridDim.x;
            ctl[2] = spB;
            ctl[3] = fB2;
        }
        __syncthreads();
    }
    if (ctl[0]) {
        if (t == 0) tb_job_start<K>(smem, reg1, 1, 1, 0, ctl[2] >> K, 0, kSteps - 1, ctl[3]);
        __syncthreads();
        tb_job_drain<K>(smem, lut32, t);
        if (t < kSteps) states[(size_t)ctl[1] * kSteps + t] = st[kSteps + t];
    }
}

size_t bp_slot_bytes(int K) {
    switch (K) {
        case 2: return (size_t)kSteps * Geo<2>::BP_ROW;
        case 3: return (size_t)kSteps * Geo<3>::BP_ROW;
        case 4: return (size_t)kSteps * Geo<4>::BP_ROW;
        case 5: return (size_t)kSteps * Geo<5>::BP_ROW;
        case 6: return (size_t)kSteps * Geo<6>::BP_ROW;
        case 7: return (size_t)kSteps * Geo<7>::BP_ROW;
    }
    return 0;
}

template <int K>
static int launch_k(const float* dX, int nseq, int pivot, int margin,
                    int32_t* dStates, uint8_t* ws, int grid,
                    const uint4* f2tab, cudaStream_t stream) {
    const int smem = VitSmem<K>::BYTES;
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev]) {
        if (check_cuda(cudaFuncSetAttribute(tailbite_kernel<K>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                       "cudaFuncSetAttribute(tailbite)"))
            return RC_DEVICE_ERROR;
        attr_set[dev] = true;
    }
    for (int s0 = 0; s0 < nseq; s0 += grid) {
        const int n = nseq - s0 < grid ? nseq - s0 : grid;
        prof_begin_launch(stream, PROF_TAILBITE, (double)n * kSteps);
        tailbite_kernel<K><<<n, kVT, smem, stream>>>(
            dX + (size_t)s0 * kSteps, pivot, margin, dStates + (size_t)s0 * kSteps,
            ws, f2tab);
        prof_end_launch(stream);
        note_launch();
        if (check_cuda(cudaGetLastError(), "tailbite_kernel launch"))
            return RC_DEVICE_ERROR;
    }
    return RC_OK;
}

template <int K>
static int launch_lazy_k(const float* dX, int nseq, int pivot, int margin, int32_t* dStates,
                         uint8_t* ws, int grid, const uint4* f2tab, const float* lut32,
                         cudaStream_t stream) {
    const int smem = LazySmem<K>::BYTES;
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev]) {
        if (check_cuda(cudaFuncSetAttribute(tailbite_lazy_kernel<K>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                       "cudaFuncSetAttribute(tailbite_lazy)"))
            return RC_DEVICE_ERROR;
        attr_set[dev] = true;
    }
    prof_begin_launch(stream, PROF_TAILBITE, (double)nseq * kSteps);
    tailbite_lazy_kernel<K><<<grid, kLazyThreads, smem, stream>>>(
        dX, nseq, pivot, margin, dStates, reinterpret_cast<float*>(ws), f2tab, lut32);
    prof_end_launch(stream);
    note_launch();
    return check_cuda(cudaGetLastError(), "tailbite_lazy_kernel launch") ? RC_DEVICE_ERROR
                                                                       : RC_OK;
}

template <int K>
static int launch_viterbi_k(const float* dX, int nseq, int T, const int32_t* dOverlap,
                            int back_from, int32_t* dStates, uint8_t* ws, int grid,
                            const uint4* f2tab, cudaStream_t stream) {
    const int smem = VitSmem<K>::BYTES;
    static bool attr_set[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr_set[dev]) {
        if (check_cuda(cudaFuncSetAttribute(viterbi_kernel<K>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                       "cudaFuncSetAttribute(viterbi)"))
            return RC_DEVICE_ERROR;
        attr_set[dev] = true;
    }
    const size_t per_seq = back_from < 0 ? (size_t)T : 1;
    for (int s0 = 0; s0 < nseq; s0 += grid) {
        const int n = nseq - s0 < grid ? nseq - s0 : grid;
        viterbi_kernel<K><<<n, kVT, smem, stream>>>(
            dX + (size_t)s0 * T, T, dOverlap ? dOverlap + s0 : nullptr, back_from,
            dStates + (size_t)s0 * per_seq, ws, f2tab);
        note_launch();
        if (check_cuda(cudaGetLastError(), "viterbi_kernel launch")) return RC_DEVICE_ERROR;
    }
    return RC_OK;
}

int launch_viterbi(const float* dX, int nseq, int T, int K, const int32_t* dOverlap,
                   int back_from, int32_t* dStates, uint8_t* ws, int grid,
                   const uint4* f2tab, cudaStream_t stream) {
    switch (K) {
        case 2: return launch_viterbi_k<2>(dX, nseq, T, dOverlap, back_from, dStates, ws, grid, f2tab, stream);
        case 3: return launch_viterbi_k<3>(dX, nseq, T, dOverlap, back_from, dStates, ws, grid, f2tab, stream);
        case 4: return launch_viterbi_k<4>(dX, nseq, T, dOverlap, back_from, dStates, ws, grid, f2tab, stream);
        case 5: return launch_viterbi_k<5>(dX, nseq, T, dOverlap, back_from, dStates, ws, grid, f2tab, stream);
        case 6: return launch_viterbi_k<6>(dX, nseq, T, dOverlap, back_from, dStates, ws, grid, f2tab, stream);
        case 7: return launch_viterbi_k<7>(dX, nseq, T, dOverlap, back_from, dStates, ws, grid, f2tab, stream);
    }
    set_error("K=%d outside 2..7", K);
    return RC_BAD_K;
}

size_t lazy_region_bytes(int K) {
    switch (K) {
        case 2: return Lazy<2>::REGION;
        case 3: return Lazy<3>::REGION;
        case 4: return Lazy<4>::REGION;
        case 5: return Lazy<5>::REGION;
        case 6: return Lazy<6>::REGION;
        case 7: return Lazy<7>::REGION;
    }
    return 0;
}

TailbitePlan tailbite_plan(int nseq, int K, int sms) {
    TailbitePlan p;
    p.lazy = lazy_pipeline(K, nseq, sms);
    p.grid = p.lazy ? sms : (nseq < sms ? nseq : sms);
    p.bytes = p.lazy ? (size_t)p.grid * 2 * lazy_region_bytes(K)
                     : (size_t)p.grid * bp_slot_bytes(K);
    return p;
}

int launch_tailbite(const float* dX, int nseq, int K, int pivot, int margin,
                    int32_t* dStates, uint8_t* ws, const TailbitePlan& plan,
                    const uint4* f2tab, const float* lut32, cudaStream_t stream) {
    const int grid = plan.grid;
    if (plan.lazy) {
        switch (K) {
            case 2: return launch_lazy_k<2>(dX, nseq, pivot, margin, dStates, ws, grid, f2tab, lut32, stream);
            case 3: return launch_lazy_k<3>(dX, nseq, pivot, margin, dStates, ws, grid, f2tab, lut32, stream);
            case 4: return launch_lazy_k<4>(dX, nseq, pivot, margin, dStates, ws, grid, f2tab, lut32, stream);
            case 5: return launch_lazy_k<5>(dX, nseq, pivot, margin, dStates, ws, grid, f2tab, lut32, stream);
            case 6: return launch_lazy_k<6>(dX, nseq, pivot, margin, dStates, ws, grid, f2tab, lut32, stream);
            case 7: return launch_lazy_k<7>(dX, nseq, pivot, margin, dStates, ws, grid, f2tab, lut32, stream);
        }
    }
    switch (K) {
        case 2: return launch_k<2>(dX, nseq, pivot, margin, dStates, ws, grid, f2tab, stream);
        case 3: return launch_k<3>(dX, nseq, pivot, margin, dStates, ws, grid, f2tab, stream);
        case 4: return launch_k<4>(dX, nseq, pivot, margin, dStates, ws, grid, f2tab, stream);
        case 5: return launch_k<5>(dX, nseq, pivot, margin, dStates, ws, grid, f2tab, stream);
        case 6: return launch_k<6>(dX, nseq, pivot, margin, dStates, ws, grid, f2tab, stream);
        case 7: return launch_k<7>(dX, nseq, pivot, margin, dStates, ws, grid, f2tab, stream);
    }
    set_error("K=%d outside 2..7", K);
    return RC_BAD_K;
}

}  // namespace exl3b
