// ldlq_lazy.cu -- the LDLQ sweep's tile kernels with the lazy-argmin encoder
// (vit_lazy.cuh): the two-tile pipeline for launches with at least two tiles
// per SM, and a one-tile-per-CTA variant (ldlq_solo_kernel, below) for
// launches whose column tiles do not fill the SMs.
//
// Persistent CTAs (one per SM, 16 forward warps + the traceback warp) take
// tiles by ticket in the same dependency order as the one-tile-per-CTA kernel
// (ldlq.cu) and run them two at a time through the four-phase pipeline:
//     F1(A) | T2(previous B)      -> write back previous B
//     F1(B) | T1(A)
//     F2(A) | T1(B)
//     F2(B) | T2(A)               -> write back A
// Before a tile's feedback the tiles below it in its column must be written
// back.  A CTA never blocks while it holds a tile that is not yet written
// back: if a new A's dependency is not ready after a short spin, the pending
// B is finished first; if B's is not, A is run alone to its end and B becomes
// the next A.  So a blocked CTA holds nothing, every awaited tile belongs to a
// CTA that keeps running, and tickets in dependency order make the waits
// finish (the argument of the one-tile-per-CTA kernel).  Each CTA owns two row
// regions of the workspace (Lazy<K>::REGION bytes each), so no slot pool is
// needed.
#include "ldlq_tile.cuh"
#include "vit_lazy.cuh"

namespace exl3b {

// Scheduling state of a lazy-sweep CTA (shared memory, after LazySmem).
struct LazySched {
    int i[2], c[2], seg[2];   // tile of slot 0 (A) and slot 1 (B)
    int sp[2];                // s_pivot of the slot's tile (pass-1 traceback result)
    int fin[2];               // final pass-2 state of the slot's tile
    int got;                  // the last fetch produced a tile
    int pend;                 // slot 1 holds the previous pair's B, awaiting T2
    int ok;                   // 0: a bounded wait failed, the CTA stops
    int carry;                // slot 0 already holds the next A
    int rdy;                  // the last dependency probe succeeded
};

template <int K>
struct LazyTileSmem {
    static constexpr int OFF_WX = LazySmem<K>::BYTES;           // 1 KB feedback staging
    static constexpr int OFF_GATHER = OFF_WX + 1024;            // feedback rows
    static constexpr int OFF_SCHED = OFF_GATHER + kGatherStageBytes;
    static constexpr int BYTES = OFF_SCHED + (int)((sizeof(LazySched) + 15) / 16 * 16);
    static_assert(BYTES <= 227 * 1024, "shared memory of one CTA");
};

// thread 0: take the next ticket into `slot` (got = 0 when the launch is done)
__device__ __forceinline__ void lazy_fetch(const LdlqTileParams& p, volatile LazySched* sc,
                                           int slot) {
    const int ticket = atomicAdd(p.tickets, 1);
    if (ticket >= p.ntiles) {
        sc->got = 0;
        return;
    }
    int i, c, seg;
    tile_of_ticket(p, ticket, i, c, seg);
    sc->i[slot] = i;
    sc->c[slot] = c;
    sc->seg[slot] = seg;
    sc->got = 1;
}

// thread 0: bounded wait until blocks i+1 .. cur-1 of the slot's column are
// written back (intra-buffer feedback).  On time-out records the failure
// (cause 2, like the one-tile kernel) and clears sc->ok.
__device__ __forceinline__ void lazy_wait_dep(const LdlqTileParams& p, volatile LazySched* sc,
                                              int slot) {
    const int i = sc->i[slot], c = sc->c[slot];
    if (!p.Lfac || i + 1 >= p.cur) return;
    const int need = p.tk - 1 - i;
    const long long t0 = clock64();
    const long long limit = p.wait_cycles;
    int seen;
    while ((seen = ld_acquire(&p.colprog[c])) < need) {
        if (ld_acquire(p.err)) { sc->ok = 0; return; }
        if (clock64() - t0 > limit) {
            if (atomicCAS(p.err, 0, 2) == 0) {
                p.err[1] = -1; p.err[2] = i; p.err[3] = c; p.err[4] = seen;
            }
            sc->ok = 0;
            return;
        }
        __nanosleep(256);
    }
}

// thread 0: is the slot's dependency already written back?  Spins at most
// ~16 us, then answers no (the caller then releases what it holds and waits).
__device__ __forceinline__ int lazy_dep_ready(const LdlqTileParams& p,
                                              const volatile LazySched* sc, int slot) {
    const int i = sc->i[slot], c = sc->c[slot];
    if (!p.Lfac || i + 1 >= p.cur) return 1;
    const int need = p.tk - 1 - i;
    const long long t0 = clock64();
    while (ld_acquire(&p.colprog[c]) < need) {
        if (clock64() - t0 > 32000) return 0;
        __nanosleep(128);
    }
    return 1;
}

// Write back the tile of `slot` from st[slot] and publish it (all threads).
template <int K>
__device__ __forceinline__ void lazy_release(const LdlqTileParams& p, char* smem,
                                             volatile LazySched* sc, int slot, int t) {
    const int32_t* st = reinterpret_cast<const int32_t*>(smem + LazySmem<K>::OFF_ST) + 256 * slot;
    if (t < kVT) tile_writeback<K>(p, sc->i[slot], sc->c[slot], sc->seg[slot], st, t);
    __syncthreads();    // every thread's writes of this tile precede the release
    if (t == 0) {
        __threadfence();
        atomicAdd(&p.colprog[sc->c[slot]], 1);
    }
}

template <int K>
__global__ void __launch_bounds__(kLazyThreads, 1)
ldlq_lazy_kernel(const __grid_constant__ LdlqTileParams p) {
    extern __shared__ __align__(16) char smem[];
    using SM = LazySmem<K>;
    using TS = LazyTileSmem<K>;
    using L = Lazy<K>;
    const int t = threadIdx.x;
    __half2 f2[64];
    vit_load_f2tab(f2, p.f2tab[K], t < kVT ? t : 0);
    float* xs = reinterpret_cast<float*>(smem + SM::OFF_X);
    int32_t* st = reinterpret_cast<int32_t*>(smem + SM::OFF_ST);
    float* wx = reinterpret_cast<float*>(smem + TS::OFF_WX);
    float* gst = reinterpret_cast<float*>(smem + TS::OFF_GATHER);
    volatile TbJob* jb = reinterpret_cast<volatile TbJob*>(smem + SM::OFF_JOB);
    volatile LazySched* sc = reinterpret_cast<volatile LazySched*>(smem + TS::OFF_SCHED);
    float* reg0 = p.lazy_ws + (size_t)(2 * blockIdx.x) * (L::REGION / 4);
    float* reg1 = reg0 + L::REGION / 4;
    const int pivot = p.pivot;
    const int n1 = (p.margin > 0 && pivot + p.margin < kSteps) ? pivot + p.margin : kSteps;
    if (t == 0) {
        jb->active = 0;
        sc->pend = 0;
        sc->ok = 1;
        sc->carry = 0;
    }
    __syncthreads();

    for (;;) {
        // ---- A into slot 0
        if (t == 0) {
            if (sc->carry) {
                sc->i[0] = sc->i[1];
                sc->c[0] = sc->c[1];
                sc->seg[0] = sc->seg[1];
                sc->carry = 0;
                sc->got = 1;
            } else {
                lazy_fetch(p, sc, 0);
            }
        }
        if (t == 0 && sc->got) sc->rdy = lazy_dep_ready(p, sc, 0);
        __syncthreads();
        if (!sc->got) break;
        if (!sc->rdy) {
            // release the pending B before blocking (it may be what A needs)
            if (sc->pend) {
                if (t == 0) tb_job_start<K>(smem, reg1, 1, 1, 0, sc->sp[1] >> K, 0,
                                            kSteps - 1, sc->fin[1]);
                __syncthreads();
                tb_job_drain<K>(smem, p.lut32, t);
                lazy_release<K>(p, smem, sc, 1, t);
                if (t == 0) sc->pend = 0;
            }
            if (t == 0) lazy_wait_dep(p, sc, 0);
            __syncthreads();
            if (!sc->ok) break;
        }
        tile_feedback_gather(p, sc->i[0], sc->c[0], xs, wx, gst, t, kLazyThreads);

        // ---- phase a: F1(A) | T2(previous B)
        if (t == 0 && sc->pend)
            tb_job_start<K>(smem, reg1, 1, 1, 0, sc->sp[1] >> K, 0, kSteps - 1, sc->fin[1]);
        __syncthreads();
        const int fA1 = lazy_pass<K>(f2, smem, 0, pivot, n1, -1, pivot, reg0, nullptr,
                                     p.lut32, t);
        if (sc->pend) {
            lazy_release<K>(p, smem, sc, 1, t);
            if (t == 0) sc->pend = 0;
        }
        // ---- B into slot 1
        if (t == 0) {
            lazy_fetch(p, sc, 1);
            sc->rdy = sc->got ? lazy_dep_ready(p, sc, 1) : 0;
        }
        __syncthreads();
        const bool hasB = sc->got != 0;
        if (!hasB || !sc->rdy) {
            // A alone: T1(A), F2(A), T2(A), write back; a B whose dependency
            // is not ready (it may be A) is carried over as the next A
            if (t == 0) {
                tb_job_start<K>(smem, reg0, 0, 0, pivot, -1, pivot, n1 - 1, fA1);
                if (hasB) sc->carry = 1;
            }
            __syncthreads();
            tb_job_drain<K>(smem, p.lut32, t);
            const int spA = jb->result;
            __syncthreads();
            const int fA2 = lazy_pass<K>(f2, smem, 0, 0, kSteps, spA >> K, 0, reg0,
                                         &st[kSteps - 1], p.lut32, t);
            if (t == 0) tb_job_start<K>(smem, reg0, 0, 1, 0, spA >> K, 0, kSteps - 1, fA2);
            __syncthreads();
            tb_job_drain<K>(smem, p.lut32, t);
            lazy_release<K>(p, smem, sc, 0, t);
            __syncthreads();
            if (!hasB) break;
            continue;
        }
        tile_feedback_gather(p, sc->i[1], sc->c[1], xs + kSteps, wx, gst, t, kLazyThreads);

        // ---- phase b: F1(B) | T1(A)
        if (t == 0) tb_job_start<K>(smem, reg0, 0, 0, pivot, -1, pivot, n1 - 1, fA1);
        __syncthreads();
        const int fB1 = lazy_pass<K>(f2, smem, 1, pivot, n1, -1, pivot, reg1, nullptr,
                                     p.lut32, t);
        if (t == 0) sc->sp[0] = jb->result;
        __syncthreads();
        // ---- phase c: F2(A) | T1(B)
        if (t == 0) tb_job_start<K>(smem, reg1, 1, 0, pivot, -1, pivot, n1 - 1, fB1);
        __syncthreads();
        const int fA2 = lazy_pass<K>(f2, smem, 0, 0, kSteps, sc->sp[0] >> K, 0, reg0,
                                     &st[kSteps - 1], p.lut32, t);
        if (t == 0) sc->sp[1] = jb->result;
        __syncthreads();
        // ---- phase d: F2(B) | T2(A)
        if (t == 0) tb_job_start<K>(smem, reg0, 0, 1, 0, sc->sp[0] >> K, 0, kSteps - 1, fA2);
        __syncthreads();
        const int fB2 = lazy_pass<K>(f2, smem, 1, 0, kSteps, sc->sp[1] >> K, 0, reg1,
                                     &st[2 * kSteps - 1], p.lut32, t);
        lazy_release<K>(p, smem, sc, 0, t);
        if (t == 0) {
            sc->fin[1] = fB2;
            sc->pend = 1;
        }
        __syncthreads();
    }
    // the previous pair's B, if it still waits for its pass-2 traceback
    if (sc->ok && sc->pend) {
        if (t == 0) tb_job_start<K>(smem, reg1, 1, 1, 0, sc->sp[1] >> K, 0, kSteps - 1, sc->fin[1]);
        __syncthreads();
        tb_job_drain<K>(smem, p.lut32, t);
        lazy_release<K>(p, smem, sc, 1, t);
    }
}

// One tile at a time per CTA, for launches whose column tiles do not fill the
// CTAs: there every CTA of the two-tile pipeline holds a lone tile (its next
// tile waits on the one it holds) and runs it through the "A alone" sequence
// above, with the traceback warp's register cap on the forward warps.  Here
// the CTA has the 16 forward warps only -- 128 registers per thread instead
// of 96 -- and warp 0 runs each traceback between the passes while the
// others wait: F1, T1, F2, T2, write-back, next ticket.  The same passes and
// jobs as the pipeline, so the same states.  A CTA that waits for a
// dependency holds no tile, so the ticket argument of the pipeline holds.
template <int K>
__global__ void __launch_bounds__(kVT, 1)
ldlq_solo_kernel(const __grid_constant__ LdlqTileParams p) {
    extern __shared__ __align__(16) char smem[];
    using SM = LazySmem<K>;
    using TS = LazyTileSmem<K>;
    using L = Lazy<K>;
    const int t = threadIdx.x;
    __half2 f2[64];
    vit_load_f2tab(f2, p.f2tab[K], t);
    float* xs = reinterpret_cast<float*>(smem + SM::OFF_X);
    int32_t* st = reinterpret_cast<int32_t*>(smem + SM::OFF_ST);
    float* wx = reinterpret_cast<float*>(smem + TS::OFF_WX);
    float* gst = reinterpret_cast<float*>(smem + TS::OFF_GATHER);
    volatile TbJob* jb = reinterpret_cast<volatile TbJob*>(smem + SM::OFF_JOB);
    volatile LazySched* sc = reinterpret_cast<volatile LazySched*>(smem + TS::OFF_SCHED);
    float* reg0 = p.lazy_ws + (size_t)(2 * blockIdx.x) * (L::REGION / 4);
    const int pivot = p.pivot;
    const int n1 = (p.margin > 0 && pivot + p.margin < kSteps) ? pivot + p.margin : kSteps;
    if (t == 0) {
        jb->active = 0;
        sc->ok = 1;
    }
    __syncthreads();
    for (;;) {
        if (t == 0) {
            lazy_fetch(p, sc, 0);
            if (sc->got) lazy_wait_dep(p, sc, 0);
        }
        __syncthreads();
        if (!sc->got || !sc->ok) break;
        tile_feedback_gather(p, sc->i[0], sc->c[0], xs, wx, gst, t, kVT);
        const int f1 = lazy_pass<K>(f2, smem, 0, pivot, n1, -1, pivot, reg0, nullptr,
                                    p.lut32, t);
        if (t == 0) tb_job_start<K>(smem, reg0, 0, 0, pivot, -1, pivot, n1 - 1, f1);
        __syncthreads();
        if (t < 32) tb_job_run<K>(smem, p.lut32, t);
        __syncthreads();
        const int sp = jb->result;
        __syncthreads();
        const int f2s = lazy_pass<K>(f2, smem, 0, 0, kSteps, sp >> K, 0, reg0,
                                     &st[kSteps - 1], p.lut32, t);
        if (t == 0) tb_job_start<K>(smem, reg0, 0, 1, 0, sp >> K, 0, kSteps - 1, f2s);
        __syncthreads();
        if (t < 32) tb_job_run<K>(smem, p.lut32, t);
        __syncthreads();
        lazy_release<K>(p, smem, sc, 0, t);
        __syncthreads();
    }
}

template <int K>
static int launch_solo_tile_k(const LdlqTileParams& p, unsigned grid, cudaStream_t stream) {
    static bool attr[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev]) {
        if (check_cuda(cudaFuncSetAttribute(ldlq_solo_kernel<K>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            LazyTileSmem<K>::BYTES),
                       "cudaFuncSetAttribute(ldlq_solo)"))
            return RC_DEVICE_ERROR;
        attr[dev] = true;
    }
    ldlq_solo_kernel<K><<<grid, kVT, LazyTileSmem<K>::BYTES, stream>>>(p);
    note_launch();
    return check_cuda(cudaGetLastError(), "ldlq_solo_kernel launch") ? RC_DEVICE_ERROR : RC_OK;
}

int launch_solo_tile(int K, const LdlqTileParams& p, unsigned grid, cudaStream_t stream) {
    switch (K) {
        case 2: return launch_solo_tile_k<2>(p, grid, stream);
        case 3: return launch_solo_tile_k<3>(p, grid, stream);
        case 4: return launch_solo_tile_k<4>(p, grid, stream);
        case 5: return launch_solo_tile_k<5>(p, grid, stream);
        case 6: return launch_solo_tile_k<6>(p, grid, stream);
        case 7: return launch_solo_tile_k<7>(p, grid, stream);
    }
    set_error("solo tile kernel: K=%d outside 2..7", K);
    return RC_BAD_K;
}

template <int K>
static int launch_lazy_tile_k(const LdlqTileParams& p, unsigned grid, cudaStream_t stream) {
    static bool attr[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev]) {
        if (check_cuda(cudaFuncSetAttribute(ldlq_lazy_kernel<K>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            LazyTileSmem<K>::BYTES),
                       "cudaFuncSetAttribute(ldlq_lazy)"))
            return RC_DEVICE_ERROR;
        attr[dev] = true;
    }
    ldlq_lazy_kernel<K><<<grid, kLazyThreads, LazyTileSmem<K>::BYTES, stream>>>(p);
    note_launch();
    return check_cuda(cudaGetLastError(), "ldlq_lazy_kernel launch") ? RC_DEVICE_ERROR : RC_OK;
}

int launch_lazy_tile(int K, const LdlqTileParams& p, unsigned grid, cudaStream_t stream) {
    switch (K) {
        case 2: return launch_lazy_tile_k<2>(p, grid, stream);
        case 3: return launch_lazy_tile_k<3>(p, grid, stream);
        case 4: return launch_lazy_tile_k<4>(p, grid, stream);
        case 5: return launch_lazy_tile_k<5>(p, grid, stream);
        case 6: return launch_lazy_tile_k<6>(p, grid, stream);
        case 7: return launch_lazy_tile_k<7>(p, grid, stream);
    }
    set_error("lazy tile kernel: K=%d outside 2..7", K);
    return RC_BAD_K;
}

}  // namespace exl3b
