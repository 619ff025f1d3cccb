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

// ---- tracebacks of the one-tile kernel from staged rows (K = 4)
// No pass uses the best-array ring while a traceback runs.  Thread 32 streams
// the rows the traceback will read, in its order, into the ring with bulk
// copies (this GPU's global memory -> this CTA's shared memory; one "full"
// and one "empty" mbarrier per slot), up to Lazy<K>::RING rows ahead.  Warp 0
// reads each row's candidates from its slot and the decode values from an
// fp16 copy of the code table in shared memory (exact: the decode values are
// fp16 values).  A
// row then costs shared-memory loads and two warp minima instead of a round
// trip to L2 for its 2^K candidates and decode values.  Same candidates, same
// operations, same first-index minimum as tb_job_run.  Measured per k-block
// at 32 column tiles: K = 4 0.664 -> 0.593 ms (128 column tiles: 0.756 ->
// 0.641); K = 3 0.713 -> 0.788 (its 32 KB rows leave two slots, and the
// copies cannot keep ahead), so K = 3 keeps tb_job_run.
#ifndef EXL3B_SOLO_STAGE
#define EXL3B_SOLO_STAGE 1
#endif

template <int K>
struct SoloSmem {
    static constexpr bool STAGE = K == 4 && EXL3B_SOLO_STAGE;
    static constexpr int NR = Lazy<K>::RING;                  // staging slots
    static constexpr int OFF_LUT = (LazyTileSmem<K>::BYTES + 127) / 128 * 128;
    static constexpr int OFF_BAR = OFF_LUT + (STAGE ? 65536 * 2 : 0);
    static constexpr int BYTES = OFF_BAR + (STAGE ? 2 * NR * 8 : 0);
    static_assert(BYTES <= 227 * 1024, "shared memory of one CTA");
    static_assert(NR * Lazy<K>::ROW_BYTES <= LazySmem<K>::OFF_X, "slots inside the ring");
};

__device__ __forceinline__ bool solo_mbar_wait(uint32_t bar, uint32_t parity, long long limit) {
    const long long t0 = clock64();
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
        if (ok) return true;
        if (clock64() - t0 > limit) return false;
    }
}

// thread 32: stage rows r0 - 1 .. max(stop, 1) (running row count g0 at the
// first) into the ring; use u of slot g % NR waits for the release of use
// u - 1.  Returns false if a wait timed out; `issued` counts the copies sent.
template <int K>
__device__ __forceinline__ bool solo_stage_rows(const float* rows, int r0, int stop, char* smem,
                                                uint32_t full0, uint32_t empty0, int g0,
                                                long long limit, int& issued) {
    using G = Geo<K>;
    using L = Lazy<K>;
    constexpr int NR = SoloSmem<K>::NR;
    const uint32_t ring = (uint32_t)__cvta_generic_to_shared(smem + LazySmem<K>::OFF_RING);
    const int n = r0 - max(stop, 1);
    for (int i = 0; i < n; ++i) {
        const int q = r0 - 1 - i, gr = g0 + i, slot = gr % NR;
        if (gr >= NR && !solo_mbar_wait(empty0 + 8 * slot, ((gr / NR) - 1) & 1, limit))
            return false;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                     :: "r"(full0 + 8 * slot), "r"(L::ROW_BYTES) : "memory");
        asm volatile(
            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
            :: "r"(ring + (uint32_t)(slot * L::ROW_BYTES)), "l"(rows + (size_t)q * G::SPRE),
               "r"(L::ROW_BYTES), "r"(full0 + 8 * slot)
            : "memory");
        ++issued;
    }
    return true;
}

// warp 0: the armed traceback job over the staged rows (running row count g0
// at row r0 - 1).  Returns false if a wait timed out.
template <int K>
__device__ __forceinline__ bool solo_traceback(char* smem, const __half* __restrict__ lut16,
                                               int lane, uint32_t full0, uint32_t empty0,
                                               int g0, long long limit) {
    using G = Geo<K>;
    using SM = LazySmem<K>;
    using L = Lazy<K>;
    constexpr int NR = SoloSmem<K>::NR;
    static_assert(G::NC <= 32 && !L::HALF && L::BULK, "one candidate per lane, full rows");
    volatile TbJob* jb = reinterpret_cast<volatile TbJob*>(smem + SM::OFF_JOB);
    const bool want = jb->want_states != 0;
    const int slot0 = jb->slot, rol = jb->rol, overlap = jb->overlap, stop = jb->stop;
    const int r0 = jb->r;
    int s = jb->s;
    __syncwarp();
    const float* xs = reinterpret_cast<const float*>(smem + SM::OFF_X) + 256 * slot0;
    int32_t* st = reinterpret_cast<int32_t*>(smem + SM::OFF_ST) + 256 * slot0;
    const float* ring = reinterpret_cast<const float*>(smem + SM::OFF_RING);
    const float INF = __int_as_float(0x7f800000);
    bool ok = true;
    int r = r0;
    for (; r > stop; --r) {
        const int j = (s & 0xFFFF) >> K;      // states are 16-bit
        const int m = j >> K;
        const int q = r - 1;
        const float x = xs[(q - rol) & 255];
        int slot = 0;
        if (q >= 1) {
            const int gr = g0 + (r0 - 1 - q);
            slot = gr % NR;
            ok = __all_sync(0xffffffffu, solo_mbar_wait(full0 + 8 * slot, (gr / NR) & 1, limit));
            if (!ok) break;
        }
        uint32_t kc = 0xFFFFFFFFu, kw = 0xFFFFFFFFu;
        if (lane < G::NC) {
            const int idx = m + lane * G::P;
            const float b = (q == 0) ? ((overlap < 0 || idx == overlap) ? 0.0f : INF)
                                     : ring[slot * (L::ROW_BYTES / 4) + G::baddr(idx)];
            const float d = __fsub_rn(__half2float(lut16[j + (lane << (16 - K))]), x);
            kc = __float_as_uint(__fadd_rn(__fmul_rn(d, d), b));
            kw = (uint32_t)lane;
        }
        const uint32_t cmin = __reduce_min_sync(0xffffffffu, kc);
        const uint32_t wmin = __reduce_min_sync(0xffffffffu, kc == cmin ? kw : 0xFFFFFFFFu);
        if (q >= 1) {
            // this lane's reads of the slot precede the next copy into it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];"
                             :: "r"(empty0 + 8 * slot) : "memory");
        }
        s = j + ((int)wmin << (16 - K));
        if (want && lane == 0) st[q] = s;
    }
    __syncwarp();
    if (lane == 0) {
        jb->r = r;
        jb->s = s;
        jb->active = 0;
        jb->result = s;
    }
    __syncwarp();
    return ok;
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
    using SS = SoloSmem<K>;
    __half* lut16 = reinterpret_cast<__half*>(smem + SS::OFF_LUT);
    const uint32_t full0 = (uint32_t)__cvta_generic_to_shared(smem + SS::OFF_BAR);
    const uint32_t empty0 = full0 + 8 * SS::NR;
    int g = 0;                  // rows staged so far (every thread keeps the count)
    if (t == 0) {
        jb->active = 0;
        sc->ok = 1;
        if (SS::STAGE) {
            for (int i = 0; i < 2 * SS::NR; ++i)
                asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" :: "r"(full0 + 8 * i)
                             : "memory");
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        }
    }
    if (SS::STAGE)
        for (int i = t; i < 65536; i += kVT) lut16[i] = __float2half_rn(p.lut32[i]);
    __syncthreads();
    // one traceback job (armed by thread 0 before the call's barrier): warp 0
    // over staged rows with thread 32 staging them, or warp 0 alone
    auto traceback = [&](bool& fail) {
        if constexpr (SS::STAGE) {
            const int r0 = jb->r, stop = jb->stop;
            const float* rows = jb->rows;
            int issued = 0;
            bool ok = true;
            if (t < 32)
                ok = solo_traceback<K>(smem, lut16, t, full0, empty0, g, p.wait_cycles);
            else if (t == 32)
                ok = solo_stage_rows<K>(rows, r0, stop, smem, full0, empty0, g, p.wait_cycles,
                                        issued);
            fail = __syncthreads_or(!ok) != 0;
            if (fail && t == 32) {
                // the copies still in flight land before the CTA leaves
                for (int i = issued > SS::NR ? issued - SS::NR : 0; i < issued; ++i)
                    solo_mbar_wait(full0 + 8 * ((g + i) % SS::NR), ((g + i) / SS::NR) & 1,
                                   p.wait_cycles);
                if (atomicCAS(p.err, 0, 5) == 0) {
                    p.err[1] = -1; p.err[2] = sc->i[0]; p.err[3] = sc->c[0]; p.err[4] = r0;
                }
            }
            g += max(0, r0 - max(stop, 1));
        } else {
            if (t < 32) tb_job_run<K>(smem, p.lut32, t);
            fail = false;
        }
        __syncthreads();
    };
    for (;;) {
        if (t == 0) {
            lazy_fetch(p, sc, 0);
            if (sc->got) lazy_wait_dep(p, sc, 0);
        }
        __syncthreads();
        if (!sc->got || !sc->ok) break;
        tile_feedback_gather(p, sc->i[0], sc->c[0], xs, wx, gst, t, kVT);
        bool fail = false;
        const int f1 = lazy_pass<K>(f2, smem, 0, pivot, n1, -1, pivot, reg0, nullptr,
                                    p.lut32, t);
        // the pass's generic writes to the ring precede the staging copies
        if (SS::STAGE) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (t == 0) tb_job_start<K>(smem, reg0, 0, 0, pivot, -1, pivot, n1 - 1, f1);
        __syncthreads();
        traceback(fail);
        if (fail) break;
        const int sp = jb->result;
        __syncthreads();
        const int f2s = lazy_pass<K>(f2, smem, 0, 0, kSteps, sp >> K, 0, reg0,
                                     &st[kSteps - 1], p.lut32, t);
        if (SS::STAGE) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        if (t == 0) tb_job_start<K>(smem, reg0, 0, 1, 0, sp >> K, 0, kSteps - 1, f2s);
        __syncthreads();
        traceback(fail);
        if (fail) break;
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
                                            SoloSmem<K>::BYTES),
                       "cudaFuncSetAttribute(ldlq_solo)"))
            return RC_DEVICE_ERROR;
        attr[dev] = true;
    }
    ldlq_solo_kernel<K><<<grid, kVT, SoloSmem<K>::BYTES, stream>>>(p);
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
