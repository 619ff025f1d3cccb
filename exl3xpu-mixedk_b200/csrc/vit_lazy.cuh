// vit_lazy.cuh -- tail-biting Viterbi with the argmin taken lazily.
//
// Same trellis, costs and results as vit_tailbite (viterbi.cuh), bit for bit:
// only where each step's predecessor choice is decided changes.
//
//  * Forward passes keep the minimum only (the "untraced" ACS: two
//    subtractions, one packed square, one packed add, one three-input min per
//    predecessor pair -- about half the work of tracking the argmin).  Every
//    step the traceback will cross is kept as a row of the tile's row region
//    in global memory (row q = best_q), in one of two ways (Lazy<K>::BULK):
//    - K <= 4 (rows of 16 to 64 KB): the best arrays rotate through a ring
//      in shared memory (Lazy<K>::RING arrays), and each time half a ring of
//      rows is complete one thread copies them, as they lie there (the
//      Geo<K>::baddr layout), with one TMA bulk store.  The forward threads
//      issue no global stores, so the per-step barrier never waits for
//      global writes to be acknowledged, and the proxy fence that hands their
//      shared-memory writes to the copy engine is paid once per batch.
//    - K >= 5 (rows of 8 KB and less): each thread stores its outputs of the
//      step to the row itself (natural index order, one or two vector
//      stores), which measured faster there than the copy engine.
//    The end state of a pass (the first-index argmin over the last step's
//    costs) is found by rescanning only the group(s) that reach the minimum.
//  * The traceback recomputes, for the one group j = s >> K on the path, the
//    2^K candidate costs cost_{r-1}(j + w 2^(16-K)) = fl(fl(f - x)^2) + best_{r-1}
//    from the stored row with the same fp32 operations as the forward step,
//    and takes their lexicographic (cost, w) minimum: the first-index argmin
//    the forward pass would have recorded.
//  * The traceback is a small state machine in shared memory that a 17th
//    warp (the "job warp", threads kVT .. kVT + 31) runs during a forward pass
//    of ANOTHER tile.  The 16 forward warps synchronise their steps on a named
//    barrier of their own, so the job warp never waits for them nor they for
//    it: it reads only completed rows of its own tile, and its serial latency
//    (fetch, cost, warp reduction per row) stays off the forward critical
//    path.  The two meet again at the end of the pass.  A CTA therefore keeps
//    two tiles in flight and runs them in four phases per pair (F = forward
//    pass, T = traceback; pass 2 needs pass 1's traceback, the write-back
//    needs pass 2's):
//        F1(A) | T2(previous B)
//        F1(B) | T1(A)
//        F2(A) | T1(B)
//        F2(B) | T2(A)
//    A phase ends when both its forward pass and its traceback are done.
//  * Rows are 2^(18-K) bytes per step (K = 2: 64 KB, K = 4: 16 KB, K = 7:
//    2 KB).  At K = 2 the row writes approach HBM bandwidth and bound the
//    forward pass; every K still runs faster than with the tracked encoder.
#pragma once
#include "viterbi.cuh"

namespace exl3b {

constexpr int kLazyThreads = kVT + 32;   // 16 forward warps + the job warp

#ifndef EXL3B_LAZY_RING_KB
#define EXL3B_LAZY_RING_KB 64    // shared memory of the best-array ring
#endif

template <int K>
struct Lazy {
    using G = Geo<K>;
    static constexpr int ROW_BYTES = G::SPRE * 4;                 // one best array
    static constexpr int NPL = G::NC > 32 ? G::NC / 32 : 1;       // candidates per lane
    // rows by TMA bulk store from a shared-memory ring (else by the threads)
    static constexpr bool BULK = K <= 4;
    // K = 2 (64 KB rows, whose writes bound the pass at the HBM rate): only
    // the even rows are stored (row q at q / 2); the traceback rebuilds the 4
    // entries it needs of an odd row q from row q - 1 with the forward step's
    // fp32 operations (16 candidates over the job warp's lanes).  Measured on
    // the standalone encoder at 20 tiles per SM: K = 2 0.723 -> 0.593 ms per
    // tile-slot; the same scheme at K = 3 (64 candidates) and K = 4 (256)
    // measured 2% and 20% slower: their rows cost less than the longer
    // traceback.
#ifndef EXL3B_LAZY_HALF_ROWS
#define EXL3B_LAZY_HALF_ROWS 1
#endif
    static constexpr bool HALF = K == 2 && EXL3B_LAZY_HALF_ROWS;
    static constexpr int ROWS = HALF ? kSteps / 2 : kSteps - 1;   // row slots (q <= 254)
    static constexpr size_t REGION = (size_t)ROWS * ROW_BYTES;    // bytes per tile region
    // half-row rebuild: (w, w') candidate pairs, per lane, lanes per w
    static constexpr int PAIRS = G::NC * G::NC;
    static constexpr int CPL = PAIRS > 32 ? PAIRS / 32 : 1;
    static constexpr int GL = PAIRS <= 32 ? G::NC : (G::NC < 32 ? 32 / G::NC : 1);
    // the ring of best arrays (64 KB: K = 2: 2, K = 3: 2, K = 4: 4; two when
    // the threads store the rows) and the rows per bulk copy (half the ring,
    // aligned: a batch's arrays are adjacent)
    static constexpr int RING_FIT = (EXL3B_LAZY_RING_KB * 1024) / ROW_BYTES;
    static constexpr int RING = (BULK && RING_FIT > 2) ? RING_FIT : 2;
    static constexpr int BATCH = RING / 2;
    // a row is the shared-memory image of one best array, unpadded
    static_assert(VitSmem<K>::B_BYTES == ROW_BYTES, "row = smem best array");
    static_assert(ROW_BYTES % 16 == 0, "bulk copies move multiples of 16 bytes");
    static_assert(RING >= 2 && (RING & (RING - 1)) == 0, "ring of 2^n arrays");
};

// TMA bulk store of one best array (shared -> global, async proxy), its
// bulk-group bookkeeping, and the proxy fences around it.
__device__ __forceinline__ void row_fence_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void row_copy(float* dst, const float* src, int bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;\n\t"
                 "cp.async.bulk.commit_group;"
                 :: "l"(dst), "r"((uint32_t)__cvta_generic_to_shared(src)), "r"(bytes)
                 : "memory");
}
// every issued copy has read its shared-memory source
__device__ __forceinline__ void row_copies_read() {
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// every issued copy is complete in global memory and ordered before this
// thread's later generic-proxy accesses
__device__ __forceinline__ void row_copies_done() {
    asm volatile("cp.async.bulk.wait_group 0;\n\tfence.proxy.async.global;" ::: "memory");
}

// Traceback job state (shared memory; read by all lanes of the job warp,
// written by its lane 0).  r: the next row to resolve (s = s_r known); rows r-1 .. stop are
// read; the job ends with s = s_stop.
struct TbJob {
    const float* rows;   // this tile's row region
    int slot;            // pipeline slot of the tile (its xs / st)
    int want_states;     // pass 2: write every state into st[slot]
    int rol;             // roll of the pass (x of step i = xs[(i - rol) & 255])
    int overlap;         // best_0 = 0 at `overlap` (or everywhere if < 0), +inf elsewhere
    int stop;
    int r;
    int s;
    int pending;         // unused
    int active;
    int result;          // s_stop once done
    int pad;
};

// Shared memory of a lazy-pipeline CTA.
template <int K>
struct LazySmem {
    using G = Geo<K>;
    static constexpr int B_BYTES = VitSmem<K>::B_BYTES;
    static constexpr int OFF_RING = 0;                    // Lazy<K>::RING best arrays
    static constexpr int OFF_X = Lazy<K>::RING * B_BYTES; // xs[2][256] fp32
    static constexpr int OFF_ST = OFF_X + 2048;           // st[2][256] int32
    static constexpr int OFF_RED = OFF_ST + 2048;         // reductions, broadcast words
    static constexpr int OFF_JOB = OFF_RED + 256;         // TbJob
    static constexpr int OFF_EXTRA = OFF_JOB + 64;        // caller-owned tail
    static constexpr int BYTES = OFF_EXTRA;
};

// Run the armed traceback job to its end (the job warp; every lane calls it;
// job state in registers).  Per row r (s = s_r known; group j = s >> K): lane
// w (and w + 32, ... for K >= 6) loads best_{r-1}[(j >> K) + w P] at its
// position in the row (Geo<K>::baddr for bulk-copied rows, natural otherwise;
// L2-coherent loads: other warps or the copy engine wrote the rows) and the
// decode value of predecessor
// j + w 2^(16-K), forms the forward step's cost fl(fl(f - x)^2) + best, and
// the warp takes the lexicographic (cost, w) minimum with two redux.sync
// minima (costs are >= +0 or +inf, so their bit patterns order like the
// floats).  s_{r-1} = j + w* 2^(16-K).  Ends with jb->result = s_stop.
template <int K>
__device__ __forceinline__ void tb_job_run(char* smem, const float* __restrict__ lut32,
                                           int lane) {
    using G = Geo<K>;
    using SM = LazySmem<K>;
    volatile TbJob* jb = reinterpret_cast<volatile TbJob*>(smem + SM::OFF_JOB);
    if (!jb->active) return;
    const float* rows = jb->rows;
    const int slot = jb->slot;
    const bool want = jb->want_states != 0;
    const int rol = jb->rol;
    const int overlap = jb->overlap;
    const int stop = jb->stop;
    int r = jb->r;
    int s = jb->s;
    __syncwarp();
    const float* xs = reinterpret_cast<const float*>(smem + SM::OFF_X) + 256 * slot;
    int32_t* st = reinterpret_cast<int32_t*>(smem + SM::OFF_ST) + 256 * slot;
    const float INF = __int_as_float(0x7f800000);
    using L = Lazy<K>;
    for (; r > stop; --r) {
        const int j = (s & 0xFFFF) >> K;      // states are 16-bit
        const int m = j >> K;
        const int q = r - 1;
        const float* row = rows + (size_t)(L::HALF ? (q >> 1) : q) * G::SPRE;
        const float x = xs[(q - rol) & 255];
        // odd row q of a half-row region: lane group w (GL lanes) rebuilds
        // best_q[m + w P] = min_w' fl(fl(f(s') - x_{q-1})^2) + best_{q-1}[s' >> K],
        // s' = m + w P + w' 2^(16-K), from row q - 1 (the boundary mask when
        // q - 1 = 0); lane w then takes its group's value
        float bh = INF;
        if (L::HALF && (q & 1)) {
            const float xp = xs[(q - 1 - rol) & 255];
            const float* rp = rows + (size_t)((q - 1) >> 1) * G::SPRE;
            const int w = lane / L::GL;
            if (w < G::NC) {
#pragma unroll
                for (int k = 0; k < L::CPL; ++k) {
                    const int sp = m + w * G::P + ((((lane % L::GL) * L::CPL) + k) << (16 - K));
                    const int pi = sp >> K;
                    const float bp = (q == 1) ? ((overlap < 0 || pi == overlap) ? 0.0f : INF)
                                              : __ldcg(rp + G::baddr(pi));
                    const float d = __fsub_rn(__ldg(lut32 + sp), xp);
                    bh = fminf(bh, __fadd_rn(__fmul_rn(d, d), bp));
                }
            }
#pragma unroll
            for (int off = 1; off < L::GL; off <<= 1)
                bh = fminf(bh, __shfl_xor_sync(0xffffffffu, bh, off));
            bh = __shfl_sync(0xffffffffu, bh, (lane < G::NC ? lane : 0) * L::GL);
        }
        uint32_t kc = 0xFFFFFFFFu;      // this lane's best cost bits, first index
        uint32_t kw = 0xFFFFFFFFu;
#pragma unroll
        for (int k = 0; k < L::NPL; ++k) {
            const int w = lane + 32 * k;
            if (w < G::NC) {
                const int idx = m + w * G::P;
                const float b = (q == 0) ? ((overlap < 0 || idx == overlap) ? 0.0f : INF)
                              : (L::HALF && (q & 1)) ? bh
                              : __ldcg(row + (L::BULK ? G::baddr(idx) : idx));
                const float d = __fsub_rn(__ldg(lut32 + j + (w << (16 - K))), x);
                const uint32_t c = __float_as_uint(__fadd_rn(__fmul_rn(d, d), b));
                if (c < kc) { kc = c; kw = (uint32_t)w; }
            }
        }
        const uint32_t cmin = __reduce_min_sync(0xffffffffu, kc);
        const uint32_t wmin = __reduce_min_sync(0xffffffffu, kc == cmin ? kw : 0xFFFFFFFFu);
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
}

// The job warp runs the job to its end; then the whole CTA synchronises.
template <int K>
__device__ __forceinline__ void tb_job_drain(char* smem, const float* __restrict__ lut32,
                                             int t) {
    if (t >= kVT) tb_job_run<K>(smem, lut32, t - kVT);
    __syncthreads();
}

// Arm the job (thread 0; the caller synchronises before the next pass).
template <int K>
__device__ __forceinline__ void tb_job_start(char* smem, const float* rows, int slot,
                                             int want_states, int rol, int overlap, int stop,
                                             int r, int s) {
    using SM = LazySmem<K>;
    TbJob* jb = reinterpret_cast<TbJob*>(smem + SM::OFF_JOB);
    jb->rows = rows;
    jb->slot = slot;
    jb->want_states = want_states;
    jb->rol = rol;
    jb->overlap = overlap;
    jb->stop = stop;
    jb->r = r;
    jb->s = s;
    jb->pending = 0;
    jb->active = 1;
    jb->result = s;
}

// One forward pass of the tile in pipeline slot `slot` (targets xs[slot]):
// untraced steps that store best_q for q in [max(stop, 1), nsteps - 2] to
// `rows`, then the first-index argmin over the end states (pass 2: restricted
// to group `overlap`).  Threads 0 .. kVT-1 run the
// trellis (named barrier 1 between steps); the job warp runs the armed
// traceback job (if any) meanwhile.  Every thread of the CTA (kLazyThreads)
// calls it; both the pass and the job are complete on return.  Returns
// s_{nsteps-1}, and when `st_last` is set stores it there.
template <int K>
__device__ __forceinline__ int lazy_pass(const __half2 (&f2)[64], char* smem, int slot,
                                         int rol, int nsteps, int overlap, int stop,
                                         float* __restrict__ rows, int32_t* st_last,
                                         const float* __restrict__ lut32, int t) {
    using G = Geo<K>;
    using SM = LazySmem<K>;
    using L = Lazy<K>;
    constexpr int BB = SM::B_BYTES / 4;                   // floats per best array
    float* ring = reinterpret_cast<float*>(smem + SM::OFF_RING);
    float* Bc = ring;                                     // best_i: ring slot i % RING
    float* Bn = ring;
    const float* xs = reinterpret_cast<const float*>(smem + SM::OFF_X) + 256 * slot;
    float* redc = reinterpret_cast<float*>(smem + SM::OFF_RED);
    int* reds = reinterpret_cast<int*>(smem + SM::OFF_RED + 64);
    int* bcast = reinterpret_cast<int*>(smem + SM::OFF_RED + 128);
    float* zword = reinterpret_cast<float*>(smem + SM::OFF_RED + 192);
    const float INF = __int_as_float(0x7f800000);
    if (t == 0) *zword = 0.0f;
    if (t < kVT)
        for (int idx = t; idx < G::SPRE; idx += kVT)
            Bc[G::baddr(idx)] = (overlap < 0 || idx == overlap) ? 0.0f : INF;
    __syncthreads();
    float zr;
    asm volatile("ld.volatile.shared.f32 %0, [%1];" : "=f"(zr)
                 : "r"((uint32_t)__cvta_generic_to_shared(zword)));

    // rows the traceback reads: best_q, q in [max(stop, 1), nsteps - 2]
    // (half rows: the even q of [lo & ~1, hi]).
    // Step i writes best_{i+1} into ring slot (i + 1) % RING.  Rows go out in
    // aligned batches of BATCH (rows b BATCH .. b BATCH + BATCH - 1, clipped to
    // [lo, hi]; adjacent slots; half rows: one even row per copy): when step i
    // completes a batch, every thread fences its writes to the async proxy
    // before the step barrier and thread 0 issues one bulk copy after it.  Before every step barrier thread 0
    // waits until the copies issued so far have read their slots; the
    // earliest reuse of a batch's slot is RING - BATCH >= 1 steps after that.
    const int lo = max(stop, 1), hi = nsteps - 2;
    if (t < kVT && !L::BULK) {
        // thread-stored rows; the two buffers alternate.  (Addressing them by
        // step parity measured 3-4% faster than swapping pointers at K = 5, 6
        // and 3% slower at K = 7.)
        Bn = ring + BB;
        for (int i = 0; i < nsteps - 1; ++i) {
            const float x = xs[(i - rol) & 255];
            float* grow = (i + 1 >= lo && i + 1 <= hi) ? rows + (size_t)(i + 1) * G::SPRE
                                                       : nullptr;
            if (K < 7) {
                Bc = ring + (i & 1) * BB;
                Bn = ring + ((i + 1) & 1) * BB;
            }
            vit_step<K, false>(f2, x, Bc, Bn, t, zr, grow);
            if (K == 7) { float* tmp = Bc; Bc = Bn; Bn = tmp; }
            asm volatile("bar.sync 1, %0;" :: "r"(kVT) : "memory");
        }
        Bc = ring + ((nsteps - 1) & 1) * BB;
        Bn = ring + (nsteps & 1) * BB;
    } else if (t < kVT) {
        for (int i = 0; i < nsteps - 1; ++i) {
            const float x = xs[(i - rol) & 255];
            Bc = ring + (i & (L::RING - 1)) * BB;
            Bn = ring + ((i + 1) & (L::RING - 1)) * BB;
            const int q = i + 1;                  // the row this step writes
            vit_step<K, false>(f2, x, Bc, Bn, t, zr);
            // half rows: the even q in [lo & ~1, hi] (q >= 2), one per copy
            const bool flush = L::HALF ? ((q & 1) == 0 && q >= 2 && q >= (lo & ~1) && q <= hi)
                                       : (q >= lo && q <= hi &&
                                          ((q % L::BATCH) == L::BATCH - 1 || q == hi));
            if (flush) row_fence_shared();        // this thread's writes -> async proxy
            if (t == 0) row_copies_read();        // earlier copies have read their slots
            asm volatile("bar.sync 1, %0;" :: "r"(kVT) : "memory");
            if (flush && t == 0) {
                if (L::HALF) {
                    row_copy(rows + (size_t)(q >> 1) * G::SPRE, ring + (q & (L::RING - 1)) * BB,
                             L::ROW_BYTES);
                } else {
                    const int first = max(q - q % L::BATCH, lo);
                    row_copy(rows + (size_t)first * G::SPRE,
                             ring + (first & (L::RING - 1)) * BB,
                             (q - first + 1) * L::ROW_BYTES);
                }
            }
        }
        Bc = ring + ((nsteps - 1) & (L::RING - 1)) * BB;
        Bn = ring + (nsteps & (L::RING - 1)) * BB;
    }
    if (t < kVT) {
        // final step, untraced: best_n[j] = min_w cost_{n-1}(j + w 2^(16-K)).
        // The pass ends at the first-index argmin over cost_{n-1}: the lowest
        // state s = j + w 2^(16-K) whose cost is v* = min_j best_n[j] (pass 2:
        // only group j == overlap).  Each thread rescans the candidates of its
        // groups that reach v* (usually one group in the whole CTA) with the
        // forward step's fp32 operations and takes the group's lexicographic
        // (cost, w) minimum -- its first-index argmin -- and the CTA the lowest
        // such state.
        const float x = xs[(nsteps - 1 - rol) & 255];
        vit_step<K, false>(f2, x, Bc, Bn, t, zr);
        float v = INF;
#pragma unroll
        for (int e = 0; e < G::NOUT; ++e) {
            const int j = G::out_j(t, e);
            if (overlap < 0 || j == overlap) v = fminf(v, Bn[G::baddr(j)]);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
            v = fminf(v, __shfl_xor_sync(0xffffffffu, v, off));
        if ((t & 31) == 0) redc[t >> 5] = v;
        asm volatile("bar.sync 1, %0;" :: "r"(kVT) : "memory");
        float vs = redc[0];
        for (int wv = 1; wv < kVT / 32; ++wv) vs = fminf(vs, redc[wv]);
        int bs = 0x7fffffff;
        for (int e = 0; e < G::NOUT; ++e) {
            const int j = G::out_j(t, e);
            if ((overlap < 0 || j == overlap) && Bn[G::baddr(j)] == vs) {
                const int m = j >> K;
                float gc = INF;
                int gw = 0;
                for (int w = 0; w < G::NC; ++w) {
                    const float d = __fsub_rn(lut32[j + (w << (16 - K))], x);
                    const float c = __fadd_rn(__fmul_rn(d, d), Bc[G::baddr(m + w * G::P)]);
                    if (c < gc) { gc = c; gw = w; }
                }
                bs = min(bs, j + (gw << (16 - K)));
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
            bs = min(bs, __shfl_xor_sync(0xffffffffu, bs, off));
        if ((t & 31) == 0) reds[t >> 5] = bs;
        // the rows are in global memory before the pass ends (the next phase's
        // traceback reads them)
        if (L::BULK && t == 0) row_copies_done();
    } else {
        tb_job_run<K>(smem, lut32, t - kVT);
    }
    __syncthreads();
    if (t == 0) {
        int s = reds[0];
        for (int wv = 1; wv < kVT / 32; ++wv) s = min(s, reds[wv]);
        *bcast = s;
        if (st_last) *st_last = s;
    }
    __syncthreads();
    const int out = *bcast;
    __syncthreads();
    return out;
}

}  // namespace exl3b
