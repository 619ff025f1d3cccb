// ldlq.cu -- BlockLDLQ sweep with the trellis encoder fused per tile.
//
// Reference: quantize/quantize.py:631-746 (ldlq_viterbi) and :360-378
// (pack_states).  Layouts on device ([k][n] row-major, k = in, n = out):
//   Wq    fp32 [k][n]   unit-scaled inner weights
//   Lfac  fp32 [k][k]   block-LDL factor (identity 16x16 diagonal blocks)
//   prod  fp32 [k][n]   feedback cache of finished buffers
//   E     fp32 [k][n]   Wq - hatW of finished blocks
//   hatW  fp32 [k][n]   decoded weights (output)
//   trellis int16 [k/16][n_seg/16][16K] per column segment (output)
//
// Sweep (host loop, all launches on one stream): k-blocks right to left in
// launch buffers of max(buf_cols, 512) rows.  One tile-kernel launch per
// buffer covers all its k-blocks x
// column tiles.  Launches with at least two tiles per SM use the persistent
// lazy-argmin kernel (ldlq_lazy.cu), launches whose column tiles do not fill
// the SMs its one-tile-per-CTA variant (same file); the others, one CTA per
// tile with the traced encoder, below.  Each CTA takes a ticket in dependency order (k-block
// descending, column ascending) and, when it needs the block below it in the
// same column (intra-buffer feedback), waits on that column's progress
// counter.  The producer of that block took an earlier ticket, so it is
// resident and finishes: no deadlock, and no wave quantisation (320 column
// tiles on 148 SMs would otherwise leave the third wave 84% idle).  The wait is
// bounded; on time-out the CTA sets an error word and returns.  After a
// buffer, prod[:16lo] += Lfac[buf, :16lo]^T E[buf] on tcgen05 tensor cores
// (gemm_tc.cu, 3xTF32, TMA-fed).  Columns never interact
// (Lfac couples rows only), so each CTA owns one column tile of one k-block:
//   WXWX = (Wq + Lfac[later, blk]^T . E[later]) + prod     (quantize.py:676-682)
//   x[t] = WXWX[perm[t]]                                   (:684-686)
//   states = tail-biting encode(x)                         (:687-731)
//   hatW[perm[t]] = lut[states[t]], E = Wq - hatW          (:736-741)
//   trellis = pack(states)                                 (:846, :360-378)
#include <stdlib.h>
#include <string.h>

#include "exl3b_internal.h"
#include "ldlq_tile.cuh"
#include "viterbi.cuh"

namespace exl3b {

// Column tiles up to which a launch of `grid` CTAs at K runs one tile per CTA
// at a time (ldlq_solo_kernel): `grid`, where each column's chain of k-blocks
// keeps at most one CTA busy -- except at K = 6, where the one-tile kernel
// measured 5.5% slower (0.694 against 0.658 ms per k-block at 32 column
// tiles; K = 2, 3, 4, 5, 7: 9.5, 8, 7.7, 6.4, 8% faster).  EXL3B_SOLO_COLS (a
// column count, 0 = never) replaces it for every K; the tests use it to run
// both kernels on the same shapes.
static int solo_max_cols(int grid, int K) {
    const char* e = getenv("EXL3B_SOLO_COLS");
    if (e != nullptr && *e != 0) return atoi(e);
    return K == 6 ? 0 : grid;
}

// sched (shared): [0] k-block i, [1] column tile c, [2] backpointer slot,
// [3] ok, [4] column segment.  Re-read where needed instead of being kept
// live in registers across the encode.
template <int K>
__device__ __forceinline__ void ldlq_tile_body(const LdlqTileParams& p, char* smem,
                                               const volatile int* sched) {
    using SM = VitSmem<K>;
    const int t = threadIdx.x;
    float* xs = reinterpret_cast<float*>(smem + SM::OFF_X);
    // the traceback staging area is free until the traceback: 16x16 staging
    // and the feedback rows
    static_assert(1024 + kGatherStageBytes <= kTbBytes, "gather staging fits");
    float* wx = reinterpret_cast<float*>(smem + SM::OFF_TB);
    tile_feedback_gather(p, sched[0], sched[1], xs, wx, wx + 256, t, kVT);
    // ---- trellis encode
    {
        __half2 f2[64];
        vit_load_f2tab(f2, p.f2tab[K], t);
        uint8_t* bp = p.bp_ws + (size_t)sched[2] * p.bp_slot;
        vit_tailbite<K>(f2, smem, p.pivot, p.margin, bp, t);
    }
    // ---- write-back: the column tile and its segment are re-read from shared
    // memory here rather than kept live in registers across the encode.
    tile_writeback<K>(p, sched[0], sched[1], sched[4],
                      reinterpret_cast<const int32_t*>(smem + SM::OFF_ST), t);
}

// slot-holder tag: (SM id << 20) | (ticket + 1), nonzero
__device__ __forceinline__ int holder_tag(int ticket) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    return (int)((smid << 20) | (unsigned)((ticket + 1) & 0xFFFFF));
}

template <int K>
__global__ void __launch_bounds__(kVT, 1)
ldlq_tile_kernel(const __grid_constant__ LdlqTileParams p) {
    extern __shared__ __align__(16) char smem[];
    __shared__ int sched[5];            // i, c, slot, ok, segment
    const int t = threadIdx.x;
    if (t == 0) {
        const int ticket = atomicAdd(p.tickets, 1);
        int i, c, seg;
        tile_of_ticket(p, ticket, i, c, seg);
        int ok = 1;
        // backpointer slot: nslots exceeds the CTAs the device can hold
        // resident at once (SMs x occupancy), so at every instant a slot is
        // free.  CTAs of a wave start together and race for the slots their
        // predecessors just released, so a single pass can lose every race:
        // keep scanning (hashed start, read before CAS) until one is won,
        // within the same time bound as the dependency wait.
        int slot = -1;
        int cause = 0, seen = -1;
        {
            const unsigned h = (unsigned)ticket * 2654435761u;
            const int start = (int)(h % (unsigned)p.nslots);
            const long long t0 = clock64();
            const long long limit = p.wait_cycles;
            while (slot < 0) {
                for (int k = 0; k < p.nslots && slot < 0; ++k) {
                    int cand = start + k;
                    if (cand >= p.nslots) cand -= p.nslots;
                    if (ld_acquire(&p.slots[cand]) == 0 &&
                        atomicCAS(&p.slots[cand], 0, holder_tag(ticket)) == 0)
                        slot = cand;
                }
                if (slot >= 0) break;
                if (clock64() - t0 > limit) break;
                __nanosleep(128);
            }
        }
        if (slot < 0) { ok = 0; cause = 1; }
        // intra-buffer feedback needs blocks i+1 .. cur-1 of this column
        if (ok && p.Lfac && i + 1 < p.cur) {
            const int need = p.tk - 1 - i;
            const long long t0 = clock64();
            const long long limit = p.wait_cycles;
            while ((seen = ld_acquire(&p.colprog[c])) < need) {
                if (ld_acquire(p.err)) { ok = 0; break; }
                if (clock64() - t0 > limit) { ok = 0; cause = 2; break; }
                __nanosleep(256);
            }
        }
        if (!ok && cause) {
            // first failure records what it was: cause (1 slot, 2 wait),
            // ticket, k-block, column, progress seen
            if (atomicCAS(p.err, 0, cause) == 0) {
                p.err[1] = ticket; p.err[2] = i; p.err[3] = c; p.err[4] = seen;
                // holders (ticket + 1) of the first slots, for diagnosis
                for (int q = 0; q < 8; ++q) p.err[5 + q] = p.slots[q];
                int held = 0;
                for (int q = 0; q < p.nslots; ++q) held += p.slots[q] != 0;
                p.err[13] = held;
            }
        } else if (!ok) {
            atomicCAS(p.err, 0, 3);
        }
        sched[0] = i;
        sched[1] = c;
        sched[2] = slot;
        sched[3] = ok;
        sched[4] = seg;
    }
    __syncthreads();
    if (!sched[3]) {
        if (t == 0 && sched[2] >= 0) atomicExch(&p.slots[sched[2]], 0);
        return;
    }
    ldlq_tile_body<K>(p, smem, sched);
    __syncthreads();    // every thread's writes of this tile precede the release
    if (t == 0) {
        __threadfence();
        atomicExch(&p.slots[sched[2]], 0);
        atomicAdd(&p.colprog[sched[1]], 1);
    }
}

template <int K>
static int launch_tile_k(const LdlqTileParams& p, unsigned grid, cudaStream_t stream) {
    static bool attr[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev]) {
        if (check_cuda(cudaFuncSetAttribute(ldlq_tile_kernel<K>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            VitSmem<K>::BYTES),
                       "cudaFuncSetAttribute(ldlq_tile)"))
            return RC_DEVICE_ERROR;
        attr[dev] = true;
    }
    ldlq_tile_kernel<K><<<grid, kVT, VitSmem<K>::BYTES, stream>>>(p);
    note_launch();
    return check_cuda(cudaGetLastError(), "ldlq_tile_kernel launch") ? RC_DEVICE_ERROR : RC_OK;
}

// Most CTAs of the K=2..7 tile kernels one SM can hold at once (driver
// occupancy calculation), cached per device.  Sizes the backpointer-slot pool.
int ldlq_tile_max_resident_per_sm() {
    static int cache[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (cache[dev]) return cache[dev];
    int m = 1, nb = 0;
#define EXL3B_OCC(K)                                                                   \
    cudaFuncSetAttribute(ldlq_tile_kernel<K>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                         VitSmem<K>::BYTES);                                           \
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, ldlq_tile_kernel<K>, kVT,    \
                                                      VitSmem<K>::BYTES) == cudaSuccess \
        && nb > m) m = nb;
    EXL3B_OCC(2) EXL3B_OCC(3) EXL3B_OCC(4) EXL3B_OCC(5) EXL3B_OCC(6) EXL3B_OCC(7)
#undef EXL3B_OCC
    cache[dev] = m;
    return m;
}

static int launch_tile(int K, const LdlqTileParams& p, unsigned grid, cudaStream_t stream) {
    switch (K) {
        case 2: return launch_tile_k<2>(p, grid, stream);
        case 3: return launch_tile_k<3>(p, grid, stream);
        case 4: return launch_tile_k<4>(p, grid, stream);
        case 5: return launch_tile_k<5>(p, grid, stream);
        case 6: return launch_tile_k<6>(p, grid, stream);
        case 7: return launch_tile_k<7>(p, grid, stream);
    }
    set_error("K=%d outside 2..7", K);
    return RC_BAD_K;
}

int ldlq_sweep(const SweepArgs& a, cudaStream_t stream) {
    const int tk = a.k / 16, tn = a.n / 16;
    LdlqTileParams p;
    memset(&p, 0, sizeof(p));
    p.Wq = a.Wq; p.E = a.E; p.hatW = a.hatW; p.Lfac = a.Lfac;
    p.prod = a.Lfac ? a.prod : nullptr;
    p.k = a.k; p.n = a.n; p.pivot = a.pivot; p.margin = a.margin; p.tk = tk;
    p.nseg = a.nseg;
    for (int s = 0; s <= a.nseg; ++s) p.seg_c0[s] = a.seg_c0[s];
    for (int s = 0; s < a.nseg; ++s) { p.seg_K[s] = a.seg_K[s]; p.seg_trellis[s] = a.seg_trellis[s]; }
    p.states = a.states; p.xout = a.xout; p.bp_ws = a.bp_ws; p.bp_slot = a.bp_slot;
    p.lazy_ws = a.lazy_ws;
    const int sms = device_sms();
    p.slots = a.slots; p.nslots = a.nslots; p.colprog = a.colprog; p.err = a.err;
    // wait bound in SM clock cycles, counted at 2 cycles per ns (>= the
    // B200's 1965 MHz maximum clock, so the bound is never shorter in time)
    p.wait_cycles = (long long)(a.wait_ns * 2.0);
    for (int K = 0; K < 8; ++K) p.f2tab[K] = a.f2tab[K];
    p.lut32 = a.lut32;

    // k-blocks [lo, hi) of buffer end `cur`: one launch per distinct K over the
    // column segments of that K
    int kmin = 8;
    for (int s = 0; s < a.nseg; ++s) kmin = a.seg_K[s] < kmin ? a.seg_K[s] : kmin;
    auto launch = [&](int cur, int lo, int hi) -> int {
        p.cur = cur;
        p.top = hi - 1;
        struct Group { int K, nls; int ls_seg[kMaxSeg]; int ls_pre[kMaxSeg + 1]; long long nb; };
        Group g[kMaxSeg];
        int ng = 0, big = 0;
        long long total = 0;
        bool done[kMaxSeg] = {};
        for (int s0 = 0; s0 < a.nseg; ++s0) {
            if (done[s0]) continue;
            Group& G = g[ng];
            G.K = a.seg_K[s0];
            G.nls = 0;
            G.ls_pre[0] = 0;
            for (int s1 = s0; s1 < a.nseg; ++s1) {
                if (a.seg_K[s1] != G.K) continue;
                done[s1] = true;
                G.ls_seg[G.nls] = s1;
                G.ls_pre[G.nls + 1] = G.ls_pre[G.nls] + (a.seg_c0[s1 + 1] - a.seg_c0[s1]);
                ++G.nls;
            }
            G.nb = (long long)(hi - lo) * G.ls_pre[G.nls];
            total += G.nb;
            if (G.nb > g[big].nb) big = ng;
            ++ng;
        }
        // Segments of different K side by side: columns never interact, so the
        // largest group runs on the caller's stream with its share of the SMs
        // and the others, one after another, on the helper stream with the
        // rest (own ticket counter, row regions after the first share's).  A
        // narrow segment alone on the whole GPU would leave its CTAs waiting
        // for the block below in their column.  Only when every launch keeps
        // at least two tiles per CTA (the lazy pipeline); else one after
        // another on the caller's stream, each over all SMs.
        int grid_big = sms, grid_side = 0;
        bool conc = false;
        if (ng > 1 && a.side && a.lazy_ws && sms > 1) {
            // SMs in proportion to each side's work: tiles x the time of a
            // tile at its K (lazy encoder, ms per tile-slot x 1000, measured on
            // B200 at 20 tiles per SM: K = 2..7)
            static const double kTileCost[8] = {0, 0, 593, 547, 522, 495, 523, 535};
            double wtot = 0.0, wbig = 0.0;
            for (int i = 0; i < ng; ++i) {
                const double w = (double)g[i].nb * kTileCost[g[i].K];
                wtot += w;
                if (w > wbig) {
                    wbig = w;
                    big = i;
                }
            }
            grid_big = (int)((double)sms * wbig / wtot + 0.5);
            grid_big = grid_big < 1 ? 1 : (grid_big > sms - 1 ? sms - 1 : grid_big);
            grid_side = sms - grid_big;
            conc = lazy_pipeline(g[big].K, g[big].nb, grid_big);
            for (int i = 0; i < ng; ++i)
                if (i != big) conc = conc && lazy_pipeline(g[i].K, g[i].nb, grid_side);
        }
        // profiling: a concurrent group is one interval on the caller's stream
        // (fork to join) doing all its tiles
        if (conc) prof_begin_launch(stream, PROF_TILE, (double)total * 256.0);
        if (conc && (check_cuda(cudaEventRecord(a.ev_fork, stream), "segment fork") ||
                     check_cuda(cudaStreamWaitEvent(a.side, a.ev_fork, 0), "segment fork")))
            return RC_DEVICE_ERROR;
        for (int i = 0; i < ng; ++i) {
            const Group& G = g[i];
            const bool on_side = conc && i != big;
            cudaStream_t s = on_side ? a.side : stream;
            p.nls = G.nls;
            for (int m = 0; m < G.nls; ++m) p.ls_seg[m] = G.ls_seg[m];
            for (int m = 0; m <= G.nls; ++m) p.ls_pre[m] = G.ls_pre[m];
            p.tickets = on_side ? a.tickets2 : a.tickets;
            p.lazy_ws = on_side ? a.lazy_ws + (size_t)grid_big * 2 * (lazy_region_bytes(kmin) / 4)
                                : a.lazy_ws;
            if (check_cuda(cudaMemsetAsync(p.tickets, 0, sizeof(int), s), "memset tickets"))
                return RC_DEVICE_ERROR;
            p.ntiles = (int)G.nb;
            const int grid = conc ? (on_side ? grid_side : grid_big) : sms;
            if (!conc) prof_begin_launch(s, PROF_TILE, (double)G.nb * 256.0);
            // at least two tiles per SM: persistent CTAs, lazy argmin; one tile
            // per CTA at a time when the column tiles do not fill the CTAs
            const bool lazy = a.lazy_ws != nullptr && lazy_pipeline(G.K, G.nb, grid);
            const bool solo = a.lazy_ws != nullptr && G.K >= kLazyMinK &&
                              G.ls_pre[G.nls] <= solo_max_cols(grid, G.K);
            const int rc = solo ? launch_solo_tile(G.K, p, (unsigned)grid, s)
                         : lazy ? launch_lazy_tile(G.K, p, (unsigned)grid, s)
                                : launch_tile(G.K, p, (unsigned)G.nb, s);
            if (!conc) prof_end_launch(s);
            if (rc) return rc;
        }
        if (conc && (check_cuda(cudaEventRecord(a.ev_join, a.side), "segment join") ||
                     check_cuda(cudaStreamWaitEvent(stream, a.ev_join, 0), "segment join")))
            return RC_DEVICE_ERROR;
        if (conc) prof_end_launch(stream);
        return RC_OK;
    };
    if (!a.Lfac) {
        // no feedback: every tile is independent, one launch
        return launch(a.block_hi, a.block_lo, a.block_hi);
    }
    // Launch buffers of max(buf_cols, kMinLaunchRows) rows.  buf_cols is the
    // reference's blocking of the feedback-cache update; every block's target
    // is Wq + sum over later rows of Lfac^T E whatever the blocking (only the
    // fp32 summation order changes).  With the staged feedback gather, 512-
    // and 1024-row launches measured fastest (config 2: 383 ms per layer
    // against 398 ms at 128 rows): fewer launch tails and GEMM round trips.
    constexpr int kMinLaunchRows = 512;
    const int rows = a.buf_cols > kMinLaunchRows ? a.buf_cols : kMinLaunchRows;
    const int buf_tiles = rows / 16;
    // buffers are anchored at tk like the reference: [tk - b - buf_tiles, tk - b)
    for (int cur = tk; cur > 0; cur -= buf_tiles) {
        const int lo = cur - buf_tiles > 0 ? cur - buf_tiles : 0;
        const int hi_l = cur < a.block_hi ? cur : a.block_hi;
        const int lo_l = lo > a.block_lo ? lo : a.block_lo;
        if (lo_l >= hi_l) continue;
        int rc = launch(cur, lo_l, hi_l);
        if (rc) return rc;
        if (lo > 0 && lo >= a.block_lo) {
            // prod[0:16lo, :] += Lfac[16lo:16cur, 0:16lo]^T . E[16lo:16cur, :]
            prof_begin_launch(stream, PROF_GEMM,
                              (double)(16 * lo) * a.n * (16 * (cur - lo)) * 2.0);
            rc = launch_gemm_tn_acc_tc(16 * lo, a.n, 16 * (cur - lo),
                                       a.Lfac + (size_t)16 * lo * a.k, a.k,
                                       a.E + (size_t)16 * lo * a.n, a.n,
                                       a.prod, a.n, a.err, stream, 1.0f, 0,
                                       a.split_ws, a.split_bytes);
            prof_end_launch(stream);
            if (rc) return rc;
        }
    }
    return RC_OK;
}

// ------------------------------------------------------------------ bitstream
// pack_states (quantize.py:360-378): states int32 [nt][256] -> int16 [nt][16K]
__global__ void pack_kernel(const int32_t* __restrict__ st, int nt, int K,
                            int16_t* __restrict__ out) {
    const int words = 8 * K;
    const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (size_t)nt * words) return;
    const size_t tile = gid / words;
    const int w = (int)(gid % words);
    const int32_t* s = st + tile * 256;
    uint32_t word = 0;
    for (int j = 0; j < 32; ++j) {
        const int q = 32 * w + j;
        const int step = q / K, b = q - step * K;
        word |= (((uint32_t)s[step] >> (K - 1 - b)) & 1u) << (31 - j);
    }
    out[tile * 16 * K + 2 * w] = (int16_t)(word & 0xFFFFu);
    out[tile * 16 * K + 2 * w + 1] = (int16_t)(word >> 16);
}

// State t of a tile (quantize.py:381-402): the 16-bit circular window of
// its 256K-bit stream ending at bit (t+1)K.  Stream bit q is bit 31 - (q & 31)
// of u32 word q >> 5, a word being int16 halves (low half first); the window
// lies in words b0 >> 5 and the next one (circularly), so two words, read as
// four 16-bit halves, give it with one 64-bit shift.
__device__ __forceinline__ uint32_t tile_state(const uint16_t* __restrict__ w16, int K, int t) {
    const int nbits = 256 * K;
    int b0 = t * K + K - 16;
    if (b0 < 0) b0 += nbits;
    const int wi = b0 >> 5, bi = b0 & 31;
    const int wj = (wi + 1 == 8 * K) ? 0 : wi + 1;
    const uint32_t a = (uint32_t)__ldg(w16 + 2 * wi) | ((uint32_t)__ldg(w16 + 2 * wi + 1) << 16);
    const uint32_t b = (uint32_t)__ldg(w16 + 2 * wj) | ((uint32_t)__ldg(w16 + 2 * wj + 1) << 16);
    const uint64_t v = ((uint64_t)a << 32) | b;
    return (uint32_t)(v >> (48 - bi)) & 0xFFFFu;
}

// unpack_states: trellis [nt][16K] -> states int32 [nt][256]
__global__ void unpack_kernel(const int16_t* __restrict__ tr, int nt, int K,
                              int32_t* __restrict__ st) {
    const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (size_t)nt * 256) return;
    const size_t tile = gid / 256;
    const uint16_t* w16 = reinterpret_cast<const uint16_t*>(tr) + tile * 16 * K;
    st[gid] = (int32_t)tile_state(w16, K, (int)(gid % 256));
}

// Element (r, cc) of a [16 tk][16 tn] matrix -> (tile, step t): the inverse
// of tc_perm inside tile (r / 16, cc / 16).  One thread per element in
// row-major order keeps the matrix side of decode and verify coalesced.
__device__ __forceinline__ void elem_tile_step(size_t gid, int tn, size_t& tile, int& t) {
    const int n = 16 * tn;
    const size_t r = gid / n;
    const int cc = (int)(gid - r * n);
    tile = (r >> 4) * (size_t)tn + (cc >> 4);
    t = tc_perm_inv((int)(r & 15), cc & 15);
}

// decode_trellis (quantize.py:405-415): trellis [tk][tn][16K] -> W [k][n]
__global__ void decode_kernel(const int16_t* __restrict__ tr, int tk, int tn, int K,
                              const float* __restrict__ lut, float* __restrict__ W) {
    const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (size_t)tk * tn * 256) return;
    size_t tile;
    int t;
    elem_tile_step(gid, tn, tile, t);
    const uint16_t* w16 = reinterpret_cast<const uint16_t*>(tr) + tile * 16 * K;
    W[gid] = __ldg(lut + tile_state(w16, K, t));
}

// Self-check (quantize.py:849-853, :958-963): one thread per weight, in
// hatW's row-major order, decodes its state from the trellis window and
// compares the decoded value with the encoder's hatW (bit pattern) and, with
// states, the state with the encoder's.  A warp adds its mismatch count once.
__global__ void verify_kernel(const int16_t* __restrict__ tr, int tk, int tn, int K,
                              const float* __restrict__ lut, const float* __restrict__ hatW,
                              int ldw, const int32_t* __restrict__ states, int ld_states,
                              int* __restrict__ bad) {
    const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    bool miss = false;
    if (gid < (size_t)tk * tn * 256) {
        size_t tile;
        int t;
        elem_tile_step(gid, tn, tile, t);
        const uint16_t* w16 = reinterpret_cast<const uint16_t*>(tr) + tile * 16 * K;
        const uint32_t s = tile_state(w16, K, t);
        const size_t r = gid / (16 * tn);
        const float hw = hatW[r * (size_t)ldw + (gid - r * 16 * tn)];
        miss = __float_as_uint(__ldg(lut + s)) != __float_as_uint(hw);
        if (states) {
            const size_t i = tile / tn, c = tile - i * tn;
            miss = miss || (uint32_t)(states[(i * ld_states + c) * 256 + t] & 0xFFFF) != s;
        }
    }
    const unsigned m = __ballot_sync(0xffffffffu, miss);
    if ((threadIdx.x & 31) == 0 && m) atomicAdd(bad, __popc(m));
}

int launch_verify(const int16_t* tr, int tk, int tn, int K, const float* lut,
                  const float* hatW, int ldw, const int32_t* states, int ld_states, int* bad,
                  cudaStream_t stream) {
    const size_t total = (size_t)tk * tn * 256;
    if (total)
        verify_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(
            tr, tk, tn, K, lut, hatW, ldw, states, ld_states, bad);
    note_launch();
    return check_cuda(cudaGetLastError(), "verify launch") ? RC_DEVICE_ERROR : RC_OK;
}

int launch_pack(const int32_t* st, int nt, int K, int16_t* out, cudaStream_t stream) {
    const size_t total = (size_t)nt * 8 * K;
    if (total) pack_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(st, nt, K, out);
    note_launch();
    return check_cuda(cudaGetLastError(), "pack launch") ? RC_DEVICE_ERROR : RC_OK;
}

int launch_unpack(const int16_t* tr, int nt, int K, int32_t* st, cudaStream_t stream) {
    const size_t total = (size_t)nt * 256;
    if (total) unpack_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(tr, nt, K, st);
    note_launch();
    return check_cuda(cudaGetLastError(), "unpack launch") ? RC_DEVICE_ERROR : RC_OK;
}

int launch_decode(const int16_t* tr, int tk, int tn, int K, const float* lut, float* W,
                  cudaStream_t stream) {
    const size_t total = (size_t)tk * tn * 256;
    if (total) decode_kernel<<<(unsigned)((total + 255) / 256), 256, 0, stream>>>(tr, tk, tn, K, lut, W);
    note_launch();
    return check_cuda(cudaGetLastError(), "decode launch") ? RC_DEVICE_ERROR : RC_OK;
}

}  // namespace exl3b
