// ldlq_tile.cuh -- pieces shared by the two LDLQ sweep tile kernels: the
// launch parameter block, the tensor-core permutation, the ticket -> tile
// mapping, the per-tile feedback + gather and the per-tile write-back + pack.
// (ldlq.cu: one CTA per tile with the traced encoder; ldlq_lazy.cu: persistent
// CTAs with the lazy-argmin pipeline.)
#pragma once
#include "exl3b_internal.h"
#include "viterbi.cuh"

namespace exl3b {

constexpr int kMaxSeg = 8;

struct LdlqTileParams {
    const float* Wq;
    float* E;
    float* hatW;
    const float* Lfac;      // null: no feedback
    const float* prod;      // null: no feedback
    int k, n;
    int cur;                // buffer end block (exclusive)
    int top;                // first (highest) k-block of this launch
    int tk;                 // k-blocks of the whole matrix
    int pivot, margin;
    int* tickets;           // launch ticket counter (zeroed before launch)
    int ntiles;             // tiles of this launch (persistent kernel: fetch bound)
    int* colprog;           // [tn] k-blocks finished per column (sweep-wide)
    int* slots;             // [nslots] backpointer-slot ownership flags
    int nslots;
    int* err;               // error word (set on a wait time-out)
    long long wait_cycles;  // bound of every dependency / slot wait (SM clock cycles)
    int nseg;
    int seg_c0[kMaxSeg + 1];     // segment column-tile starts, seg_c0[nseg] = tn
    int seg_K[kMaxSeg];
    int16_t* seg_trellis[kMaxSeg];
    // segments encoded by this launch (all of one K): ids and column prefix
    int nls;
    int ls_seg[kMaxSeg];
    int ls_pre[kMaxSeg + 1];     // ls_pre[m] = columns of segments ls_seg[0..m)
    int32_t* states;        // [tk][tn][256] or null
    float* xout;            // [tk][tn][256] or null (encoder targets, for checks)
    uint8_t* bp_ws;         // wave slots
    size_t bp_slot;         // bytes per slot
    float* lazy_ws;         // lazy pipeline: 2 row regions per CTA
    const uint4* f2tab[8];  // per K
    const float* lut32;     // decode table fp32 [65536]
};

// sequence step t -> row-major position in the 16x16 tile (quantize.py:101-118)
__device__ __forceinline__ int tc_perm(int t) {
    const int tt = t >> 3, q = t & 7;
    const int r0 = (tt & 3) * 2, c0 = tt >> 2;
    const int row = r0 + (q & 1) + ((q & 2) ? 8 : 0);
    const int col = c0 + ((q & 4) ? 8 : 0);
    return row * 16 + col;
}

// (row, col) in the 16x16 tile -> sequence step t, the inverse of tc_perm
__device__ __forceinline__ int tc_perm_inv(int row, int col) {
    const int tt = (col & 7) * 4 + ((row & 7) >> 1);
    const int q = (row & 1) | ((row >> 3) << 1) | ((col >> 3) << 2);
    return tt * 8 + q;
}

__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

constexpr long long kWaitNs = 4000000000LL;   // default bound of any dependency wait: 4 s

// Ticket -> (k-block i, column tile c, segment) of this launch: k-blocks from
// `top` down, columns of the launch's segments in order within a block.
__device__ __forceinline__ void tile_of_ticket(const LdlqTileParams& p, int ticket, int& i,
                                               int& c, int& seg) {
    const int ncols = p.ls_pre[p.nls];
    i = p.top - ticket / ncols;
    const int lc = ticket % ncols;
    int m = 0;
    while (m + 1 < p.nls && lc >= p.ls_pre[m + 1]) ++m;
    seg = p.ls_seg[m];
    c = p.seg_c0[seg] + (lc - p.ls_pre[m]);
}

// Feedback and gather of tile (i, c) into xs[256] (quantize.py:676-686):
//   WXWX = (Wq + Lfac[later, blk]^T . E[later]) + prod,  x[t] = WXWX[perm[t]].
// The later rows r of this buffer (16 (i+1) <= r < 16 cur) are staged in
// chunks of kGatherRows: every thread of the CTA issues coalesced 16-byte
// loads of the rows' 16-wide slices Lfac[r, 16 i ..] and E[r, 16 c ..] (E
// at L2, ld.global.cg: other CTAs of this launch wrote it), so a chunk costs
// one memory round trip; then thread (a, col) accumulates
// fma(Lfac[r, 16 i + a], E[r, 16 c + col], acc) over r ascending from
// shared memory.  wx: 1 KB shared staging; stage: 2 x kGatherRows x 64 bytes
// (16 KB), 16-byte aligned.  Every thread of the CTA (nthreads) calls it.
constexpr int kGatherRows = 128;
constexpr int kGatherStageBytes = 2 * kGatherRows * 16 * 4;

__device__ __forceinline__ void tile_feedback_gather(const LdlqTileParams& p, int i, int c,
                                                     float* xs, float* wx, float* stage,
                                                     int t, int nthreads) {
    const int tn = p.seg_c0[p.nseg];
    const size_t n = (size_t)p.n;
    const int a = (t >> 4) & 15, col = t & 15;
    const size_t row = (size_t)(16 * i + a);
    const size_t gc = (size_t)(16 * c + col);
    float w = 0.0f, pr = 0.0f;
    if (t < 256) {
        w = p.Wq[row * n + gc];
        if (p.Lfac) pr = p.prod[row * n + gc];
    }
    if (p.Lfac) {
        const int r_lo = 16 * (i + 1), r_hi = 16 * p.cur;
        if (r_lo < r_hi) {
            float acc = 0.0f;
            float4* sL = reinterpret_cast<float4*>(stage);
            float4* sE = sL + kGatherRows * 4;
            for (int r0 = r_lo; r0 < r_hi; r0 += kGatherRows) {
                const int nq = 4 * min(kGatherRows, r_hi - r0);   // float4 per slice set
                for (int q = t; q < nq; q += nthreads) {
                    const size_t r = (size_t)(r0 + (q >> 2));
                    const int o = 4 * (q & 3);
                    sL[q] = *reinterpret_cast<const float4*>(p.Lfac + r * p.k + 16 * i + o);
                    sE[q] = __ldcg(reinterpret_cast<const float4*>(p.E + r * n + 16 * c + o));
                }
                __syncthreads();
                if (t < 256) {
                    const float* L = reinterpret_cast<const float*>(sL);
                    const float* Ev = reinterpret_cast<const float*>(sE);
                    for (int rr = 0; rr < nq / 4; ++rr)
                        acc = fmaf(L[rr * 16 + a], Ev[rr * 16 + col], acc);
                }
                __syncthreads();
            }
            w = w + acc;
        }
        w = w + pr;
    }
    if (t < 256) wx[t] = w;
    __syncthreads();
    if (t < 256) {
        const float x = wx[tc_perm(t)];
        xs[t] = x;
        if (p.xout) p.xout[((size_t)i * tn + c) * 256 + t] = x;
    }
    __syncthreads();
}

// Write-back of tile (i, c) from its 256 states st[] (quantize.py:736-741,
// :846, :360-378): hatW[perm[t]] = lut[s_t], E = Wq - hatW, states, and the
// packed trellis -- stream bit q = t*K + b (MSB first within a symbol); u32
// word w holds stream bits [32w, 32w+32) MSB first; stored as int16 low half
// first.  No barrier inside; the caller makes st[] visible first.
template <int K>
__device__ __forceinline__ void tile_writeback(const LdlqTileParams& p, int i, int c, int seg,
                                               const int32_t* st, int t) {
    const int tn = p.seg_c0[p.nseg];
    const size_t n = (size_t)p.n;
    if (t < 256) {
        const int s = st[t] & 0xFFFF;        // states are 16-bit
        const int pos = tc_perm(t);
        const size_t idx = (size_t)(16 * i + (pos >> 4)) * n + (size_t)(16 * c + (pos & 15));
        const float v = p.lut32[s];
        p.hatW[idx] = v;
        p.E[idx] = p.Wq[idx] - v;
        if (p.states) p.states[((size_t)i * tn + c) * 256 + t] = s;
    }
    constexpr int NW = 8 * K;
    if (t < NW) {
        uint32_t word = 0;
#pragma unroll 4
        for (int j = 0; j < 32; ++j) {
            const int q = 32 * t + j;
            const int step = q / K, b = q - step * K;
            const uint32_t bit = ((uint32_t)st[step] >> (K - 1 - b)) & 1u;
            word |= bit << (31 - j);
        }
        const int seg_tn = p.seg_c0[seg + 1] - p.seg_c0[seg];
        int16_t* out = p.seg_trellis[seg] +
                       ((size_t)i * seg_tn + (c - p.seg_c0[seg])) * (16 * K);
        out[2 * t] = (int16_t)(word & 0xFFFFu);
        out[2 * t + 1] = (int16_t)(word >> 16);
    }
}

// ldlq_lazy.cu: persistent lazy-argmin tile kernel for K = 2..7, `grid` CTAs
int launch_lazy_tile(int K, const LdlqTileParams& p, unsigned grid, cudaStream_t stream);
// ldlq_lazy.cu: the same encoder one tile at a time per CTA (narrow launches)
int launch_solo_tile(int K, const LdlqTileParams& p, unsigned grid, cudaStream_t stream);

}  // namespace exl3b
