// viterbi.cuh -- tail-biting trellis Viterbi for one 16x16 tile per CTA.
//
// Algorithm (reference: quantize/quantize.py:218-354, viterbi() and
// quantize_seq_tailbite(), emit_mode "sq"): 256-step shift-register trellis,
// 16-bit state s, K bits enter per step, decode value f(s) = lut[s].
//   cost_0(s)  = (f(s) - x_0)^2                    (+ 0/inf boundary mask)
//   best_i(j)  = min_w cost_{i-1}(j + w*2^(16-K))   first index on ties
//   cost_i(s)  = (f(s) - x_i)^2 + best_i(s >> K)
// Two passes: pass 1 on the sequence rolled by `pivot` with a free boundary
// (optionally only pivot+margin steps), giving the wrap bits; pass 2 pinned to
// them at both ends.
//
// B200 design:
//  * The 2^16-entry cost table is never stored.  Only best_i (2^(16-K) fp32)
//    lives in shared memory, double-buffered; cost_i(s) is recomputed inside
//    the min of the next step.  fp32 operations and their order are the
//    reference's, so the result is bit-identical.
//  * The trellis splits into 2^(16-2K) butterflies: inputs best_i[m + w*P]
//    (w < 2^K, P = 2^(16-2K)) feed outputs best_{i+1}[m*2^K + v].  Each of the
//    512 threads owns 128 fixed states (whole butterflies for K <= 3, a slice of
//    one butterfly for K >= 4) and holds their decode values in 64 packed-fp16
//    registers for the whole kernel (EXL3 decode values are exact in fp16), so
//    one add-compare-select is: mixed fp16-fp32 sub, fmul, fadd, compare, 2
//    predicated FMA-pipe updates --
//    no shared-memory gather on the inner loop.
//  * Backpointers: each thread packs its outputs' K-bit argmins into one
//    8/16/32/64-bit word per step and stores it coalesced to global scratch
//    (row of 512 words per step).  Traceback runs on device: the CTA stages
//    chunks of rows into shared memory, one thread follows the path.
#pragma once
#include "exl3b_common.cuh"

namespace exl3b {

constexpr int kVT = 512;                 // threads per tile CTA
constexpr int kTbBytes = 64 * 1024;      // traceback staging buffer

template <int K>
struct Geo {
    static_assert(K >= 2 && K <= 7, "K must be 2..7");
    static constexpr int NC = 1 << K;                 // predecessors per state
    static constexpr int SPRE = 1 << (16 - K);        // best-array size
    static constexpr int LOGP = 16 - 2 * K;
    static constexpr int P = 1 << LOGP;               // butterflies
    static constexpr bool WHOLE = P >= kVT;           // K <= 3
    static constexpr int NB = WHOLE ? P / kVT : 1;    // butterflies per thread
    static constexpr int TPB = WHOLE ? 1 : kVT / P;   // threads per butterfly
    static constexpr int NJ = WHOLE ? NC : NC / TPB;  // outputs per butterfly per thread
    static constexpr int NOUT = NB * NJ;              // outputs per thread
    static constexpr int NSTATE = NOUT * NC;          // states per thread (128)
    static_assert(NSTATE == 128, "each thread owns 128 states");
    static constexpr int BPE = (K <= 2) ? 2 : (K <= 4 ? 4 : 8);  // bits / backpointer
    static constexpr int BPTB = NOUT * BPE / 8;       // backpointer bytes / thread / step
    static constexpr int BP_ROW = kVT * BPTB;         // backpointer bytes per step
    static constexpr int TB_ROWS = kTbBytes / BP_ROW; // rows per traceback chunk
    // best-array smem layout: transposed for K >= 6 (a butterfly's 64 or 128
    // inputs as 16-byte loads); natural for K <= 5, where a butterfly's 2^K
    // inputs are loads that a warp's lanes share or spread over distinct
    // banks -- a transposed layout there turns every output store into an 8-
    // to 16-way bank conflict (a warp's lanes write rows apart in one column).
    // (16-byte output stores measured slower than scalar ones: the extra live
    // registers cost more than the conflicts they remove.)
    static constexpr bool TRANSPOSED = K >= 6;
    // transposed row stride: NC floats, padded by 4 when a row is < 32 words
    // so that four consecutive butterflies start in different bank groups
    static constexpr int ROW = (NC < 32) ? NC + 4 : NC;
    static constexpr int NCH = (NJ >= 4) ? 1 : 4 / NJ;  // partial min chains
    // traced steps update (best, idx) once per predecessor pair instead of
    // once per candidate (measured faster at these K, slower at K = 3..5)
    static constexpr bool PAIR_UPDATE = (K == 2) || (K >= 6);

    // output index j of thread t's e-th output
    static __device__ __forceinline__ int out_j(int t, int e) {
        if (WHOLE) return (t + kVT * (e / NC)) * NC + (e % NC);
        return t * NJ + e;
    }
    // butterfly of thread t for its b-th butterfly
    static __device__ __forceinline__ int bfly(int t, int b) {
        return WHOLE ? t + kVT * b : t / TPB;
    }
    // shared-memory address of best[idx].  Transposed for K >= 5 so that a
    // butterfly's 2^K inputs are contiguous (16-byte vector loads).
    static __device__ __forceinline__ int baddr(int idx) {
        if (TRANSPOSED) return (idx & (P - 1)) * ROW + (idx >> LOGP);
        return idx;
    }
    // backpointer of output j inside one staged row
    static __device__ __forceinline__ int bp_read(const uint8_t* row, int j) {
        int tt, e;
        if (WHOLE) {
            const int m = j >> K;
            tt = m & (kVT - 1);
            e = (m / kVT) * NC + (j & (NC - 1));
        } else {
            tt = j / NJ;
            e = j % NJ;
        }
        const int bit = e * BPE;
        const int byte = row[tt * BPTB + (bit >> 3)];
        return (byte >> (bit & 7)) & ((1 << BPE) - 1);
    }
};

// Shared-memory layout of a tile CTA (dynamic shared memory).
template <int K>
struct VitSmem {
    static constexpr int B_BYTES =
        (Geo<K>::TRANSPOSED ? Geo<K>::P * Geo<K>::ROW : Geo<K>::SPRE) * 4;
    static constexpr int OFF_B0 = 0;
    static constexpr int OFF_B1 = B_BYTES;
    static constexpr int OFF_X = 2 * B_BYTES;          // 256 fp32 targets
    static constexpr int OFF_ST = OFF_X + 1024;        // 256 int32 states
    static constexpr int OFF_RED = OFF_ST + 1024;      // reduction scratch
    static constexpr int OFF_TB = OFF_RED + 256;       // traceback rows
    static constexpr int OFF_EXTRA = OFF_TB + kTbBytes; // caller-owned tail
    static constexpr int BYTES = OFF_EXTRA;
};

// Load this thread's 128 decode values (fp16-exact) into packed registers.
template <int K>
__device__ __forceinline__ void vit_load_f(__half2 (&f2)[64],
                                           const __half* __restrict__ lut16,
                                           int t) {
    using G = Geo<K>;
#pragma unroll
    for (int e = 0; e < G::NOUT; ++e) {
        const int j = G::out_j(t, e);
#pragma unroll
        for (int w = 0; w < G::NC; w += 2) {
            const __half a = lut16[j + w * G::SPRE];
            const __half b = lut16[j + (w + 1) * G::SPRE];
            f2[(e * G::NC + w) >> 1] = __halves2half2(a, b);
        }
    }
}

// Same 64 words from a pre-paired table laid out [16][kVT] uint4 (word r2 of
// thread t in component r2 % 4 of entry (r2 / 4) * kVT + t): 16 coalesced
// 16-byte loads instead of 128 scattered half loads.
__device__ __forceinline__ void vit_load_f2tab(__half2 (&f2)[64],
                                               const uint4* __restrict__ tab,
                                               int t) {
#pragma unroll
    for (int q = 0; q < 16; ++q) {
        uint4 v = tab[q * kVT + t];
        f2[4 * q + 0] = *reinterpret_cast<__half2*>(&v.x);
        f2[4 * q + 1] = *reinterpret_cast<__half2*>(&v.y);
        f2[4 * q + 2] = *reinterpret_cast<__half2*>(&v.z);
        f2[4 * q + 3] = *reinterpret_cast<__half2*>(&v.w);
    }
}

// Compare-and-update of one add-compare-select: if c < best then best = c and
// idx = W.  Strict < keeps the first (lowest) predecessor on ties, like
// torch.min.  Only the compare runs on the (half-rate) ALU pipe: both updates
// are predicated FMA-pipe instructions -- best = c + 0 (exact: costs are >= +0
// or +inf) and idx = 0 * 0 + W, the index held as the float whose bit pattern
// is W (a subnormal; fp32 arithmetic without flush-to-zero keeps it exact), so
// reading it back is a bit cast.  `zr` is a zero the compiler cannot see
// through (it comes from a volatile shared-memory load), so neither update
// folds back into an ALU move.
template <int W>
__device__ __forceinline__ void acs_update(float& best, float& idx, float c, float zr) {
    asm("{\n\t.reg .pred p;\n\t"
        "setp.lt.f32 p, %2, %0;\n\t"
        "@p add.rn.f32 %0, %2, %3;\n\t"
        "@p fma.rn.f32 %1, %3, %3, %4;\n\t}"
        : "+f"(best), "+f"(idx)
        : "f"(c), "f"(zr), "f"(__uint_as_float((uint32_t)W)));
}

// Costs of predecessors W and W + 1 of one output -- the low and high halves
// of one packed decode register: c = fl(fl(f - x)^2) + bw for both.  The
// sm_100 mixed-precision subtract takes each fp16 half directly (exact
// widening, one fp32 rounding: bit-identical to fl(float(f) - x)); the square
// and the add are one packed fp32x2 multiply and one packed add (IEEE
// round-to-nearest in each lane, identical to the scalar operations).  bw2
// holds (best_i of predecessor W, of W + 1).  The unpack sits in the same asm
// block as the subtractions, which consume x, so the compiler cannot hoist 128
// unpacked decode values out of the step loop (128 extra registers).
// (Computing one of the two differences as a mixed-precision FMA, f * 1 - x,
// moves it to the FMA pipe but measured slower.)
__device__ __forceinline__ void cost_pair(__half2 h2, float x, uint64_t bw2, float& c0,
                                          float& c1) {
    const uint32_t r = *reinterpret_cast<const uint32_t*>(&h2);
    asm("{\n\t.reg .b16 lo, hi;\n\t.reg .f32 d0, d1;\n\t.reg .b64 dd, cc;\n\t"
        "mov.b32 {lo, hi}, %2;\n\t"
        "sub.rn.f32.f16 d0, lo, %3;\n\t"
        "sub.rn.f32.f16 d1, hi, %3;\n\t"
        "mov.b64 dd, {d0, d1};\n\t"
        "mul.rn.f32x2 dd, dd, dd;\n\t"
        "add.rn.f32x2 cc, dd, %4;\n\t"
        "mov.b64 {%0, %1}, cc;\n\t}"
        : "=f"(c0), "=f"(c1) : "r"(r), "f"(x), "l"(bw2));
}

__device__ __forceinline__ float min3(float a, float b, float c) {
    float d;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Both candidates of a predecessor pair against (best, idx), equivalent to the
// two strict-< updates in ascending order (first index on ties):
//   m = min(best, c0, c1); improved = m < best;
//   the winner is W + 1 exactly when improved and c0 != m (c0 == m means W
//   wins, also when c1 == c0).
// Three ALU instructions (min, two compares) and two predicated FMA-pipe index
// writes (the subnormal-bit-pattern index of acs_update); best = m is a rename.
template <int W>
__device__ __forceinline__ void acs_update_pair(float& best, float& idx, float c0, float c1,
                                                float zr) {
    asm("{\n\t.reg .pred p, q;\n\t.reg .f32 m;\n\t"
        "min.f32 m, %0, %2, %3;\n\t"
        "setp.lt.f32 p, m, %0;\n\t"
        "setp.ne.and.f32 q, %2, m, p;\n\t"
        "@p fma.rn.f32 %1, %4, %4, %5;\n\t"
        "@q fma.rn.f32 %1, %4, %4, %6;\n\t"
        "mov.f32 %0, m;\n\t}"
        : "+f"(best), "+f"(idx)
        : "f"(c0), "f"(c1), "f"(zr), "f"(__uint_as_float((uint32_t)W)),
          "f"(__uint_as_float((uint32_t)(W + 1))));
}

// TRACK = false: the step's backpointers are never read (pass-1 steps before
// the traceback stop), so only the minimum is kept: one three-input min per
// predecessor pair instead of compares and selects.  The minimum value is the
// same either way.
// TRACK = true: per-candidate compare-and-update (acs_update) or, where it
// measured faster (Geo::PAIR_UPDATE: K = 2 and K >= 6), one update per pair
// (acs_update_pair).  Partial chains (NCH > 1, for the small-NJ shapes K >= 6)
// take whole pairs: chain (W / 2) mod NCH; each chain sees its candidates in
// ascending order, and the chains merge lexicographically on (value, index).
template <int K, int W, int NJ, int NCH, bool TRACK>
struct AcsPair {
    // predecessors W, W + 1 (W even) for all NJ outputs of butterfly slice b
    static __device__ __forceinline__ void run(const __half2 (&f2)[64], float x, uint64_t bw2,
                                               int b, float (&best)[NJ][NCH],
                                               float (&bi)[NJ][NCH], float zr) {
        constexpr int ch = (W >> 1) % NCH;
        constexpr bool first = (W >> 1) < NCH;
#pragma unroll
        for (int u = 0; u < NJ; ++u) {
            float c0, c1;
            cost_pair(f2[(((b * NJ + u) << K) + W) >> 1], x, bw2, c0, c1);
            if (TRACK) {
                if (first) {
                    best[u][ch] = c0;
                    bi[u][ch] = __uint_as_float((uint32_t)W);
                    acs_update<W + 1>(best[u][ch], bi[u][ch], c1, zr);
                } else if (Geo<K>::PAIR_UPDATE) {
                    acs_update_pair<W>(best[u][ch], bi[u][ch], c0, c1, zr);
                } else {
                    acs_update<W>(best[u][ch], bi[u][ch], c0, zr);
                    acs_update<W + 1>(best[u][ch], bi[u][ch], c1, zr);
                }
            } else {
                best[u][ch] = first ? fminf(c0, c1) : min3(best[u][ch], c0, c1);
            }
        }
    }
};

template <int K, int W, int NJ, int NCH, bool TRACK>
struct AcsLoop {
    static __device__ __forceinline__ void run(const __half2 (&f2)[64], float x,
                                               const float (&bin)[1 << K], int b,
                                               float (&best)[NJ][NCH], float (&bi)[NJ][NCH],
                                               float zr) {
        uint64_t bw2;
        asm("mov.b64 %0, {%1, %2};" : "=l"(bw2) : "f"(bin[W]), "f"(bin[W + 1]));
        AcsPair<K, W, NJ, NCH, TRACK>::run(f2, x, bw2, b, best, bi, zr);
        AcsLoop<K, W + 2, NJ, NCH, TRACK>::run(f2, x, bin, b, best, bi, zr);
    }
};
template <int K, int NJ, int NCH, bool TRACK>
struct AcsLoop<K, (1 << K), NJ, NCH, TRACK> {
    static __device__ __forceinline__ void run(const __half2 (&)[64], float,
                                               const float (&)[1 << K], int,
                                               float (&)[NJ][NCH], float (&)[NJ][NCH],
                                               float) {}
};

// Butterfly inputs best_i[m + w*P], w < 2^K, into registers.
template <int K>
__device__ __forceinline__ void vit_load_bin(const float* __restrict__ Bc, int m,
                                             float (&bin)[1 << K]) {
    using G = Geo<K>;
    if (G::TRANSPOSED) {
#pragma unroll
        for (int w4 = 0; w4 < G::NC; w4 += 4) {
            const float4 q = *reinterpret_cast<const float4*>(&Bc[G::baddr(m) + w4]);
            bin[w4] = q.x; bin[w4 + 1] = q.y; bin[w4 + 2] = q.z; bin[w4 + 3] = q.w;
        }
    } else {
#pragma unroll
        for (int w = 0; w < G::NC; ++w) bin[w] = Bc[m + w * G::P];
    }
}

// One trellis step: best_{i+1} = min-plus over this thread's states using
// best_i (Bc) and target x; writes best_{i+1} (Bn), returns packed argmins
// (output e's argmin w in bits [e*BPE, e*BPE + BPE)); 0 when !TRACK.
// grow (untraced steps of the slice geometries, K >= 4; the lazy pass uses it
// at K >= 5): also store this thread's outputs to a global row in natural
// index order -- contiguous NJ floats per thread, one or two vector stores.
template <int K, bool TRACK = true>
__device__ __forceinline__ uint64_t vit_step(const __half2 (&f2)[64], float x,
                                             const float* __restrict__ Bc,
                                             float* __restrict__ Bn, int t, float zr,
                                             float* __restrict__ grow = nullptr) {
    using G = Geo<K>;
    constexpr int NCH = G::NCH;
    constexpr int NJ = G::NJ;
    uint64_t bits = 0;
#pragma unroll
    for (int b = 0; b < G::NB; ++b) {
        const int m = G::bfly(t, b);
        float best[NJ][NCH];
        float bi[NJ][NCH];
        float bin[1 << K];
        vit_load_bin<K>(Bc, m, bin);
        AcsLoop<K, 0, NJ, NCH, TRACK>::run(f2, x, bin, b, best, bi, zr);
        float outv[NJ];
#pragma unroll
        for (int u = 0; u < NJ; ++u) {
            float bv = best[u][0];
            const int e = b * NJ + u;
            if (TRACK) {
                float bx = bi[u][0];
#pragma unroll
                for (int ch = 1; ch < NCH; ++ch) {   // (value, index) lexicographic
                    const bool take =
                        best[u][ch] < bv || (best[u][ch] == bv && bi[u][ch] < bx);
                    bv = take ? best[u][ch] : bv;
                    bx = take ? bi[u][ch] : bx;
                }
                bits |= static_cast<uint64_t>(__float_as_uint(bx)) << (e * G::BPE);
            } else {
#pragma unroll
                for (int ch = 1; ch < NCH; ++ch) bv = fminf(bv, best[u][ch]);
            }
            outv[u] = bv;
        }
#pragma unroll
        for (int u = 0; u < NJ; ++u) Bn[G::baddr(G::out_j(t, b * NJ + u))] = outv[u];
        if (!TRACK && !G::WHOLE && grow != nullptr) {
            float* dst = grow + G::out_j(t, 0);
            if (NJ >= 4) {
#pragma unroll
                for (int q = 0; q < NJ / 4; ++q)
                    reinterpret_cast<float4*>(dst)[q] =
                        make_float4(outv[(4 * q) % NJ], outv[(4 * q + 1) % NJ],
                                    outv[(4 * q + 2) % NJ], outv[(4 * q + 3) % NJ]);
            } else if (NJ == 2) {
                *reinterpret_cast<float2*>(dst) = make_float2(outv[0], outv[1 % NJ]);
            } else {
                dst[0] = outv[0];
            }
        }
    }
    return bits;
}

template <int K>
__device__ __forceinline__ void vit_store_bits(uint8_t* __restrict__ row,
                                               uint64_t bits, int t) {
    using G = Geo<K>;
    if (G::BPTB == 8) reinterpret_cast<uint64_t*>(row)[t] = bits;
    else if (G::BPTB == 4) reinterpret_cast<uint32_t*>(row)[t] = (uint32_t)bits;
    else if (G::BPTB == 2) reinterpret_cast<uint16_t*>(row)[t] = (uint16_t)bits;
    else row[t] = (uint8_t)bits;
}

__device__ __forceinline__ void lex_min(float& c, int& s, float oc, int os) {
    const bool take = oc < c || (oc == c && os < s);
    c = take ? oc : c;
    s = take ? os : s;
}

// One Viterbi pass over `nsteps` targets xs[(i - rol) & 255].
//   overlap < 0 : free boundary;  >= 0 : s_0>>K and s_last mod 2^(16-K) pinned.
//   stop        : traceback ends at step `stop` (state returned).
//   st          : if non-null, receives states[0..nsteps) (pass 2).
// bp: this CTA's global backpointer rows [256][BP_ROW].  All threads return
// the state at step `stop`.
template <int K>
__device__ __forceinline__ int vit_pass(const __half2 (&f2)[64], char* smem, int rol,
                        int nsteps, int overlap, int stop, int32_t* st,
                        uint8_t* __restrict__ bp, int t) {
    using G = Geo<K>;
    using SM = VitSmem<K>;
    float* Bc = reinterpret_cast<float*>(smem + SM::OFF_B0);
    float* Bn = reinterpret_cast<float*>(smem + SM::OFF_B1);
    const float* xs = reinterpret_cast<const float*>(smem + SM::OFF_X);
    float* redc = reinterpret_cast<float*>(smem + SM::OFF_RED);
    int* reds = reinterpret_cast<int*>(smem + SM::OFF_RED + 64);
    int* bcast = reinterpret_cast<int*>(smem + SM::OFF_RED + 128);
    float* zword = reinterpret_cast<float*>(smem + SM::OFF_RED + 192);
    const float INF = __int_as_float(0x7f800000);
    if (t == 0) *zword = 0.0f;

    // best_0: 0 (free) or 0 at `overlap`, +inf elsewhere -> cost_0 = E_0 + mask
    for (int idx = t; idx < G::SPRE; idx += kVT)
        Bc[G::baddr(idx)] = (overlap < 0 || idx == overlap) ? 0.0f : INF;
    __syncthreads();
    float zr;
    asm volatile("ld.volatile.shared.f32 %0, [%1];" : "=f"(zr)
                 : "r"((uint32_t)__cvta_generic_to_shared(zword)));

    // steps whose backpointer row lies at or before `stop` are never traced
    // back through: minimum only
    const int nfree = min(max(stop, 0), nsteps - 1);
    for (int i = 0; i < nfree; ++i) {
        const float x = xs[(i - rol) & 255];
        vit_step<K, false>(f2, x, Bc, Bn, t, zr);
        float* tmp = Bc; Bc = Bn; Bn = tmp;
        __syncthreads();
    }
    for (int i = nfree; i < nsteps - 1; ++i) {
        const float x = xs[(i - rol) & 255];
        const uint64_t bits = vit_step<K>(f2, x, Bc, Bn, t, zr);
        vit_store_bits<K>(bp + (size_t)(i + 1) * G::BP_ROW, bits, t);
        float* tmp = Bc; Bc = Bn; Bn = tmp;
        __syncthreads();
    }

    // Final argmin over cost_{n-1}(s), lowest s on ties (torch.argmin).  One
    // more step gives best_n[j] = min_w cost_{n-1}(j + w*2^(16-K)) with the
    // first w attaining it, i.e. the lowest state of group j at that value;
    // the lexicographic (value, state) minimum over all groups is the global
    // first-index argmin.  Pass 2's end mask (s mod 2^(16-K) == overlap, +inf
    // elsewhere) keeps only group j == overlap.
    {
        const float x = xs[(nsteps - 1 - rol) & 255];
        const uint64_t bits = vit_step<K>(f2, x, Bc, Bn, t, zr);
        float bc = INF;
        int bs = 0x7fffffff;
#pragma unroll
        for (int e = 0; e < G::NOUT; ++e) {
            const int j = G::out_j(t, e);
            float v = Bn[G::baddr(j)];
            if (overlap >= 0 && j != overlap) v = INF;
            const int w = (int)((bits >> (e * G::BPE)) & ((1u << G::BPE) - 1u));
            lex_min(bc, bs, v, j + (w << (16 - K)));
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float oc = __shfl_xor_sync(0xffffffffu, bc, off);
            const int os = __shfl_xor_sync(0xffffffffu, bs, off);
            lex_min(bc, bs, oc, os);
        }
        if ((t & 31) == 0) { redc[t >> 5] = bc; reds[t >> 5] = bs; }
        __syncthreads();
    }

    // traceback (thread 0), backpointer rows staged through shared memory
    int s = 0;
    if (t == 0) {
        float bc = redc[0];
        s = reds[0];
        for (int wv = 1; wv < kVT / 32; ++wv) lex_min(bc, s, redc[wv], reds[wv]);
        if (st) st[nsteps - 1] = s;
    }
    uint8_t* tb = reinterpret_cast<uint8_t*>(smem + SM::OFF_TB);
    int hi = nsteps - 1;
    while (hi > stop) {
        const int lo = max(stop + 1, hi - G::TB_ROWS + 1);
        const int n16 = (hi - lo + 1) * (G::BP_ROW / 16);
        const uint4* src = reinterpret_cast<const uint4*>(bp + (size_t)lo * G::BP_ROW);
        uint4* dst = reinterpret_cast<uint4*>(tb);
        for (int q = t; q < n16; q += kVT) dst[q] = src[q];
        __syncthreads();
        if (t == 0) {
            for (int i = hi; i >= lo; --i) {
                const int j = s >> K;
                const int w = G::bp_read(tb + (size_t)(i - lo) * G::BP_ROW, j);
                s = j + (w << (16 - K));
                if (st) st[i - 1] = s;
            }
        }
        __syncthreads();
        hi = lo - 1;
    }
    if (t == 0) *bcast = s;
    __syncthreads();
    const int out = *bcast;
    __syncthreads();
    return out;
}

// Full tail-biting encode of the tile whose 256 targets sit in smem OFF_X.
// Writes the 256 pass-2 states to smem OFF_ST.
template <int K>
__device__ __forceinline__ void vit_tailbite(const __half2 (&f2)[64], char* smem,
                                             int pivot, int margin,
                                             uint8_t* __restrict__ bp, int t) {
    using SM = VitSmem<K>;
    int32_t* st = reinterpret_cast<int32_t*>(smem + SM::OFF_ST);
    const int n1 = (margin > 0 && pivot + margin < kSteps) ? pivot + margin : kSteps;
    const int sp = vit_pass<K>(f2, smem, pivot, n1, -1, pivot, nullptr, bp, t);
    vit_pass<K>(f2, smem, 0, kSteps, sp >> K, 0, st, bp, t);
}

}  // namespace exl3b
