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
// 128-row buffers; per k-block one tile kernel over its column tiles (waves
// of at most one CTA per SM); after a buffer, prod[:16lo] += Lfac[buf, :16lo]^T
// E[buf].  Columns never interact (Lfac couples rows only), so each CTA owns
// one column tile of the current k-block:
//   WXWX = (Wq + Lfac[later, blk]^T . E[later]) + prod     (quantize.py:676-682)
//   x[t] = WXWX[perm[t]]                                   (:684-686)
//   states = tail-biting encode(x)                         (:687-731)
//   hatW[perm[t]] = lut[states[t]], E = Wq - hatW          (:736-741)
//   trellis = pack(states)                                 (:846, :360-378)
#include <string.h>

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
    int i;                  // k-block
    int cur;                // buffer end block (exclusive)
    int c_base;             // first column tile of this wave
    int pivot, margin;
    int nseg;
    int seg_c0[kMaxSeg + 1];     // segment column-tile starts, seg_c0[nseg] = tn
    int seg_K[kMaxSeg];
    int16_t* seg_trellis[kMaxSeg];
    int32_t* states;        // [tk][tn][256] or null
    float* xout;            // [tk][tn][256] or null (encoder targets, for checks)
    uint8_t* bp_ws;         // wave slots
    size_t bp_slot;         // bytes per slot
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

template <int K>
__device__ __forceinline__ void ldlq_tile_body(const LdlqTileParams& p, char* smem,
                                               int c, int seg) {
    using SM = VitSmem<K>;
    const int t = threadIdx.x;
    float* xs = reinterpret_cast<float*>(smem + SM::OFF_X);
    float* wx = reinterpret_cast<float*>(smem + SM::OFF_TB);   // 16x16 staging
    const int tn = p.seg_c0[p.nseg];
    const size_t n = (size_t)p.n;

    // ---- feedback: WXWX tile
    if (t < 256) {
        const int a = t >> 4, col = t & 15;
        const size_t row = (size_t)(16 * p.i + a);
        const size_t gc = (size_t)(16 * c + col);
        float w = p.Wq[row * n + gc];
        if (p.Lfac) {
            const int r_lo = 16 * (p.i + 1), r_hi = 16 * p.cur;
            if (r_lo < r_hi) {
                float acc = 0.0f;
                for (int r = r_lo; r < r_hi; ++r)
                    acc = fmaf(p.Lfac[(size_t)r * p.k + 16 * p.i + a], p.E[(size_t)r * n + gc], acc);
                w = w + acc;
            }
            w = w + p.prod[row * n + gc];
        }
        wx[t] = w;
    }
    __syncthreads();
    if (t < 256) {
        const float x = wx[tc_perm(t)];
        xs[t] = x;
        if (p.xout) p.xout[((size_t)p.i * tn + c) * 256 + t] = x;
    }
    __syncthreads();

    // ---- trellis encode
    {
        __half2 f2[64];
        vit_load_f2tab(f2, p.f2tab[K], t);
        uint8_t* bp = p.bp_ws + (size_t)blockIdx.x * p.bp_slot;
        vit_tailbite<K>(f2, smem, p.pivot, p.margin, bp, t);
    }

    // ---- write-back: decoded tile, error, states
    const int32_t* st = reinterpret_cast<const int32_t*>(smem + SM::OFF_ST);
    if (t < 256) {
        const int s = st[t];
        const int pos = tc_perm(t);
        const size_t idx = (size_t)(16 * p.i + (pos >> 4)) * n + (size_t)(16 * c + (pos & 15));
        const float v = p.lut32[s];
        p.hatW[idx] = v;
        p.E[idx] = p.Wq[idx] - v;
        if (p.states) p.states[((size_t)p.i * tn + c) * 256 + t] = s;
    }
    // ---- pack: stream bit q = t*K + b (MSB first within a symbol); u32 word
    // w holds stream bits [32w, 32w+32) MSB first; stored as int16 low half
    // first (quantize.py:360-378)
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
                       ((size_t)p.i * seg_tn + (c - p.seg_c0[seg])) * (16 * K);
        out[2 * t] = (int16_t)(word & 0xFFFFu);
        out[2 * t + 1] = (int16_t)(word >> 16);
    }
}

__global__ void __launch_bounds__(kVT, 1)
ldlq_tile_kernel(const __grid_constant__ LdlqTileParams p) {
    extern __shared__ __align__(16) char smem[];
    const int c = p.c_base + blockIdx.x;
    int seg = 0;
    while (seg + 1 < p.nseg && c >= p.seg_c0[seg + 1]) ++seg;
    switch (p.seg_K[seg]) {
        case 2: ldlq_tile_body<2>(p, smem, c, seg); break;
        case 3: ldlq_tile_body<3>(p, smem, c, seg); break;
        case 4: ldlq_tile_body<4>(p, smem, c, seg); break;
        case 5: ldlq_tile_body<5>(p, smem, c, seg); break;
        case 6: ldlq_tile_body<6>(p, smem, c, seg); break;
        case 7: ldlq_tile_body<7>(p, smem, c, seg); break;
        default: break;
    }
}

static int max_smem_for(const int* Ks, int nseg) {
    int m = 0;
    for (int s = 0; s < nseg; ++s) {
        int b = 0;
        switch (Ks[s]) {
            case 2: b = VitSmem<2>::BYTES; break;
            case 3: b = VitSmem<3>::BYTES; break;
            case 4: b = VitSmem<4>::BYTES; break;
            case 5: b = VitSmem<5>::BYTES; break;
            case 6: b = VitSmem<6>::BYTES; break;
            case 7: b = VitSmem<7>::BYTES; break;
        }
        m = b > m ? b : m;
    }
    return m;
}

int ldlq_sweep(const SweepArgs& a, cudaStream_t stream) {
    const int tk = a.k / 16, tn = a.n / 16;
    LdlqTileParams p;
    memset(&p, 0, sizeof(p));
    p.Wq = a.Wq; p.E = a.E; p.hatW = a.hatW; p.Lfac = a.Lfac;
    p.prod = a.Lfac ? a.prod : nullptr;
    p.k = a.k; p.n = a.n; p.pivot = a.pivot; p.margin = a.margin;
    p.nseg = a.nseg;
    for (int s = 0; s <= a.nseg; ++s) p.seg_c0[s] = a.seg_c0[s];
    for (int s = 0; s < a.nseg; ++s) { p.seg_K[s] = a.seg_K[s]; p.seg_trellis[s] = a.seg_trellis[s]; }
    p.states = a.states; p.xout = a.xout; p.bp_ws = a.bp_ws; p.bp_slot = a.bp_slot;
    for (int K = 0; K < 8; ++K) p.f2tab[K] = a.f2tab[K];
    p.lut32 = a.lut32;

    const int smem = max_smem_for(a.seg_K, a.nseg);
    static bool attr[kMaxDevices] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!attr[dev]) {
        if (check_cuda(cudaFuncSetAttribute(ldlq_tile_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            VitSmem<2>::BYTES),
                       "cudaFuncSetAttribute(ldlq_tile)"))
            return RC_DEVICE_ERROR;
        attr[dev] = true;
    }
    const int buf_tiles = a.buf_cols / 16 > 0 ? a.buf_cols / 16 : 1;
    // buffers are anchored at tk like the reference: [tk - 8m - 8, tk - 8m)
    for (int cur = tk; cur > 0; cur -= buf_tiles) {
        const int lo = cur - buf_tiles > 0 ? cur - buf_tiles : 0;
        if (lo >= a.block_hi || cur <= a.block_lo) {
            continue;
        }
        p.cur = cur;
        for (int i = cur - 1; i >= lo; --i) {
            if (i >= a.block_hi || i < a.block_lo) continue;
            p.i = i;
            for (int c0 = 0; c0 < tn; c0 += a.wave) {
                const int nb = tn - c0 < a.wave ? tn - c0 : a.wave;
                p.c_base = c0;
                // profiling units: weights encoded by this launch
                prof_begin_launch(stream, PROF_TILE, (double)nb * 256.0);
                ldlq_tile_kernel<<<nb, kVT, smem, stream>>>(p);
                prof_end_launch(stream);
                note_launch();
                if (check_cuda(cudaGetLastError(), "ldlq_tile_kernel launch"))
                    return RC_DEVICE_ERROR;
            }
        }
        if (a.Lfac && lo > 0 && lo >= a.block_lo) {
            // prod[0:16lo, :] += Lfac[16lo:16cur, 0:16lo]^T . E[16lo:16cur, :]
            prof_begin_launch(stream, PROF_GEMM,
                              (double)(16 * lo) * a.n * (16 * (cur - lo)) * 2.0);
            int rc = launch_gemm_tn_acc_f32(16 * lo, a.n, 16 * (cur - lo),
                                            a.Lfac + (size_t)16 * lo * a.k, a.k,
                                            a.E + (size_t)16 * lo * a.n, a.n,
                                            a.prod, a.n, stream);
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

// unpack_states (quantize.py:381-402): state t = the 16-bit circular window
// of the 256K-bit stream ending at bit (t+1)K.
__global__ void unpack_kernel(const int16_t* __restrict__ tr, int nt, int K,
                              int32_t* __restrict__ st) {
    const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (size_t)nt * 256) return;
    const size_t tile = gid / 256;
    const int t = (int)(gid % 256);
    const uint16_t* w16 = reinterpret_cast<const uint16_t*>(tr) + tile * 16 * K;
    const int nbits = 256 * K;
    const int b0 = (t * K + K - 16 + nbits) % nbits;
    uint32_t s = 0;
    for (int j = 0; j < 16; ++j) {
        const int q = (b0 + j) % nbits;
        const int wi = q >> 5, bi = q & 31;
        const uint32_t word = (uint32_t)w16[2 * wi] | ((uint32_t)w16[2 * wi + 1] << 16);
        s = (s << 1) | ((word >> (31 - bi)) & 1u);
    }
    st[gid] = (int32_t)s;
}

// decode_trellis (quantize.py:405-415): trellis [tk][tn][16K] -> W [k][n]
__global__ void decode_kernel(const int16_t* __restrict__ tr, int tk, int tn, int K,
                              const float* __restrict__ lut, float* __restrict__ W) {
    const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (size_t)tk * tn * 256) return;
    const size_t tile = gid / 256;
    const int t = (int)(gid % 256);
    const int i = (int)(tile / tn), c = (int)(tile % tn);
    const uint16_t* w16 = reinterpret_cast<const uint16_t*>(tr) + tile * 16 * K;
    const int nbits = 256 * K;
    const int b0 = (t * K + K - 16 + nbits) % nbits;
    uint32_t s = 0;
    for (int j = 0; j < 16; ++j) {
        const int q = (b0 + j) % nbits;
        const int wi = q >> 5, bi = q & 31;
        const uint32_t word = (uint32_t)w16[2 * wi] | ((uint32_t)w16[2 * wi + 1] << 16);
        s = (s << 1) | ((word >> (31 - bi)) & 1u);
    }
    const int pos = tc_perm(t);
    W[(size_t)(16 * i + (pos >> 4)) * (16 * tn) + (16 * c + (pos & 15))] = lut[s];
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
