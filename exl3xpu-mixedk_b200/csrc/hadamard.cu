// hadamard.cu -- block-128 random-sign Hadamard incoherence on device.
//
// Reference: quantize/quantize.py:125-176 (hadamard128, had_left, had_right,
// to_inner, from_inner, rotate_hessian).  Every transform there is two-sided
// with block-diagonal normalised Sylvester H_128, so each 128x128 block of
// the matrix transforms independently:
//     Y_blk = post_c * ( mid_r * (H . (pre_r * X_blk * pre_c)) ) . H
// One CTA owns one block: coalesced load (optionally transposed) into padded
// shared memory, fast Walsh-Hadamard butterflies along columns then rows
// (4 values per lane, 2 in-register levels + 5 shuffle levels), one exact
// 2^-7 scale for the two 1/sqrt(128) factors, coalesced store (optionally
// transposed).  HBM-bound: one read and one write per element.
// The butterfly order differs from the reference's fp32 GEMM, so results
// agree to fp32 rounding, not bit for bit.
#include "exl3b_internal.h"

namespace exl3b {

constexpr int kHB = 128;          // Hadamard block
constexpr int kHT = 512;          // threads per CTA
constexpr int kHLD = kHB + 1;     // padded smem row

template <typename T> __device__ __forceinline__ float to_f(T v);
template <> __device__ __forceinline__ float to_f<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) {
    return __bfloat162float(v);
}
template <> __device__ __forceinline__ float to_f<__half>(__half v) { return __half2float(v); }

// 128-point unnormalised WHT of 4 values per lane: element e = lane + 32 q.
__device__ __forceinline__ void fwht128(float (&v)[4], int lane) {
    // index bits 6 (q>>1) and 5 (q&1) are inside the lane
    const float a = v[0] + v[2], b = v[0] - v[2];   // bit 6: pairs (0,2) (1,3)
    const float c = v[1] + v[3], d = v[1] - v[3];
    v[0] = a + c; v[1] = a - c; v[2] = b + d; v[3] = b - d;   // bit 5
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) {
        const bool hi = lane & s;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float o = __shfl_xor_sync(0xffffffffu, v[q], s);
            v[q] = hi ? (o - v[q]) : (v[q] + o);
        }
    }
}


template <typename T>
__global__ void __launch_bounds__(kHT)
had2_kernel(HadParams p) {
    extern __shared__ float tile[];   // [128][129]
    const int rb = blockIdx.y, cb = blockIdx.x;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const T* X = static_cast<const T*>(p.X);
    const int r0 = rb * kHB, c0 = cb * kHB;

    // load: coalesced along the input's contiguous axis
    for (int idx = t; idx < kHB * kHB; idx += kHT) {
        const int a = idx / kHB, b = idx % kHB;     // b contiguous in memory
        int r, c;
        float v;
        if (p.trans_in) {                            // X[c][r], r contiguous
            r = b; c = a;
            v = to_f<T>(X[(size_t)(c0 + c) * p.ldx + (r0 + r)]);
        } else {
            r = a; c = b;
            v = to_f<T>(X[(size_t)(r0 + r) * p.ldx + (c0 + c)]);
        }
        v = v * p.pre_scale;
        if (p.pre_scale_dev) v = v * p.pre_scale_dev[0];
        if (p.pre_r) v = v * p.pre_r[r0 + r];
        if (p.pre_c) v = v * p.pre_c[c0 + c];
        if (p.pre_r_div) v = v / p.pre_r_div[r0 + r];
        if (p.pre_c_div) v = v / p.pre_c_div[c0 + c];
        tile[r * kHLD + c] = v;
    }
    __syncthreads();
    // transform along r (each column); 16 warps x 8 columns
    for (int c = warp; c < kHB; c += kHT / 32) {
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = tile[(lane + 32 * q) * kHLD + c];
        if (!p.skip_left) fwht128(v, lane);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const int r = lane + 32 * q;
            float o = v[q];
            if (p.mid_r) o = o * p.mid_r[r0 + r];
            tile[r * kHLD + c] = o;
        }
    }
    __syncthreads();
    // transform along c (each row)
    for (int r = warp; r < kHB; r += kHT / 32) {
        float v[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) v[q] = tile[r * kHLD + lane + 32 * q];
        if (!p.skip_right) fwht128(v, lane);
#pragma unroll
        for (int q = 0; q < 4; ++q) tile[r * kHLD + lane + 32 * q] = v[q];
    }
    __syncthreads();
    // normalisation: 1/sqrt(128) per applied transform; both -> exact 2^-7
    const float norm = (p.skip_left || p.skip_right)
                           ? ((p.skip_left && p.skip_right) ? 1.0f : 0.08838834764831845f)
                           : 0.0078125f;
    // store (x 2^-7 exact), optional post multiplier, sum of squares
    double ss = 0.0;
    for (int idx = t; idx < kHB * kHB; idx += kHT) {
        const int a = idx / kHB, b = idx % kHB;
        int r, c;
        if (p.trans_out) { c = a; r = b; } else { r = a; c = b; }
        float v = tile[r * kHLD + c] * norm;
        if (p.post_c) v = v * p.post_c[c0 + c];
        if (p.trans_out) p.Y[(size_t)(c0 + c) * p.ldy + (r0 + r)] = v;
        else p.Y[(size_t)(r0 + r) * p.ldy + (c0 + c)] = v;
        ss += (double)v * (double)v;
    }
    if (p.row_sumsq) {   // per-row partials over this block's 128 columns
        __syncthreads();
        for (int r = warp; r < kHB; r += kHT / 32) {
            double rs = 0.0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float v = tile[r * kHLD + lane + 32 * q] * norm;
                rs += (double)v * (double)v;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
            if (lane == 0) p.row_sumsq[(size_t)(r0 + r) * gridDim.x + cb] = rs;
        }
    }
    if (p.sumsq) {
        __shared__ double red[kHT / 32];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        if (t == 0) {
            double s = 0.0;
            for (int w = 0; w < kHT / 32; ++w) s += red[w];
            p.sumsq[(size_t)rb * gridDim.x + cb] = s;
        }
    }
}

int launch_had2(const HadParams& p, cudaStream_t stream) {
    if (p.rows % kHB || p.cols % kHB || p.rows <= 0 || p.cols <= 0) {
        set_error("Hadamard dims %dx%d must be positive multiples of 128", p.rows, p.cols);
        return RC_BAD_REQUEST;
    }
    const int smem = kHB * kHLD * sizeof(float);
    dim3 grid(p.cols / kHB, p.rows / kHB);
    static bool attr[kMaxDevices][3] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    switch (p.in_dtype) {
        case 0:
            if (!attr[dev][0]) {
                cudaFuncSetAttribute(had2_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
                attr[dev][0] = true;
            }
            had2_kernel<float><<<grid, kHT, smem, stream>>>(p);
            break;
        case 1:
            if (!attr[dev][1]) {
                cudaFuncSetAttribute(had2_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
                attr[dev][1] = true;
            }
            had2_kernel<__nv_bfloat16><<<grid, kHT, smem, stream>>>(p);
            break;
        case 2:
            if (!attr[dev][2]) {
                cudaFuncSetAttribute(had2_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
                attr[dev][2] = true;
            }
            had2_kernel<__half><<<grid, kHT, smem, stream>>>(p);
            break;
        default:
            set_error("input dtype id %d", p.in_dtype);
            return RC_BAD_REQUEST;
    }
    note_launch();
    return check_cuda(cudaGetLastError(), "had2_kernel launch") ? RC_DEVICE_ERROR : RC_OK;
}

// ------------------------------------------------------------ one-sided
// had_left / had_right (quantize.py:135-146): the block-128 Hadamard along one
// axis of X [rows][cols] only, so the other axis needs no multiple of 128.
// fl32(1/sqrt(128)) is applied once after the butterflies (the reference's
// fp32 GEMM with the normalised matrix rounds differently: agreement to fp32
// rounding, like the two-sided transforms).
constexpr float kInvSqrt128 = 0.08838834764831845f;

// along the last axis: one warp per contiguous 128-vector, 4 values per lane
__global__ void __launch_bounds__(256)
had_last_kernel(const float* __restrict__ X, float* __restrict__ Y, size_t nvec) {
    const size_t v = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (v >= nvec) return;
    const float* x = X + v * kHB;
    float a[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) a[q] = x[lane + 32 * q];
    fwht128(a, lane);
    float* y = Y + v * kHB;
#pragma unroll
    for (int q = 0; q < 4; ++q) y[lane + 32 * q] = a[q] * kInvSqrt128;
}

// along the first axis: a CTA stages a 128-row x 32-column tile (coalesced
// along the columns), each of its 8 warps transforms 4 columns
__global__ void __launch_bounds__(256)
had_first_kernel(const float* __restrict__ X, float* __restrict__ Y, int cols) {
    __shared__ float tile[kHB][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * kHB;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c = c0 + lane;
    for (int r = warp; r < kHB; r += 8)
        tile[r][lane] = c < cols ? X[(size_t)(r0 + r) * cols + c] : 0.0f;
    __syncthreads();
    for (int j = warp; j < 32; j += 8) {
        float a[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) a[q] = tile[lane + 32 * q][j];
        fwht128(a, lane);
#pragma unroll
        for (int q = 0; q < 4; ++q) tile[lane + 32 * q][j] = a[q] * kInvSqrt128;
    }
    __syncthreads();
    if (c < cols)
        for (int r = warp; r < kHB; r += 8) Y[(size_t)(r0 + r) * cols + c] = tile[r][lane];
}

int launch_had_axis(const float* X, int rows, int cols, int axis, float* Y,
                    cudaStream_t stream) {
    if (rows <= 0 || cols <= 0 || (axis == 0 ? rows : cols) % kHB || axis < 0 || axis > 1) {
        set_error("Hadamard along axis %d of [%d, %d]: that dim must be a positive "
                  "multiple of 128", axis, rows, cols);
        return RC_BAD_REQUEST;
    }
    if (axis == 1) {
        const size_t nvec = (size_t)rows * (cols / kHB);
        had_last_kernel<<<(unsigned)((nvec * 32 + 255) / 256), 256, 0, stream>>>(X, Y, nvec);
    } else {
        dim3 grid((cols + 31) / 32, rows / kHB);
        had_first_kernel<<<grid, 256, 0, stream>>>(X, Y, cols);
    }
    note_launch();
    return check_cuda(cudaGetLastError(), "one-sided Hadamard launch") ? RC_DEVICE_ERROR : RC_OK;
}

// ------------------------------------------------------------ channel scales
// EXL3 per-channel magnitude folds (quantize.py:785-800, 854-862, 1025-1041).

// rms[r] = fl32(sqrt(fl32(mean_c X[r][c]^2)))   (one warp per row)
template <typename T>
__global__ void row_rms_kernel(const T* __restrict__ X, int rows, int cols,
                               float* __restrict__ rms) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= rows) return;
    double s = 0.0;
    for (int c = lane; c < cols; c += 32) {
        const float v = to_f<T>(X[(size_t)warp * cols + c]);
        s += (double)v * (double)v;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) rms[warp] = sqrtf((float)(s / cols));
}

int launch_row_rms(const void* X, int dtype, int rows, int cols, float* rms, cudaStream_t stream) {
    const int grid = (rows * 32 + 255) / 256;
    switch (dtype) {
        case 0: row_rms_kernel<float><<<grid, 256, 0, stream>>>((const float*)X, rows, cols, rms); break;
        case 1: row_rms_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>((const __nv_bfloat16*)X, rows, cols, rms); break;
        case 2: row_rms_kernel<__half><<<grid, 256, 0, stream>>>((const __half*)X, rows, cols, rms); break;
        default: set_error("dtype %d", dtype); return RC_BAD_REQUEST;
    }
    note_launch();
    return check_cuda(cudaGetLastError(), "row_rms launch") ? RC_DEVICE_ERROR : RC_OK;
}

// r_out /= mean(r_out) (if > 1e-30); zero_out -> 0.1; div_c = sv * r_out;
// store_c = zero_out ? 0 : r_out   (one CTA)
__global__ void chan_out_kernel(float* __restrict__ r_out, const float* __restrict__ sv, int n,
                                float* __restrict__ div_c, float* __restrict__ store_c) {
    __shared__ double red[32];
    __shared__ float rm;
    double s = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += r_out[i];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
        rm = (float)(tot / n);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        float r = r_out[i];
        if (rm > 1e-30f) r = r / rm;
        const bool zero = fabsf(r) < 1e-30f;
        const float rr = zero ? 0.1f : r;
        r_out[i] = rr;
        div_c[i] = sv[i] * rr;
        store_c[i] = zero ? 0.0f : rr;
    }
}

int launch_chan_out(float* r_out, const float* sv, int n, float* div_c, float* store_c,
                    cudaStream_t stream) {
    chan_out_kernel<<<1, 1024, 0, stream>>>(r_out, sv, n, div_c, store_c);
    note_launch();
    return check_cuda(cudaGetLastError(), "chan_out launch") ? RC_DEVICE_ERROR : RC_OK;
}

// r_in[k] = sqrt(mean over n); < 1e-30 -> 0.1; div_r = su * r_in
__global__ void chan_in_kernel(const double* __restrict__ parts, int k, int nparts, int ncols,
                               const float* __restrict__ su, float* __restrict__ r_in,
                               float* __restrict__ div_r) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= k) return;
    double s = 0.0;
    for (int j = 0; j < nparts; ++j) s += parts[(size_t)i * nparts + j];
    float r = sqrtf((float)(s / ncols));
    r = fabsf(r) < 1e-30f ? 0.1f : r;
    r_in[i] = r;
    div_r[i] = su[i] * r;
}

int launch_chan_in(const double* row_parts, int k, int nparts, const float* su, float* r_in,
                   float* div_r, cudaStream_t stream) {
    chan_in_kernel<<<(k + 255) / 256, 256, 0, stream>>>(row_parts, k, nparts, nparts * 128,
                                                        su, r_in, div_r);
    note_launch();
    return check_cuda(cudaGetLastError(), "chan_in launch") ? RC_DEVICE_ERROR : RC_OK;
}

// stored EXL3 fields: suh = half(su * r_in * Wscale), svh = half(sv * store_c)
__global__ void chan_store_kernel(const float* __restrict__ su, const float* __restrict__ r_in,
                                  const float* __restrict__ wscale, const float* __restrict__ sv,
                                  const float* __restrict__ store_c, int k, int n,
                                  __half* __restrict__ suh, __half* __restrict__ svh) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const float ws = wscale ? wscale[0] : 1.0f;
    if (i < k) suh[i] = __float2half_rn((su[i] * r_in[i]) * ws);
    if (i < n) svh[i] = __float2half_rn(sv[i] * store_c[i]);
}

int launch_chan_store(const float* su, const float* r_in, const float* wscale,
                      const float* sv, const float* store_c, int k, int n,
                      __half* suh, __half* svh, cudaStream_t stream) {
    const int m = k > n ? k : n;
    chan_store_kernel<<<(m + 255) / 256, 256, 0, stream>>>(su, r_in, wscale, sv, store_c, k, n,
                                                           suh, svh);
    note_launch();
    return check_cuda(cudaGetLastError(), "chan_store launch") ? RC_DEVICE_ERROR : RC_OK;
}

// ------------------------------------------------------------ transposes
// quantize() harness path (quantize.py:933-942, 961-965):
//   fwd: Y[k][n] = X[n][k] / (row[n] * col[k])        (mags nullable -> 1)
//   inv: Y[n][k] = (X[k][n] * s) * (row[n] * col[k])
// 32x32 smem tiles; optional per-CTA sum of squares of Y (fwd).
template <bool INV>
__global__ void __launch_bounds__(256)
transpose_scale_kernel(const float* __restrict__ X, int rows_x, int cols_x,
                       const float* __restrict__ rmag, const float* __restrict__ cmag,
                       const float* __restrict__ s, float* __restrict__ Y,
                       double* __restrict__ sumsq) {
    __shared__ float tile[32][33];
    const int bx = blockIdx.x * 32, by = blockIdx.y * 32;   // x: cols of X
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 8 rows per pass
    for (int r = ty; r < 32; r += 8) {
        const int gr = by + r, gc = bx + tx;
        float v = 0.0f;
        if (gr < rows_x && gc < cols_x) v = X[(size_t)gr * cols_x + gc];
        tile[r][tx] = v;
    }
    __syncthreads();
    double ss = 0.0;
    for (int r = ty; r < 32; r += 8) {
        const int gy = bx + r, gx = by + tx;        // Y[gy][gx] = X[gx][gy]
        if (gy < cols_x && gx < rows_x) {
            float v = tile[tx][r];
            if (!INV) {
                // Y[k][n] from X[n][k]: X row index = n (gx), col = k (gy)
                const float m = (rmag ? rmag[gx] : 1.0f) * (cmag ? cmag[gy] : 1.0f);
                if (rmag || cmag) v = v / m;
            } else {
                // Y[n][k] from X[k][n]: X row = k (gx), col = n (gy)
                v = v * s[0];
                if (rmag || cmag) v = v * ((rmag ? rmag[gy] : 1.0f) * (cmag ? cmag[gx] : 1.0f));
            }
            Y[(size_t)gy * rows_x + gx] = v;
            ss += (double)v * (double)v;
        }
    }
    if (sumsq) {
        __shared__ double red[8];
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
        if (tx == 0) red[ty] = ss;
        __syncthreads();
        if (threadIdx.x == 0) {
            double t = 0.0;
            for (int w = 0; w < 8; ++w) t += red[w];
            sumsq[(size_t)blockIdx.y * gridDim.x + blockIdx.x] = t;
        }
    }
}

int launch_transpose_scale(bool inv, const float* X, int rows_x, int cols_x,
                           const float* rmag, const float* cmag, const float* s,
                           float* Y, double* sumsq, cudaStream_t stream) {
    dim3 grid((cols_x + 31) / 32, (rows_x + 31) / 32);
    if (inv) transpose_scale_kernel<true><<<grid, 256, 0, stream>>>(X, rows_x, cols_x, rmag, cmag, s, Y, sumsq);
    else transpose_scale_kernel<false><<<grid, 256, 0, stream>>>(X, rows_x, cols_x, rmag, cmag, s, Y, sumsq);
    note_launch();
    return check_cuda(cudaGetLastError(), "transpose_scale launch") ? RC_DEVICE_ERROR : RC_OK;
}

// ------------------------------------------------------------ reductions
// Deterministic sum of n doubles (one CTA, fixed order) -> out[0].
__global__ void sum_f64_kernel(const double* __restrict__ in, int n, double* __restrict__ out) {
    __shared__ double red[1024 / 32];
    double s = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += in[i];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
        out[0] = tot;
    }
}

// scale = fl32(sqrt(fl32(sumsq / count))) / lut_rms  (quantize.py:803, :941)
__global__ void rms_scale_kernel(const double* __restrict__ sumsq, double count,
                                 float lut_rms, float* __restrict__ scale) {
    const float mean = (float)(sumsq[0] / count);
    scale[0] = sqrtf(mean) / lut_rms;
}

// y = x / s[0] elementwise (fp32 IEEE division), n4 float4 groups.
__global__ void div_scalar_kernel(const float4* __restrict__ x, const float* __restrict__ s,
                                  float4* __restrict__ y, size_t n4) {
    const float d = s[0];
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += (size_t)gridDim.x * blockDim.x) {
        float4 v = x[i];
        v.x = v.x / d; v.y = v.y / d; v.z = v.z / d; v.w = v.w / d;
        y[i] = v;
    }
}

int launch_rms_scale(const double* partials, int nparts, double count, float lut_rms,
                     double* tmp1, float* scale, cudaStream_t stream) {
    sum_f64_kernel<<<1, 1024, 0, stream>>>(partials, nparts, tmp1);
    rms_scale_kernel<<<1, 1, 0, stream>>>(tmp1, count, lut_rms, scale);
    note_launch(2);
    return check_cuda(cudaGetLastError(), "rms_scale launch") ? RC_DEVICE_ERROR : RC_OK;
}

int launch_div_scalar(const float* x, const float* s, float* y, size_t n, cudaStream_t stream) {
    if (n % 4) { set_error("div_scalar size %zu not a multiple of 4", n); return RC_BAD_REQUEST; }
    const size_t n4 = n / 4;
    int grid = (int)((n4 + 255) / 256);
    if (grid > 148 * 16) grid = 148 * 16;
    div_scalar_kernel<<<grid, 256, 0, stream>>>(reinterpret_cast<const float4*>(x), s,
                                                reinterpret_cast<float4*>(y), n4);
    note_launch();
    return check_cuda(cudaGetLastError(), "div_scalar launch") ? RC_DEVICE_ERROR : RC_OK;
}

// ------------------------------------------------------------ Hessian damping
// quantize.py:810-814: dead diagonal entries -> 1, then diag += percdamp *
// mean(diag).  One CTA: the mean in double, rounded to fp32 like torch's
// fp32 result; damp = fl32(percdamp_f32 * mean).
__global__ void damp_kernel(float* __restrict__ G, int k, float percdamp,
                            int* __restrict__ nonfinite) {
    __shared__ double red[32];
    __shared__ float damp;
    double s = 0.0;
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        float d = G[(size_t)i * k + i];
        if (d == 0.0f) { d = 1.0f; G[(size_t)i * k + i] = d; }
        s += d;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
        damp = percdamp * (float)(tot / k);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < k; i += blockDim.x) {
        float* d = &G[(size_t)i * k + i];
        *d = *d + damp;
    }
}

// fallback escalation (quantize.py:824-826): diag += extra * mean(diag), fp64
__global__ void damp_f64_kernel(double* __restrict__ G, int k, double extra) {
    __shared__ double red[32];
    __shared__ double add;
    double s = 0.0;
    for (int i = threadIdx.x; i < k; i += blockDim.x) s += G[(size_t)i * k + i];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double tot = 0.0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) tot += red[w];
        add = extra * (tot / k);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < k; i += blockDim.x) G[(size_t)i * k + i] += add;
}

int launch_damp_f64(double* G, int k, double extra, cudaStream_t stream) {
    damp_f64_kernel<<<1, 1024, 0, stream>>>(G, k, extra);
    note_launch();
    return check_cuda(cudaGetLastError(), "damp_f64 launch") ? RC_DEVICE_ERROR : RC_OK;
}

// count of non-finite entries (quantize.py:821 torch.isfinite(G).all())
__global__ void count_nonfinite_kernel(const float* __restrict__ G, size_t n, int* __restrict__ cnt) {
    int c = 0;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x)
        c += isfinite(G[i]) ? 0 : 1;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
    if ((threadIdx.x & 31) == 0 && c) atomicAdd(cnt, c);
}

int launch_count_nonfinite(const float* G, size_t n, int* cnt, cudaStream_t stream) {
    cudaMemsetAsync(cnt, 0, sizeof(int), stream);
    count_nonfinite_kernel<<<148 * 4, 256, 0, stream>>>(G, n, cnt);
    note_launch();
    return check_cuda(cudaGetLastError(), "count_nonfinite launch") ? RC_DEVICE_ERROR : RC_OK;
}

int launch_damp(float* G, int k, float percdamp, cudaStream_t stream) {
    damp_kernel<<<1, 1024, 0, stream>>>(G, k, percdamp, nullptr);
    note_launch();
    return check_cuda(cudaGetLastError(), "damp launch") ? RC_DEVICE_ERROR : RC_OK;
}

}  // namespace exl3b
