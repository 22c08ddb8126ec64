// Activation quantizers feeding the integer-MMA projections.  All of them write
// int8 codes in the F8 B-fragment layout (frag_offset in common.cuh) or, when
// c16_mt > 0, the C16 A-fragment layout of c16_mt token tiles (c16_offset).
//   * HE4 learned-gain/clip codes (Projection.forward, w1a1_eagle/model.py:128-140)
//   * per-token 16-bit fixed point as two int8 planes (pure one-bit-weight blocks)
//   * W1A1 sign binarisation with the fixed-order per-token mean|x|
#include "common.cuh"
#include "kernels.cuh"

namespace bd {

template <typename T>
__device__ __forceinline__ T block_sum_256(T v, T *scratch) {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    T total = scratch[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) total += scratch[w];
    __syncthreads();
    return total;
}

// Grid (rows, ceil(cols / 1024)): each thread quantizes 4 consecutive columns.
// The parameters (gain, norm weight, bound) are read before the dependency
// wait; after it, one round trip brings the thread's columns 4 (t + 256 i) + j
// of the row (i < 4, so rows up to 4096 columns stay in registers) for both the
// rms and the codes.  Code sums go either to partial[row][y] (partial = true,
// no zeroing needed) or, with integer atomics, to a zeroed full[row].
__global__ void __launch_bounds__(256) quantize_codes_kernel(const float *__restrict__ x, int64_t cols, int64_t ld,
                                                             const float *__restrict__ gain,
                                                             const float *__restrict__ bound_ptr, int bits,
                                                             int8_t *__restrict__ codes, int32_t *__restrict__ sums,
                                                             bool partial, int32_t *flags, int32_t *zero_sums,
                                                             int zero_count, const float *__restrict__ norm_w,
                                                             float eps, int c16_mt) {
    __shared__ int scratch[8];
    __shared__ float fpart[8];
    const int row = blockIdx.x;
    const int64_t k0 = static_cast<int64_t>(blockIdx.y) * 1024 + 4 * threadIdx.x;
    float gv[4], nv[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const bool live = k0 + j < cols;
        gv[j] = live ? __ldg(gain + k0 + j) : 0.0f;
        nv[j] = (norm_w && live) ? __ldg(norm_w + k0 + j) : 0.0f;
    }
    const float b = __ldg(bound_ptr);
    grid_wait();
    grid_launch_dependents();
    const float *xr = x + row * cols;
    float v[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t k = 4 * (threadIdx.x + 256 * i) + j;
            v[i][j] = (k < cols && (norm_w || i == static_cast<int>(blockIdx.y))) ? xr[k] : 0.0f;
        }
    // optional rms(x, norm_w, eps) of the whole row first (model.py:50-51, 220)
    float scale = 1.0f;
    if (norm_w) {
        float ss = 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) ss = fmaf(v[i][j], v[i][j], ss);
        for (int64_t k = 4096 + threadIdx.x; k < cols; k += blockDim.x) ss = fmaf(xr[k], xr[k], ss);
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
        if ((threadIdx.x & 31) == 0) fpart[threadIdx.x >> 5] = ss;
        __syncthreads();
        float total = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) total += fpart[w];
        scale = rsqrtf(total / static_cast<float>(cols) + eps);
    }
    if (row == 0 && blockIdx.y == 0 && zero_sums)
        for (int i = threadIdx.x; i < zero_count; i += blockDim.x) zero_sums[i] = 0;
    if (bad_bound(b) && threadIdx.x == 0 && blockIdx.y == 0) set_flag(flags, BD_FLAG_BAD_BOUND);
    Quant q;
    q.init(b, bits);
    int sum = 0;
    bool bad = false;
    if (k0 < cols) {
        float xv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            xv[j] = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (i == static_cast<int>(blockIdx.y)) xv[j] = v[i][j];
            const bool live = k0 + j < cols;
            if (blockIdx.y >= 4 && live) xv[j] = xr[k0 + j];
            if (norm_w && live) xv[j] = xv[j] * scale * nv[j];
        }
        int c[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            c[j] = 0;
            if (k0 + j < cols) {
                const float g = __fmul_rn(xv[j], gv[j]);
                bad |= !isfinite(g);
                c[j] = q.code(g);
            }
            sum += c[j];
        }
        *reinterpret_cast<char4 *>(codes + code_offset(row, k0, ld, c16_mt)) =
            make_char4(static_cast<signed char>(c[0]), static_cast<signed char>(c[1]),
                       static_cast<signed char>(c[2]), static_cast<signed char>(c[3]));
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_NONFINITE_INPUT);
    if (sums) {
        const int total = block_sum_256(sum, scratch);
        if (threadIdx.x == 0) {
            if (partial)
                sums[row * gridDim.y + blockIdx.y] = total;
            else if (total)
                atomicAdd(sums + row, total);
        }
    }
}

// Per-token 16-bit fixed point: q = rint(x * 32639 / max|x|), q = 256 hi + lo.
// One CTA per row: the row maximum needs the whole row.
__global__ void __launch_bounds__(256) quantize_planes_kernel(const float *__restrict__ x, int64_t cols, int64_t ld,
                                                              int8_t *__restrict__ hi, int8_t *__restrict__ lo,
                                                              int32_t *__restrict__ sums_hi,
                                                              int32_t *__restrict__ sums_lo,
                                                              float *__restrict__ row_scale, int32_t *flags,
                                                              int c16_mt) {
    __shared__ float fscratch[8];
    __shared__ int iscratch[8];
    grid_wait();
    grid_launch_dependents();
    const int row = blockIdx.x;
    float m = 0.0f;
    bool bad = false;
    for (int64_t k0 = 4 * threadIdx.x; k0 < cols; k0 += 4 * blockDim.x) {
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = k0 + j < cols ? x[row * cols + k0 + j] : 0.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            bad |= !isfinite(v[j]);
            m = fmaxf(m, fabsf(v[j]));
        }
    }
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
    if ((threadIdx.x & 31) == 0) fscratch[threadIdx.x >> 5] = m;
    __syncthreads();
    m = fscratch[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) m = fmaxf(m, fscratch[w]);
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_NONFINITE_INPUT);
    const float inv = m > 0.0f ? __fdiv_rn(32639.0f, m) : 0.0f;
    int shi = 0, slo = 0;
    for (int64_t k0 = 4 * threadIdx.x; k0 < cols; k0 += 4 * blockDim.x) {
        int h[4], l[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            h[j] = l[j] = 0;
            if (k0 + j < cols) {
                float r = rintf(__fmul_rn(x[row * cols + k0 + j], inv));
                r = fminf(fmaxf(r, -32639.0f), 32639.0f);
                const int qv = static_cast<int>(r);
                h[j] = (qv + 128) >> 8;
                l[j] = qv - 256 * h[j];
            }
            shi += h[j];
            slo += l[j];
        }
        const int64_t off = code_offset(row, k0, ld, c16_mt);
        *reinterpret_cast<char4 *>(hi + off) = make_char4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<char4 *>(lo + off) = make_char4(l[0], l[1], l[2], l[3]);
    }
    shi = block_sum_256(shi, iscratch);
    slo = block_sum_256(slo, iscratch);
    if (threadIdx.x == 0) {
        sums_hi[row] = shi;
        sums_lo[row] = slo;
        row_scale[row] = __fdiv_rn(m, 32639.0f);
    }
}

// W1A1: codes = x >= 0 ? +1 : -1; mean|x| in the fixed order of oracle.core.fixed_mean_abs
// (lane l of 256 adds |x[l + 256 i]| sequentially, then a balanced tree of adjacent pairs).
__global__ void __launch_bounds__(256) binarize_kernel(const float *__restrict__ x, int64_t cols, int64_t ld,
                                                       int8_t *__restrict__ codes, int32_t *__restrict__ sums,
                                                       float *__restrict__ mean_abs, uint32_t *__restrict__ words,
                                                       int64_t words_ld, int32_t *flags, int c16_mt) {
    __shared__ float fscratch[8];
    __shared__ int iscratch[8];
    grid_wait();
    grid_launch_dependents();
    const int row = blockIdx.x;
    float acc = 0.0f;
    int s = 0;
    bool bad = false;
    for (int64_t k = threadIdx.x; k < ld; k += blockDim.x) {
        int c = 0;
        if (k < cols) {
            const float v = x[row * cols + k];
            bad |= !isfinite(v);
            acc = __fadd_rn(acc, fabsf(v));
            c = v >= 0.0f ? 1 : -1;
        }
        if (codes) codes[code_offset(row, k, ld, c16_mt)] = static_cast<int8_t>(c);
        s += c;
        if (words) {
            const unsigned word = __ballot_sync(0xffffffffu, c > 0);
            if ((threadIdx.x & 31) == 0 && (k >> 5) < words_ld) words[row * words_ld + (k >> 5)] = word;
        }
    }
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, d));
    if ((threadIdx.x & 31) == 0) fscratch[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        const float a = __fadd_rn(__fadd_rn(fscratch[0], fscratch[1]), __fadd_rn(fscratch[2], fscratch[3]));
        const float b = __fadd_rn(__fadd_rn(fscratch[4], fscratch[5]), __fadd_rn(fscratch[6], fscratch[7]));
        mean_abs[row] = __fdiv_rn(__fadd_rn(a, b), static_cast<float>(cols));
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_NONFINITE_INPUT);
    s = block_sum_256(s, iscratch);
    if (threadIdx.x == 0 && sums) sums[row] = s;
}

int launch_quantize_codes(const float *x, int64_t rows, int64_t cols, int64_t ld, const float *gain,
                          const float *bound, int bits, int8_t *codes, int32_t *sums, bool partial, int32_t *flags,
                          int32_t *zero_sums, int zero_count, cudaStream_t stream, const float *norm_w, float eps,
                          int c16_mt) {
    if (rows == 0) return BD_OK;
    if (sums && !partial && cudaMemsetAsync(sums, 0, rows * sizeof(int32_t), stream) != cudaSuccess)
        return BD_ERR_LAUNCH;
    const dim3 grid(static_cast<unsigned>(rows), static_cast<unsigned>(quant_parts(cols)));
    // same shared-memory carveout as the projection kernels around it: no SM reconfiguration between them
    if (cudaFuncSetAttribute(quantize_codes_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
        return BD_ERR_LAUNCH;
    return launch_pdl(quantize_codes_kernel, grid, dim3(256), 0, stream, x, cols, ld, gain, bound, bits, codes, sums,
                      partial, flags, zero_sums, zero_count, norm_w, eps, c16_mt);
}

int launch_quantize_planes(const float *x, int64_t rows, int64_t cols, int64_t ld, int8_t *hi, int8_t *lo,
                           int32_t *sums_hi, int32_t *sums_lo, float *row_scale, int32_t *flags,
                           cudaStream_t stream, int c16_mt) {
    if (rows == 0) return BD_OK;
    return launch_pdl(quantize_planes_kernel, dim3(static_cast<unsigned>(rows)), dim3(256), 0, stream, x, cols, ld,
                      hi, lo, sums_hi, sums_lo, row_scale, flags, c16_mt);
}

int launch_binarize(const float *x, int64_t rows, int64_t cols, int64_t ld, int8_t *codes, int32_t *sums,
                    float *mean_abs, uint32_t *words, int64_t words_ld, int32_t *flags, cudaStream_t stream,
                    int c16_mt) {
    if (rows == 0) return BD_OK;
    return launch_pdl(binarize_kernel, dim3(static_cast<unsigned>(rows)), dim3(256), 0, stream, x, cols, ld, codes,
                      sums, mean_abs, words, words_ld, flags, c16_mt);
}

}  // namespace bd

extern "C" int64_t bd_codes_ld(int64_t cols) { return cols <= 0 ? 0 : (cols + 255) / 256 * 256; }

extern "C" int64_t bd_codes_bytes(int64_t rows, int64_t cols) {
    if (rows < 0 || cols < 0) return -1;
    return (rows + 7) / 8 * 8 * bd_codes_ld(cols);
}

extern "C" int bd_quantize_codes(const float *x, int64_t rows, int64_t cols, int64_t ld, const float *gain,
                                 const float *bound, int bits, int8_t *codes, int32_t *code_sums, int32_t *flags,
                                 bd_stream_t stream) {
    if (rows < 0 || rows > 0x7fffffff || cols < 0 || ld < cols || (ld & 255) || (bits != 4 && bits != 8))
        return BD_ERR_INVALID;
    if (rows > 0 && (!x || !gain || !bound || !codes || !code_sums)) return BD_ERR_INVALID;
    return bd::launch_quantize_codes(x, rows, cols, ld, gain, bound, bits, codes, code_sums, false, flags, nullptr,
                                     0, stream);
}
