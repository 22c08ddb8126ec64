// Large-M HE4 projection and its straight-through backward (QAT).
//
// Projection.forward (w1a1_eagle/model.py:128-150) at training sizes is
//   codes = quantize(x * gain, bound)       (integers, |code| <= 7 or 127)
//   D     = codes . sign(latent)^T          (exact integers, |D| < 2^24)
//   y     = (D * max(scale, 0)) * step + (sum(codes) * step) * midpoint.
// Codes and signs are exact in bf16, so D is computed by a bf16 tensor-core
// GEMM with fp32 accumulation without any rounding; these kernels produce its
// operands (row-major bf16 codes, +-1 signs) and apply the epilogue.
//
// The backward follows autograd through the surrogate branch
// (surrogate = linear(values, signs) * scale + sum(values) * midpoint, values =
// codes * step, codes' gradient straight through round, torch's 0.5/0.5 tie
// split for minimum/maximum, SIGN's backward grad * 1[|w| <= window],
// model.py:71-73).  The GEMMs dL . signs and dL^T . codes take dL = G * scale
// as two bf16 halves (hi + lo carries ~16 significant bits), so they too run on
// the tensor cores with fp32 accumulation.  Every reduction here is in a fixed
// order (per-thread sequential, then fixed trees), so results are
// deterministic.
#include "kernels.cuh"

namespace bd {

constexpr int kCols = 256;       // columns per CTA (one per thread)
constexpr int kRowChunk = 64;    // rows per CTA in the two-direction kernels

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, d));
    return v;
}

// Fixed-order block sum over 256 threads (warp butterflies, then 8 warp sums in order).
__device__ __forceinline__ float block_sum_f(float v, float *scratch) {
    v = warp_sum(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = scratch[0];
    for (int w = 1; w < 8; ++w) s = __fadd_rn(s, scratch[w]);
    return s;
}

// ------------------------------------------------------------------ forward pieces

__device__ __forceinline__ void store_code(__nv_bfloat16 *p, int c) { *p = __int2bfloat16_rn(c); }
__device__ __forceinline__ void store_code(int8_t *p, int c) { *p = static_cast<int8_t>(c); }

// x [rows, cols] -> codes [rows, ld] (row-major, bf16 or int8) and exact per-row code sums.
template <typename Code>
__global__ void __launch_bounds__(256) quantize_rows_kernel(const float *__restrict__ x, int64_t cols, int64_t ld,
                                                            const float *__restrict__ gain,
                                                            const float *__restrict__ bound, int bits,
                                                            Code *__restrict__ codes, int32_t *__restrict__ sums,
                                                            int32_t *flags) {
    __shared__ int scratch[8];
    const int64_t row = blockIdx.x;
    const float b = __ldg(bound);
    if (bad_bound(b)) {
        if (threadIdx.x == 0 && blockIdx.y == 0 && row == 0) set_flag(flags, BD_FLAG_BAD_BOUND);
        return;
    }
    Quant q;
    q.init(b, bits);
    int s = 0;
    bool bad = false;
    const int64_t c0 = static_cast<int64_t>(blockIdx.y) * 1024;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int64_t c = c0 + i * 256 + threadIdx.x;
        if (c < cols) {
            const float g = __fmul_rn(x[row * cols + c], __ldg(gain + c));
            bad |= !isfinite(g);
            const int code = q.code(g);
            store_code(codes + row * ld + c, code);
            s += code;
        }
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_NONFINITE_INPUT);
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) s += __shfl_xor_sync(0xffffffffu, s, d);
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        int t = 0;
        for (int w = 0; w < 8; ++w) t += scratch[w];
        if (t) atomicAdd(sums + row, t);  // integer: order-free and exact
    }
}

// latent [n] -> +-1 (x >= 0 -> +1, -0.0 -> +1) as bf16 and/or fp32.
__global__ void sign_rows_kernel(const float *__restrict__ latent, int64_t n, __nv_bfloat16 *__restrict__ out16,
                                 float *__restrict__ out32, int32_t *flags) {
    bool bad = false;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float v = latent[i];
        bad |= !isfinite(v);
        const float s = v >= 0.0f ? 1.0f : -1.0f;
        if (out16) out16[i] = __float2bfloat16_rn(s);
        if (out32) out32[i] = s;
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_NONFINITE_LATENT);
}

// Tiled transpose into bf16: dst[c][r] = f(src[r][c]) for r < rows, c < cols (32 x 32 tiles).
// SIGNS = true: f = +-1 of an fp32 latent (x >= 0 -> +1, -0.0 -> +1), with the finiteness check;
// SIGNS = false: f = the int8 code itself (exact in bf16).
// 64 x 64 tiles through shared memory: rows of the tile are read along the source
// rows, and each destination row of the tile (64 source rows) is written as one
// 128-byte run of bf16 pairs (single values where ldd is odd or at the last row).
constexpr int kTr = 64;

template <bool SIGNS, typename In>
__global__ void __launch_bounds__(256) transpose_bf16_kernel(const In *__restrict__ src, int64_t rows, int64_t cols,
                                                             int64_t lds, __nv_bfloat16 *__restrict__ dst,
                                                             int64_t ldd, int32_t *flags) {
    __shared__ float tile[kTr][kTr + 1];
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kTr, c0 = static_cast<int64_t>(blockIdx.x) * kTr;
    const int tx = threadIdx.x & (kTr - 1), ty = threadIdx.x / kTr;  // 64 x 4
    bool bad = false;
#pragma unroll 4
    for (int i = ty; i < kTr; i += 256 / kTr) {
        const int64_t r = r0 + i, c = c0 + tx;
        float v = 0.0f;
        if (r < rows && c < cols) {
            const float x = static_cast<float>(src[r * lds + c]);
            if (SIGNS) {
                bad |= !isfinite(x);
                v = x >= 0.0f ? 1.0f : -1.0f;
            } else {
                v = x;
            }
        }
        tile[i][tx] = v;
    }
    if (SIGNS && __any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_NONFINITE_LATENT);
    __syncthreads();
    const int lane = threadIdx.x & 31, wc = threadIdx.x >> 5;  // 32 lanes x 8 column rows at a time
    const bool pairs = (ldd & 1) == 0 && (reinterpret_cast<uintptr_t>(dst) & 3) == 0;
#pragma unroll 2
    for (int i = wc; i < kTr; i += 8) {
        const int64_t c = c0 + i, r = r0 + 2 * lane;
        if (c >= cols || r >= rows) continue;
        const __nv_bfloat16 e0 = __float2bfloat16_rn(tile[2 * lane][i]);
        if (r + 1 < rows && pairs) {
            __nv_bfloat162 two;
            two.x = e0;
            two.y = __float2bfloat16_rn(tile[2 * lane + 1][i]);
            *reinterpret_cast<__nv_bfloat162 *>(dst + c * ldd + r) = two;
        } else {
            dst[c * ldd + r] = e0;
            if (r + 1 < rows) dst[c * ldd + r + 1] = __float2bfloat16_rn(tile[2 * lane + 1][i]);
        }
    }
}

// fp32 [rows][cols] (row stride lds) -> bf16 halves hi = bf16(x), lo = bf16(x - hi) with row
// stride ldd; TRANSPOSE writes them as [cols][ldd] instead (32 x 32 tiles through shared memory).
template <bool TRANSPOSE>
__global__ void __launch_bounds__(256) split_bf16_kernel(const float *__restrict__ src, int64_t rows, int64_t cols,
                                                         int64_t lds, __nv_bfloat16 *__restrict__ hi,
                                                         __nv_bfloat16 *__restrict__ lo, int64_t ldd) {
    __shared__ float tile[32][33];
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * 32, c0 = static_cast<int64_t>(blockIdx.x) * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int i = ty; i < 32; i += 8) {
        const int64_t r = r0 + i, c = c0 + tx;
        const float v = (r < rows && c < cols) ? src[r * lds + c] : 0.0f;
        if (TRANSPOSE) {
            tile[i][tx] = v;
        } else if (r < rows && c < cols) {
            const __nv_bfloat16 h = __float2bfloat16_rn(v);
            hi[r * ldd + c] = h;
            lo[r * ldd + c] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h)));
        }
    }
    if (!TRANSPOSE) return;
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int64_t c = c0 + i, r = r0 + tx;
        if (c < cols && r < rows) {
            const float v = tile[tx][i];
            const __nv_bfloat16 h = __float2bfloat16_rn(v);
            hi[c * ldd + r] = h;
            lo[c * ldd + r] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h)));
        }
    }
}

// y[t, o] = he4_value(D[t, o], scale[o], step, sums[t], midpoint[o]) (+ residual).
__global__ void he4_epilogue_kernel(const float *__restrict__ dot, int64_t tokens, int64_t outs,
                                    const float *__restrict__ scale, const float *__restrict__ midpoint,
                                    const float *__restrict__ bound, int bits, const int32_t *__restrict__ sums,
                                    const float *__restrict__ residual, float *__restrict__ y) {
    Quant q;
    q.init(__ldg(bound), bits);
    const int64_t n = tokens * outs;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / outs, o = i - t * outs;
        float v = he4_value(static_cast<int>(dot[i]), __ldg(scale + o), q.step, __ldg(sums + t), __ldg(midpoint + o));
        if (residual) v = __fadd_rn(residual[i], v);
        y[i] = v;
    }
}

// ------------------------------------------------------------------ backward pieces

// Output-side gradients: grid (column tiles of 256, row chunks of 64).
//   dL = G * max(scale, 0) -> bf16 hi, lo;  colpart[rc][0][o] = sum_t G * (D * step);
//   colpart[rc][1][o] = sum_t G * (sums[t] * step);  rowpart[ct][t] = sum_o G * midpoint[o].
// Rows go in batches of 16: every thread requests its 16 G and D values before any
// arithmetic (the loads of a batch are in flight together), writes the transposed
// halves as whole 32-byte sectors (16 tokens), and the row sums of the batch are
// reduced once through shared memory (warp w: rows 2w, 2w + 1).
constexpr int kPrepRows = 16;
static_assert(kRowChunk % kPrepRows == 0 && kPrepRows == 2 * (kCols / 32), "two batch rows per warp");

__global__ void __launch_bounds__(kCols, 3) grad_prep_kernel(const float *__restrict__ grad, const float *__restrict__ dot,
                                                          int64_t tokens, int64_t outs, const float *__restrict__ scale,
                                                          const float *__restrict__ midpoint,
                                                          const float *__restrict__ bound, int bits,
                                                          const int32_t *__restrict__ sums,
                                                          __nv_bfloat16 *__restrict__ hi, __nv_bfloat16 *__restrict__ lo,
                                                          int64_t ld_dl, __nv_bfloat16 *__restrict__ hi_t,
                                                          __nv_bfloat16 *__restrict__ lo_t, int64_t ld_t,
                                                          float *__restrict__ colpart, float *__restrict__ rowpart) {
    __shared__ float gsum[kPrepRows][kCols];
    __shared__ float rsum[kRowChunk];
    Quant q;
    q.init(__ldg(bound), bits);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t o = static_cast<int64_t>(blockIdx.x) * kCols + threadIdx.x;
    const bool live = o < outs;
    const float s = live ? __ldg(scale + o) : 0.0f;
    const float sc = s < 0.0f ? 0.0f : s;
    const float mid = live ? __ldg(midpoint + o) : 0.0f;
    const int64_t t0 = static_cast<int64_t>(blockIdx.y) * kRowChunk;
    float acc_scale = 0.0f, acc_mid = 0.0f;
    for (int r16 = 0; r16 < kRowChunk; r16 += kPrepRows) {
        float g[kPrepRows], d[kPrepRows];
#pragma unroll
        for (int j = 0; j < kPrepRows; ++j) {
            const int64_t t = t0 + r16 + j;
            const bool on = t < tokens && live;
            g[j] = on ? grad[t * outs + o] : 0.0f;
            d[j] = on ? dot[t * outs + o] : 0.0f;
        }
        uint32_t th[kPrepRows / 2], tl[kPrepRows / 2];
#pragma unroll
        for (int j = 0; j < kPrepRows; ++j) {
            const int64_t t = t0 + r16 + j;
            float gm = 0.0f;
            if ((j & 1) == 0) th[j >> 1] = tl[j >> 1] = 0u;
            if (t < tokens && live) {
                acc_scale = __fadd_rn(acc_scale, __fmul_rn(g[j], __fmul_rn(d[j], q.step)));
                acc_mid = __fadd_rn(acc_mid, __fmul_rn(g[j], __fmul_rn(static_cast<float>(__ldg(sums + t)), q.step)));
                const float dl = __fmul_rn(g[j], sc);
                const __nv_bfloat16 h = __float2bfloat16_rn(dl);
                const __nv_bfloat16 l = __float2bfloat16_rn(__fsub_rn(dl, __bfloat162float(h)));
                hi[t * ld_dl + o] = h;
                lo[t * ld_dl + o] = l;
                th[j >> 1] |= static_cast<uint32_t>(__bfloat16_as_ushort(h)) << (16 * (j & 1));
                tl[j >> 1] |= static_cast<uint32_t>(__bfloat16_as_ushort(l)) << (16 * (j & 1));
                gm = __fmul_rn(g[j], mid);
            }
            gsum[j][threadIdx.x] = gm;
        }
        // transposed halves: tokens [r16, r16 + 8) and [r16 + 8, r16 + 16), each written
        // only where its first token exists (ld_t covers tokens rounded up to 8)
        if (hi_t && live) {
#pragma unroll
            for (int h8 = 0; h8 < 2; ++h8) {
                if (t0 + r16 + 8 * h8 < tokens) {
                    *reinterpret_cast<uint4 *>(hi_t + o * ld_t + t0 + r16 + 8 * h8) =
                        make_uint4(th[4 * h8], th[4 * h8 + 1], th[4 * h8 + 2], th[4 * h8 + 3]);
                    *reinterpret_cast<uint4 *>(lo_t + o * ld_t + t0 + r16 + 8 * h8) =
                        make_uint4(tl[4 * h8], tl[4 * h8 + 1], tl[4 * h8 + 2], tl[4 * h8 + 3]);
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int r = 2 * warp + rr;
            float v = 0.0f;
#pragma unroll
            for (int c = 0; c < kCols / 32; ++c) v = __fadd_rn(v, gsum[r][lane + 32 * c]);
            v = warp_sum(v);
            if (lane == 0) rsum[r16 + r] = v;
        }
        __syncthreads();
    }
    if (live) {
        colpart[(static_cast<int64_t>(blockIdx.y) * 2 + 0) * outs + o] = acc_scale;
        colpart[(static_cast<int64_t>(blockIdx.y) * 2 + 1) * outs + o] = acc_mid;
    }
    if (threadIdx.x < kRowChunk && t0 + threadIdx.x < tokens)
        rowpart[static_cast<int64_t>(blockIdx.x) * tokens + t0 + threadIdx.x] = rsum[threadIdx.x];
}

// d_scale[o] = sum_rc colpart[rc][0][o] * (scale[o] >= 0); d_mid[o] = sum_rc colpart[rc][1][o];
// gm[t] = sum_ct rowpart[ct][t] (all in increasing index order).
__global__ void grad_prep_reduce_kernel(const float *__restrict__ colpart, const float *__restrict__ rowpart,
                                        int64_t tokens, int64_t outs, int rchunks, int ctiles,
                                        const float *__restrict__ scale, float *__restrict__ d_scale,
                                        float *__restrict__ d_mid, float *__restrict__ gm) {
    const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < outs) {
        float a = 0.0f, m = 0.0f;
        for (int rc = 0; rc < rchunks; ++rc) {
            a = __fadd_rn(a, colpart[(static_cast<int64_t>(rc) * 2 + 0) * outs + i]);
            m = __fadd_rn(m, colpart[(static_cast<int64_t>(rc) * 2 + 1) * outs + i]);
        }
        d_scale[i] = __ldg(scale + i) >= 0.0f ? a : 0.0f;
        d_mid[i] = m;
    }
    if (i < tokens) {
        float v = 0.0f;
        for (int ct = 0; ct < ctiles; ++ct) v = __fadd_rn(v, rowpart[static_cast<int64_t>(ct) * tokens + i]);
        gm[i] = v;
    }
}

// Input-side gradients through the quantizer: grid (column tiles of 256, row chunks of 64).
//   dv = d_values (+ d_values2) + gm[t];  d_codes = dv * step;  d_clipped = d_codes * ratio;
//   tie-split masks of maximum(minimum(gained, b), -b);  d_x = d_gained * gain[k].
// Partials: colpart[rc][k] = sum_t d_gained * x;  scal[block][4] = the four d_bound sums.
__global__ void __launch_bounds__(kCols) ste_input_kernel(const float *__restrict__ dv1, const float *__restrict__ dv2,
                                                          const float *__restrict__ gm, const float *__restrict__ x,
                                                          int64_t tokens, int64_t cols, const float *__restrict__ gain,
                                                          const float *__restrict__ bound, int bits,
                                                          float *__restrict__ dx, float *__restrict__ colpart,
                                                          float *__restrict__ scal) {
    __shared__ float scratch[8];
    Quant q;
    q.init(__ldg(bound), bits);
    const float b = q.bound, nb = -q.bound;
    const int64_t k = static_cast<int64_t>(blockIdx.x) * kCols + threadIdx.x;
    const bool live = k < cols;
    const float g = live ? __ldg(gain + k) : 0.0f;
    const int64_t t0 = static_cast<int64_t>(blockIdx.y) * kRowChunk;
    float acc_gain = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f, s4 = 0.0f;
    // rows in batches of 16 whose loads are all requested before the arithmetic; the
    // sums still run over the rows in order
    for (int r16 = 0; r16 < kRowChunk && live && t0 + r16 < tokens; r16 += kPrepRows) {
        float dva[kPrepRows], xa[kPrepRows];
#pragma unroll
        for (int j = 0; j < kPrepRows; ++j) {
            const int64_t t = t0 + r16 + j;
            const int64_t i = t * cols + k;
            const bool on = t < tokens;
            dva[j] = on ? dv1[i] : 0.0f;
            if (dv2 && on) dva[j] = __fadd_rn(dva[j], dv2[i]);
            xa[j] = on ? x[i] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < kPrepRows; ++j) {
            const int64_t t = t0 + r16 + j;
            if (t >= tokens) break;
            const int64_t i = t * cols + k;
            const float d = __fadd_rn(dva[j], __ldg(gm + t));
            const float xv = xa[j];
            const float gained = __fmul_rn(xv, g);
            const float mn = fminf(gained, b);
            const float clipped = fmaxf(mn, nb);
            const int code = q.code(gained);
            const float d_codes = __fmul_rn(d, q.step);
            s1 = __fadd_rn(s1, __fmul_rn(d, static_cast<float>(code)));
            s2 = __fadd_rn(s2, __fmul_rn(d_codes, clipped));
            const float d_clipped = __fmul_rn(d_codes, q.ratio);
            const float to_mn = mn > nb ? 1.0f : (mn == nb ? 0.5f : 0.0f);
            const float d_mn = __fmul_rn(d_clipped, to_mn);
            s3 = __fadd_rn(s3, __fmul_rn(d_clipped, __fsub_rn(1.0f, to_mn)));
            const float to_g = gained < b ? 1.0f : (gained == b ? 0.5f : 0.0f);
            const float d_gained = __fmul_rn(d_mn, to_g);
            s4 = __fadd_rn(s4, __fmul_rn(d_mn, __fsub_rn(1.0f, to_g)));
            dx[i] = __fmul_rn(d_gained, g);
            acc_gain = __fadd_rn(acc_gain, __fmul_rn(d_gained, xv));
        }
    }
    if (live) colpart[static_cast<int64_t>(blockIdx.y) * cols + k] = acc_gain;
    const float v1 = block_sum_f(s1, scratch);
    const float v2 = block_sum_f(s2, scratch);
    const float v3 = block_sum_f(s3, scratch);
    const float v4 = block_sum_f(s4, scratch);
    if (threadIdx.x == 0) {
        float *p = scal + (static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x) * 4;
        p[0] = v1;
        p[1] = v2;
        p[2] = v3;
        p[3] = v4;
    }
}

// d_log_gain[k] = (sum_rc colpart[rc][k]) * gain[k]; block 0 also combines the
// d_bound partials in the autograd order and writes d_log_clip = d_bound * bound.
__global__ void __launch_bounds__(256) ste_input_reduce_kernel(const float *__restrict__ colpart,
                                                               const float *__restrict__ scal, int nblocks,
                                                               int64_t cols, int rchunks,
                                                               const float *__restrict__ gain,
                                                               const float *__restrict__ bound, int bits,
                                                               float *__restrict__ d_log_gain,
                                                               float *__restrict__ d_log_clip, int accumulate) {
    __shared__ float scratch[8];
    const int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (k < cols) {
        float a = 0.0f;
        for (int rc = 0; rc < rchunks; ++rc) a = __fadd_rn(a, colpart[static_cast<int64_t>(rc) * cols + k]);
        const float v = __fmul_rn(a, __ldg(gain + k));
        d_log_gain[k] = accumulate ? __fadd_rn(d_log_gain[k], v) : v;
    }
    if (blockIdx.x != 0) return;
    float part[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float v = 0.0f;
        for (int i = threadIdx.x; i < nblocks; i += blockDim.x) v = __fadd_rn(v, scal[static_cast<int64_t>(i) * 4 + j]);
        part[j] = block_sum_f(v, scratch);
    }
    if (threadIdx.x == 0) {
        Quant q;
        q.init(__ldg(bound), bits);
        const float recip = __frcp_rn(q.bound);
        float db = __fdiv_rn(part[0], q.maximum);
        db = __fadd_rn(db, __fmul_rn(__fmul_rn(part[1], q.maximum), -__fmul_rn(recip, recip)));
        db = __fsub_rn(db, part[2]);
        db = __fadd_rn(db, part[3]);
        const float v = __fmul_rn(db, q.bound);
        d_log_clip[0] = accumulate ? __fadd_rn(d_log_clip[0], v) : v;
    }
}

// Straight-through sign gradient: out = ((g1 + g2) * step) * 1[|latent| <= window];
// per-block sums of out^2 (fixed order) when sumsq != NULL.
__global__ void __launch_bounds__(256) ste_mask_kernel(const float *__restrict__ g1, const float *__restrict__ g2,
                                                       const float *__restrict__ latent, int64_t n, float window,
                                                       const float *__restrict__ bound, int bits,
                                                       float *__restrict__ out, float *__restrict__ sumsq) {
    __shared__ float scratch[8];
    float step = 1.0f;
    if (bound) {
        Quant q;
        q.init(__ldg(bound), bits);
        step = q.step;
    }
    float ss = 0.0f;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float g = g1[i];
        if (g2) g = __fadd_rn(g, g2[i]);
        if (bound) g = __fmul_rn(g, step);
        const float v = fabsf(latent[i]) <= window ? g : 0.0f;
        out[i] = v;
        ss = __fadd_rn(ss, __fmul_rn(v, v));
    }
    if (sumsq) {
        const float s = block_sum_f(ss, scratch);
        if (threadIdx.x == 0) sumsq[blockIdx.x] = s;
    }
}

}  // namespace bd

using namespace bd;

static unsigned elementwise_grid(int64_t n) {
    int64_t g = (n + 255) / 256;
    if (g < 1) g = 1;
    if (g > 148 * 32) g = 148 * 32;
    return static_cast<unsigned>(g);
}

extern "C" int bd_quantize_rows_bf16(const float *x, int64_t rows, int64_t cols, const float *gain,
                                     const float *bound, int bits, uint16_t *codes, int32_t *code_sums,
                                     int32_t *flags, bd_stream_t stream) {
    if (rows < 0 || cols < 1 || (bits != 4 && bits != 8) || rows > 0x7fffffff || (cols + 1023) / 1024 > 65535)
        return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    if (!x || !gain || !bound || !codes || !code_sums) return BD_ERR_INVALID;
    if (cudaMemsetAsync(code_sums, 0, rows * sizeof(int32_t), stream) != cudaSuccess) return BD_ERR_LAUNCH;
    dim3 grid(static_cast<unsigned>(rows), static_cast<unsigned>((cols + 1023) / 1024));
    quantize_rows_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
        x, cols, cols, gain, bound, bits, reinterpret_cast<__nv_bfloat16 *>(codes), code_sums, flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_quantize_rows_i8(const float *x, int64_t rows, int64_t cols, const float *gain, const float *bound,
                                   int bits, int8_t *codes, int64_t ld, int32_t *code_sums, int32_t *flags,
                                   bd_stream_t stream) {
    if (rows < 0 || cols < 1 || ld < cols || (bits != 4 && bits != 8) || rows > 0x7fffffff ||
        (cols + 1023) / 1024 > 65535)
        return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    if (!x || !gain || !bound || !codes || !code_sums) return BD_ERR_INVALID;
    if (cudaMemsetAsync(code_sums, 0, rows * sizeof(int32_t), stream) != cudaSuccess) return BD_ERR_LAUNCH;
    dim3 grid(static_cast<unsigned>(rows), static_cast<unsigned>((cols + 1023) / 1024));
    quantize_rows_kernel<int8_t><<<grid, 256, 0, stream>>>(x, cols, ld, gain, bound, bits, codes, code_sums, flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

// codes int8 [rows][ld] -> bf16 [cols][ld_t] (the weight-gradient GEMM's K-major operand)
extern "C" int bd_codes_transpose_bf16(const int8_t *codes, int64_t rows, int64_t cols, int64_t ld, uint16_t *out,
                                       int64_t ld_t, bd_stream_t stream) {
    if (rows < 1 || cols < 1 || ld < cols || ld_t < rows || (rows + kTr - 1) / kTr > 65535 || !codes || !out)
        return BD_ERR_INVALID;
    dim3 grid(static_cast<unsigned>((cols + kTr - 1) / kTr), static_cast<unsigned>((rows + kTr - 1) / kTr));
    transpose_bf16_kernel<false, int8_t><<<grid, 256, 0, stream>>>(codes, rows, cols, ld,
                                                                   reinterpret_cast<__nv_bfloat16 *>(out), ld_t,
                                                                   nullptr);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

// fp32 x [rows][cols] (row stride ldx) -> bf16 hi + lo halves [rows][ld] (or, transposed, [cols][ld])
extern "C" int bd_split_bf16(const float *x, int64_t rows, int64_t cols, int64_t ldx, int transpose, uint16_t *hi,
                             uint16_t *lo, int64_t ld, bd_stream_t stream) {
    if (rows < 1 || cols < 1 || ldx < cols || ld < (transpose ? rows : cols) || (rows + 31) / 32 > 65535 || !x ||
        !hi || !lo)
        return BD_ERR_INVALID;
    dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>((rows + 31) / 32));
    auto *h = reinterpret_cast<__nv_bfloat16 *>(hi);
    auto *l = reinterpret_cast<__nv_bfloat16 *>(lo);
    if (transpose)
        split_bf16_kernel<true><<<grid, 256, 0, stream>>>(x, rows, cols, ldx, h, l, ld);
    else
        split_bf16_kernel<false><<<grid, 256, 0, stream>>>(x, rows, cols, ldx, h, l, ld);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

// latent fp32 [rows][cols] -> +-1 bf16 [cols][ld_t] (the input-gradient GEMM's K-major operand)
extern "C" int bd_sign_cols_bf16(const float *latent, int64_t rows, int64_t cols, uint16_t *out, int64_t ld_t,
                                 int32_t *flags, bd_stream_t stream) {
    if (rows < 1 || cols < 1 || ld_t < rows || (rows + kTr - 1) / kTr > 65535 || !latent || !out)
        return BD_ERR_INVALID;
    dim3 grid(static_cast<unsigned>((cols + kTr - 1) / kTr), static_cast<unsigned>((rows + kTr - 1) / kTr));
    transpose_bf16_kernel<true, float><<<grid, 256, 0, stream>>>(latent, rows, cols, cols,
                                                                 reinterpret_cast<__nv_bfloat16 *>(out), ld_t, flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_sign_rows(const float *latent, int64_t n, uint16_t *signs_bf16, float *signs_f32, int32_t *flags,
                            bd_stream_t stream) {
    if (n < 0) return BD_ERR_INVALID;
    if (n == 0) return BD_OK;
    if (!latent || (!signs_bf16 && !signs_f32)) return BD_ERR_INVALID;
    sign_rows_kernel<<<elementwise_grid(n), 256, 0, stream>>>(
        latent, n, reinterpret_cast<__nv_bfloat16 *>(signs_bf16), signs_f32, flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_he4_epilogue(const float *dot, int64_t tokens, int64_t out_features, const float *scale,
                               const float *midpoint, const float *bound, int bits, const int32_t *code_sums,
                               const float *residual, float *y, bd_stream_t stream) {
    if (tokens < 0 || out_features < 1 || (bits != 4 && bits != 8)) return BD_ERR_INVALID;
    if (tokens == 0) return BD_OK;
    if (!dot || !scale || !midpoint || !bound || !code_sums || !y) return BD_ERR_INVALID;
    he4_epilogue_kernel<<<elementwise_grid(tokens * out_features), 256, 0, stream>>>(
        dot, tokens, out_features, scale, midpoint, bound, bits, code_sums, residual, y);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

static int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

extern "C" size_t bd_ste_workspace_bytes(int64_t tokens, int64_t out_features, int64_t in_features) {
    const int64_t rchunks = ceil_div(tokens, kRowChunk);
    const int64_t ct_out = ceil_div(out_features, kCols), ct_in = ceil_div(in_features, kCols);
    size_t bytes = 0;
    auto take = [&](int64_t n) { bytes += (static_cast<size_t>(n) * 4 + 255) / 256 * 256; };
    take(rchunks * 2 * out_features);  // grad_prep colpart
    take(ct_out * tokens);             // grad_prep rowpart
    take(rchunks * in_features);       // ste_input colpart
    take(rchunks * ct_in * 4);         // ste_input scalar partials
    return bytes;
}

struct SteWs {
    float *colpart, *rowpart, *gain_part, *scal;
};

static SteWs carve_ste(void *ws, int64_t tokens, int64_t outs, int64_t ins) {
    const int64_t rchunks = ceil_div(tokens, kRowChunk);
    const int64_t ct_out = ceil_div(outs, kCols), ct_in = ceil_div(ins, kCols);
    char *p = static_cast<char *>(ws);
    auto take = [&](int64_t n) {
        float *r = reinterpret_cast<float *>(p);
        p += (static_cast<size_t>(n) * 4 + 255) / 256 * 256;
        return r;
    };
    SteWs w;
    w.colpart = take(rchunks * 2 * outs);
    w.rowpart = take(ct_out * tokens);
    w.gain_part = take(rchunks * ins);
    w.scal = take(rchunks * ct_in * 4);
    return w;
}

extern "C" int bd_ste_grad_prep(const float *grad, const float *dot, int64_t tokens, int64_t out_features,
                                const float *scale, const float *midpoint, const float *bound, int bits,
                                const int32_t *code_sums, uint16_t *dl_hi, uint16_t *dl_lo, int64_t ld_dl,
                                uint16_t *dl_t_hi, uint16_t *dl_t_lo, int64_t ld_t, float *d_scale,
                                float *d_midpoint, float *gm, void *workspace, size_t workspace_bytes,
                                bd_stream_t stream) {
    if (tokens < 1 || out_features < 1 || (bits != 4 && bits != 8) || ld_dl < out_features) return BD_ERR_INVALID;
    if ((dl_t_hi || dl_t_lo) && (!dl_t_hi || !dl_t_lo || ld_t < tokens || ld_t % 8 ||
                                 (reinterpret_cast<uintptr_t>(dl_t_hi) & 15) || (reinterpret_cast<uintptr_t>(dl_t_lo) & 15)))
        return BD_ERR_INVALID;
    if (ceil_div(tokens, kRowChunk) > 65535) return BD_ERR_INVALID;
    if (!grad || !dot || !scale || !midpoint || !bound || !code_sums || !dl_hi || !dl_lo || !d_scale ||
        !d_midpoint || !gm)
        return BD_ERR_INVALID;
    if (!workspace || workspace_bytes < bd_ste_workspace_bytes(tokens, out_features, 1)) return BD_ERR_WORKSPACE;
    const SteWs w = carve_ste(workspace, tokens, out_features, 1);
    const int rchunks = static_cast<int>(ceil_div(tokens, kRowChunk));
    const int ctiles = static_cast<int>(ceil_div(out_features, kCols));
    grad_prep_kernel<<<dim3(ctiles, rchunks), kCols, 0, stream>>>(
        grad, dot, tokens, out_features, scale, midpoint, bound, bits, code_sums,
        reinterpret_cast<__nv_bfloat16 *>(dl_hi), reinterpret_cast<__nv_bfloat16 *>(dl_lo), ld_dl,
        reinterpret_cast<__nv_bfloat16 *>(dl_t_hi), reinterpret_cast<__nv_bfloat16 *>(dl_t_lo), ld_t, w.colpart,
        w.rowpart);
    BD_CHECK_LAUNCH();
    const int64_t n = out_features > tokens ? out_features : tokens;
    grad_prep_reduce_kernel<<<static_cast<unsigned>(ceil_div(n, 256)), 256, 0, stream>>>(
        w.colpart, w.rowpart, tokens, out_features, rchunks, ctiles, scale, d_scale, d_midpoint, gm);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_ste_input_backward(const float *d_values, const float *d_values2, const float *gm, const float *x,
                                     int64_t tokens, int64_t in_features, const float *gain, const float *bound,
                                     int bits, float *dx, float *d_log_gain, float *d_log_clip, int accumulate,
                                     void *workspace, size_t workspace_bytes, bd_stream_t stream) {
    if (tokens < 1 || in_features < 1 || (bits != 4 && bits != 8)) return BD_ERR_INVALID;
    if (ceil_div(tokens, kRowChunk) > 65535) return BD_ERR_INVALID;
    if (!d_values || !gm || !x || !gain || !bound || !dx || !d_log_gain || !d_log_clip) return BD_ERR_INVALID;
    if (!workspace || workspace_bytes < bd_ste_workspace_bytes(tokens, 1, in_features)) return BD_ERR_WORKSPACE;
    const SteWs w = carve_ste(workspace, tokens, 1, in_features);
    const int rchunks = static_cast<int>(ceil_div(tokens, kRowChunk));
    const int ctiles = static_cast<int>(ceil_div(in_features, kCols));
    ste_input_kernel<<<dim3(ctiles, rchunks), kCols, 0, stream>>>(d_values, d_values2, gm, x, tokens, in_features,
                                                                   gain, bound, bits, dx, w.gain_part, w.scal);
    BD_CHECK_LAUNCH();
    ste_input_reduce_kernel<<<static_cast<unsigned>(ceil_div(in_features, 256)), 256, 0, stream>>>(
        w.gain_part, w.scal, rchunks * ctiles, in_features, rchunks, gain, bound, bits, d_log_gain, d_log_clip,
        accumulate);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

// Number of per-block partial sums bd_ste_sign_backward writes for n elements.
extern "C" int bd_ste_sumsq_count(int64_t n) { return static_cast<int>(elementwise_grid(n)); }

extern "C" int bd_ste_sign_backward(const float *grad, const float *grad2, const float *latent, int64_t n,
                                    float window, const float *bound, int bits, float *out, float *sumsq_partials,
                                    bd_stream_t stream) {
    if (n < 0 || (bound && bits != 4 && bits != 8) || !(window >= 0.0f)) return BD_ERR_INVALID;
    if (n == 0) return BD_OK;
    if (!grad || !latent || !out) return BD_ERR_INVALID;
    ste_mask_kernel<<<elementwise_grid(n), 256, 0, stream>>>(grad, grad2, latent, n, window, bound, bits, out,
                                                             sumsq_partials);
    BD_CHECK_LAUNCH();
    return BD_OK;
}
