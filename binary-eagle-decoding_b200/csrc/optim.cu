// The QAT update of the binary projections (w1a1_eagle/numerical/worker.py:365-392):
// global gradient-norm clip (clip_grad_norm_(..., 1.0)), fused AdamW with
// weight decay 0 (torch.optim.AdamW(fused=True), worker.py:122-130), then
// scale.clamp_(min=0) and the optional clamp_latents (model.py:167-169).
//
// The latent update is fused with the re-pack of the new signs into the W8
// decode layout, so one pass reads w, g, m, v and writes w, m, v and 1 bit per
// weight.  bound_latents (model.py:153-164) is a row kernel of its own.
#include <cmath>

#include "kernels.cuh"

namespace bd {

struct AdamScalars {
    float step_size, beta1, beta2, one_minus_beta1, one_minus_beta2, eps, bias2_sqrt;
};

// One fused AdamW element update (weight decay 0), in the order of torch's
// fused kernel: m = b1 m + (1-b1) g; v = b2 v + (1-b2) g g;
// p -= (lr / bias1) * m / (sqrt(v) / sqrt(bias2) + eps).
__device__ __forceinline__ float adam_element(float p, float g, float &m, float &v, const AdamScalars &a) {
    m = __fadd_rn(__fmul_rn(a.beta1, m), __fmul_rn(a.one_minus_beta1, g));
    v = __fadd_rn(__fmul_rn(a.beta2, v), __fmul_rn(__fmul_rn(a.one_minus_beta2, g), g));
    const float denom = __fadd_rn(__fdiv_rn(__fsqrt_rn(v), a.bias2_sqrt), a.eps);
    return __fsub_rn(p, __fdiv_rn(__fmul_rn(a.step_size, m), denom));
}

// Spread the 4 low bits of x to bit 0 of each byte.
__device__ __forceinline__ uint32_t spread4_o(uint32_t x) { return (x * 0x00204081u) & 0x01010101u; }

// W8 word of (row, 128-column half h of a 256-column pair, lane t) from the 8
// ballot words g of the pair (bit l of g[i] = column 32 i + l): bit 8 j + 2 ks + r
// is column 128 h + 32 ks + 16 r + 4 t + j.
__device__ __forceinline__ uint32_t w8_word_o(const uint32_t *g, int h, int t) {
    uint32_t out = 0;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
        const uint32_t word = g[4 * h + ks];
        out |= spread4_o((word >> (4 * t)) & 0xFu) << (2 * ks);
        out |= spread4_o((word >> (16 + 4 * t)) & 0xFu) << (2 * ks + 1);
    }
    return out;
}

// One warp per (row, 256-column pair): update 256 latents, ballot their new
// signs into eight words and emit the row's (up to) eight W8 words.
__global__ void __launch_bounds__(256) adamw_latent_kernel(float *__restrict__ param, const float *__restrict__ grad,
                                                           float *__restrict__ m, float *__restrict__ v, int64_t rows,
                                                           int64_t cols, AdamScalars a,
                                                           const float *__restrict__ clip_coef, int clamp,
                                                           uint32_t *__restrict__ tiled, int stride, int offset,
                                                           int32_t *flags) {
    const int lane = threadIdx.x & 31;
    const int64_t ncp = (cols + 255) / 256;
    const int64_t nw = (cols + 127) / 128;
    const int64_t rows_pad = (rows + 7) / 8 * 8;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const float coef = clip_coef ? __ldg(clip_coef) : 1.0f;
    bool bad = false;
    for (int64_t item = warp; item < rows_pad * ncp; item += nwarps) {
        const int64_t row = item / ncp, cp = item - row * ncp;
        // all 32 loads of the item first (8 columns x p, g, m, v), so a warp keeps
        // 4 KB in flight instead of one column's 512 B
        float pv[8], gv[8], mv[8], vv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t c = cp * 256 + i * 32 + lane;
            if (row < rows && c < cols) {
                const int64_t e = row * cols + c;
                pv[i] = param[e];
                gv[i] = grad[e];
                mv[i] = m[e];
                vv[i] = v[e];
            }
        }
        uint32_t words[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t c = cp * 256 + i * 32 + lane;
            bool bit = false;
            if (row < rows && c < cols) {
                const int64_t e = row * cols + c;
                float mm = mv[i], vvi = vv[i];
                float p = adam_element(pv[i], __fmul_rn(gv[i], coef), mm, vvi, a);
                if (clamp) p = fminf(fmaxf(p, -1.0f), 1.0f);
                bad |= !isfinite(p);
                param[e] = p;
                m[e] = mm;
                v[e] = vvi;
                bit = p >= 0.0f;
            }
            words[i] = __ballot_sync(0xffffffffu, bit);
        }
        if (tiled && lane < 8) {
            const int h = lane >> 2, t = lane & 3;
            const int64_t w = 2 * cp + h;
            if (w < nw) {  // W8 stores words in groups of four per lane: [n][w / 4][lane][w % 4]
                const int64_t n = (row >> 3) * stride + offset;
                const int64_t ng = (nw + 3) / 4;
                tiled[((n * ng + (w >> 2)) * 32 + (row & 7) * 4 + t) * 4 + (w & 3)] = w8_word_o(words, h, t);
            }
        }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) set_flag(flags, BD_FLAG_NONFINITE_STATE);
}

// Element AdamW for the small parameters, optional lower clamp (scale.clamp_(min=0)).
__global__ void adamw_kernel(float *__restrict__ param, const float *__restrict__ grad, float *__restrict__ m,
                             float *__restrict__ v, int64_t n, AdamScalars a, const float *__restrict__ clip_coef,
                             float lower, int32_t *flags) {
    const float coef = clip_coef ? __ldg(clip_coef) : 1.0f;
    bool bad = false;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float mm = m[i], vv = v[i];
        float p = adam_element(param[i], __fmul_rn(grad[i], coef), mm, vv, a);
        p = fmaxf(p, lower);
        bad |= !isfinite(p);
        param[i] = p;
        m[i] = mm;
        v[i] = vv;
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_NONFINITE_STATE);
}

__device__ __forceinline__ float block_sum_o(float v, float *scratch) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, d));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = scratch[0];
    for (int w = 1; w < static_cast<int>(blockDim.x / 32); ++w) s = __fadd_rn(s, scratch[w]);
    return s;
}

// Per-block sums of squares (fixed order) into partials[blockIdx.x].
__global__ void __launch_bounds__(256) sum_squares_kernel(const float *__restrict__ x, int64_t n,
                                                          float *__restrict__ partials) {
    __shared__ float scratch[8];
    float s = 0.0f;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
    s = block_sum_o(s, scratch);
    if (threadIdx.x == 0) partials[blockIdx.x] = s;
}

// total = sqrt(sum partials); coef = min(1, max_norm / (total + 1e-6)) (clip_grad_norm_).
__global__ void __launch_bounds__(256) grad_norm_kernel(const float *__restrict__ partials, int64_t count,
                                                        float max_norm, float *__restrict__ total,
                                                        float *__restrict__ coef, int32_t *flags) {
    __shared__ float scratch[8];
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < count; i += blockDim.x) s = __fadd_rn(s, partials[i]);
    s = block_sum_o(s, scratch);
    if (threadIdx.x == 0) {
        const float norm = __fsqrt_rn(s);
        total[0] = norm;
        if (!isfinite(norm)) set_flag(flags, BD_FLAG_NONFINITE_STATE);
        const float c = __fdiv_rn(max_norm, __fadd_rn(norm, 1e-6f));
        coef[0] = fminf(c, 1.0f);
    }
}

// bound_latents: out = clamp(latent / (multiple * mean|row|), -1, 1) (mean 0 -> divide by 1);
// a sign change (a negative value rounding to -0.0) raises the flag.
__global__ void __launch_bounds__(256) bound_latents_kernel(const float *__restrict__ latent, int64_t cols,
                                                            float multiple, float *__restrict__ out,
                                                            int32_t *flags) {
    __shared__ float scratch[8];
    const int64_t row = blockIdx.x;
    const float *src = latent + row * cols;
    float s = 0.0f;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) s = __fadd_rn(s, fabsf(src[c]));
    s = block_sum_o(s, scratch);
    const float mean = __fdiv_rn(s, static_cast<float>(cols));
    const float denom = mean > 0.0f ? __fmul_rn(mean, multiple) : 1.0f;
    bool changed = false;
    for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
        const float v = src[c];
        const float b = fminf(fmaxf(__fdiv_rn(v, denom), -1.0f), 1.0f);
        changed |= (b >= 0.0f) != (v >= 0.0f);
        out[row * cols + c] = b;
    }
    if (__any_sync(0xffffffffu, changed) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_SIGN_CHANGE);
}

__global__ void clamp_kernel(float *__restrict__ x, int64_t n, float lo, float hi) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        x[i] = fminf(fmaxf(x[i], lo), hi);
}

}  // namespace bd

using namespace bd;

static unsigned grid_elems(int64_t n) {
    int64_t g = (n + 255) / 256;
    if (g < 1) g = 1;
    if (g > 148 * 32) g = 148 * 32;
    return static_cast<unsigned>(g);
}

static bool adam_ok(double lr, double beta1, double beta2, double eps, long long step) {
    return lr >= 0.0 && beta1 >= 0.0 && beta1 < 1.0 && beta2 >= 0.0 && beta2 < 1.0 && eps >= 0.0 && step >= 1;
}

// Hyperparameters arrive as doubles (as torch holds them); 1 - beta, the bias
// corrections and lr / bias1 are formed in double and rounded once to fp32.
static AdamScalars adam_scalars(double lr, double beta1, double beta2, double eps, long long step) {
    AdamScalars a;
    const double bias1 = 1.0 - std::pow(beta1, static_cast<double>(step));
    const double bias2 = 1.0 - std::pow(beta2, static_cast<double>(step));
    a.step_size = static_cast<float>(lr / bias1);
    a.beta1 = static_cast<float>(beta1);
    a.beta2 = static_cast<float>(beta2);
    a.one_minus_beta1 = static_cast<float>(1.0 - beta1);
    a.one_minus_beta2 = static_cast<float>(1.0 - beta2);
    a.eps = static_cast<float>(eps);
    a.bias2_sqrt = static_cast<float>(std::sqrt(bias2));
    return a;
}

extern "C" int bd_adamw_latent(float *param, const float *grad, float *exp_avg, float *exp_avg_sq, int64_t rows,
                               int64_t cols, double lr, double beta1, double beta2, double eps, long long step,
                               const float *clip_coef, int clamp_latents, uint32_t *signs_w8, int block_stride,
                               int block_offset, int32_t *flags, bd_stream_t stream) {
    if (rows < 0 || cols < 1 || !adam_ok(lr, beta1, beta2, eps, step) || block_stride < 1 || block_offset < 0 ||
        block_offset >= block_stride)
        return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    if (!param || !grad || !exp_avg || !exp_avg_sq) return BD_ERR_INVALID;
    const int64_t items = (rows + 7) / 8 * 8 * ((cols + 255) / 256);
    adamw_latent_kernel<<<grid_elems(items * 32), 256, 0, stream>>>(
        param, grad, exp_avg, exp_avg_sq, rows, cols, adam_scalars(lr, beta1, beta2, eps, step), clip_coef,
        clamp_latents, signs_w8, block_stride, block_offset, flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_adamw(float *param, const float *grad, float *exp_avg, float *exp_avg_sq, int64_t n, double lr,
                        double beta1, double beta2, double eps, long long step, const float *clip_coef, float lower,
                        int32_t *flags, bd_stream_t stream) {
    if (n < 0 || !adam_ok(lr, beta1, beta2, eps, step)) return BD_ERR_INVALID;
    if (n == 0) return BD_OK;
    if (!param || !grad || !exp_avg || !exp_avg_sq) return BD_ERR_INVALID;
    adamw_kernel<<<grid_elems(n), 256, 0, stream>>>(param, grad, exp_avg, exp_avg_sq, n,
                                                     adam_scalars(lr, beta1, beta2, eps, step), clip_coef, lower,
                                                     flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_sum_squares_count(int64_t n) { return static_cast<int>(grid_elems(n)); }

extern "C" int bd_sum_squares(const float *x, int64_t n, float *partials, bd_stream_t stream) {
    if (n < 1 || !x || !partials) return BD_ERR_INVALID;
    sum_squares_kernel<<<grid_elems(n), 256, 0, stream>>>(x, n, partials);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_grad_norm(const float *partials, int64_t count, float max_norm, float *total_norm,
                            float *clip_coef, int32_t *flags, bd_stream_t stream) {
    if (count < 1 || !partials || !total_norm || !clip_coef || !(max_norm > 0.0f)) return BD_ERR_INVALID;
    grad_norm_kernel<<<1, 256, 0, stream>>>(partials, count, max_norm, total_norm, clip_coef, flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_bound_latents(const float *latent, int64_t rows, int64_t cols, float multiple, float *out,
                                int32_t *flags, bd_stream_t stream) {
    if (rows < 0 || cols < 1 || rows > 0x7fffffff || !(multiple > 0.0f)) return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    if (!latent || !out) return BD_ERR_INVALID;
    bound_latents_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(latent, cols, multiple, out, flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_clamp(float *x, int64_t n, float lo, float hi, bd_stream_t stream) {
    if (n < 0 || !(lo <= hi)) return BD_ERR_INVALID;
    if (n == 0) return BD_OK;
    if (!x) return BD_ERR_INVALID;
    clamp_kernel<<<grid_elems(n), 256, 0, stream>>>(x, n, lo, hi);
    BD_CHECK_LAUNCH();
    return BD_OK;
}
