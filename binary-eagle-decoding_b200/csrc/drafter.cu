// Small per-row kernels of the block-drafter forward (w1a1_eagle/model.py):
// embedding gather, rms rows, and the per-head q/k/v post-processing
// (rms over the head with its norm weight, rotary embedding, fp16 storage with
// the cache_storage overflow check).
#include <cmath>

#include "kernels.cuh"

#include <cuda_fp16.h>

namespace bd {

// Rotary frequencies theta^(-2j/d) for j < d/2, computed once on the host
// (model.py:56-57: the exponent 2j/d as fp32, then the power), so every kernel and
// every position uses the same fp32 frequency and the fp32 angle pos * f_j is
// exactly the reference's.
constexpr int kRopeMax = 128;  // head_dim <= 256
struct RopeTable {
    float f[kRopeMax];
};

// out_j = v_j cos(a) - v_{j+d/2} sin(a), out_{j+d/2} = v_{j+d/2} cos(a) + v_j sin(a),
// a = pos * f_j, each product rounded as in the reference (no fused multiply-add).
__device__ __forceinline__ void rotate_pair(float &a, float &b, int64_t pos, float freq) {
    const float angle = __fmul_rn(static_cast<float>(pos), freq);
    float s, c;
    sincosf(angle, &s, &c);
    const float na = __fadd_rn(__fmul_rn(a, c), __fmul_rn(-b, s));
    const float nb = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
    a = na;
    b = nb;
}

// state[t] = vocabulary[ids[t]] (bf16 table -> fp32), HE4.forward's embedding (model.py:380-381).
__global__ void embed_kernel(const uint16_t *__restrict__ table, int64_t vocab, int64_t hidden,
                             const int32_t *__restrict__ ids, float *__restrict__ out, int32_t *flags) {
    grid_wait();
    grid_launch_dependents();
    const int t = blockIdx.x;
    int id = ids[t];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) set_flag(flags, BD_FLAG_BAD_TOKEN);
        id = 0;
    }
    const uint16_t *row = table + id * hidden;
    for (int64_t k = threadIdx.x; k < hidden; k += blockDim.x)
        out[t * hidden + k] = __uint_as_float(static_cast<uint32_t>(row[k]) << 16);
}

__device__ __forceinline__ float block_sum(float v, float *part) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    const int warps = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = v;
    __syncthreads();
    float total = 0.0f;
    for (int w = 0; w < warps; ++w) total += part[w];
    return total;
}

// out = x * rsqrt(mean(x^2) + eps) * w (model.py:50-51), one CTA per row.
__global__ void rms_rows_kernel(const float *__restrict__ x, int64_t cols, int64_t ldx, const float *__restrict__ w,
                                float eps, float *__restrict__ out, int64_t ldo) {
    __shared__ float part[32];
    grid_wait();
    grid_launch_dependents();
    const float *row = x + blockIdx.x * ldx;
    float ss = 0.0f;
    for (int64_t k = threadIdx.x; k < cols; k += blockDim.x) ss = fmaf(row[k], row[k], ss);
    const float scale = rsqrtf(block_sum(ss, part) / static_cast<float>(cols) + eps);
    for (int64_t k = threadIdx.x; k < cols; k += blockDim.x) out[blockIdx.x * ldo + k] = row[k] * scale * w[k];
}

// Heads of row r of src (columns col0 + h * d ...): optional rms over the head
// with weight nw, optional rotary embedding at position pos0 + r
// (model.py:54-63: out_j = v_j cos(a_j) - v_{j+d/2} sin(a_j), out_{j+d/2} =
// v_{j+d/2} cos(a_j) + v_j sin(a_j), a_j = pos * theta^(-2j/d)), stored as fp16
// at dst[(r * heads + h) * d + j] of a row stride dst_ld (elements).
// Grid (rows, heads), d/2 threads.
__global__ void heads_post_kernel(const float *__restrict__ src, int64_t ld_src, int64_t col0, int heads, int d,
                                  const float *__restrict__ nw, float eps, int rope, const RopeTable freqs, int64_t pos0,
                                  __half *__restrict__ dst, int64_t dst_ld, int32_t *flags) {
    __shared__ float part[32];
    grid_wait();
    grid_launch_dependents();
    const int r = blockIdx.x, h = blockIdx.y, j = threadIdx.x, half = d >> 1;
    const bool live = j < half;  // the block is padded to whole warps
    const float *v = src + r * ld_src + col0 + h * d;
    float a = live ? v[j] : 0.0f, b = live ? v[j + half] : 0.0f;
    if (nw) {
        const float scale = rsqrtf(block_sum(fmaf(a, a, b * b), part) / static_cast<float>(d) + eps);
        if (live) {
            a = a * scale * nw[j];
            b = b * scale * nw[j + half];
        }
    }
    if (!live) return;
    if (rope) rotate_pair(a, b, pos0 + r, freqs.f[j]);
    const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    if (!isfinite(__half2float(ha)) || !isfinite(__half2float(hb))) set_flag(flags, BD_FLAG_CACHE_OVERFLOW);
    __half *out = dst + r * dst_ld + h * d;
    out[j] = ha;
    out[j + half] = hb;
}

// q, k and v of a projected row block in one launch: grid (rows, heads + 2 kv_heads,
// layers); q heads get q_norm + rope -> q (row stride q_ld), k heads k_norm + rope
// -> the K cache row pos0 + r, v heads are stored as they are in the V cache.
// Layer z reads columns from z * src_layer, norm weights from z * norm_layer and
// writes cache rows at z * cache_layer (context rows of every layer at once).
__global__ void qkv_post_kernel(const float *__restrict__ src, int64_t ld_src, int heads, int kv_heads, int d,
                                const float *__restrict__ q_norm, const float *__restrict__ k_norm, float eps,
                                const RopeTable freqs, int64_t pos0, float *__restrict__ q, int64_t q_ld,
                                __half *__restrict__ kc, __half *__restrict__ vc, int64_t kv_ld, int64_t src_layer,
                                int64_t norm_layer, int64_t cache_layer, int32_t *flags) {
    __shared__ float part[32];
    grid_wait();
    grid_launch_dependents();
    const int r = blockIdx.x, y = blockIdx.y, j = threadIdx.x, half = d >> 1;
    src += blockIdx.z * src_layer;
    k_norm += blockIdx.z * norm_layer;
    kc += blockIdx.z * cache_layer;
    vc += blockIdx.z * cache_layer;
    const bool live = j < half;
    const float *v = src + r * ld_src + static_cast<int64_t>(y) * d;
    const float *nw = y < heads ? q_norm : (y < heads + kv_heads ? k_norm : nullptr);
    const bool rope = y < heads + kv_heads;
    // q rows stay fp32 (the attention splits them into fp16 hi + lo); k and v
    // rows are stored in the fp16 cache
    __half *out = y < heads ? nullptr
                            : (y < heads + kv_heads ? kc + r * kv_ld + (y - heads) * d
                                                    : vc + r * kv_ld + (y - heads - kv_heads) * d);
    float a = live ? v[j] : 0.0f, b = live ? v[j + half] : 0.0f;
    if (nw) {
        const float scale = rsqrtf(block_sum(fmaf(a, a, b * b), part) / static_cast<float>(d) + eps);
        if (live) {
            a = a * scale * nw[j];
            b = b * scale * nw[j + half];
        }
    }
    if (!live) return;
    if (rope) rotate_pair(a, b, pos0 + r, freqs.f[j]);
    if (y < heads) {
        float *qo = q + r * q_ld + static_cast<int64_t>(y) * d;
        qo[j] = a;
        qo[j + half] = b;
        return;
    }
    const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    if (!isfinite(__half2float(ha)) || !isfinite(__half2float(hb))) set_flag(flags, BD_FLAG_CACHE_OVERFLOW);
    out[j] = ha;
    out[j + half] = hb;
}

static RopeTable rope_table(float theta, int d) {
    RopeTable r{};
    for (int j = 0; j < d / 2 && j < kRopeMax; ++j) {
        const float e = -(static_cast<float>(2 * j) / static_cast<float>(d));
        r.f[j] = static_cast<float>(std::pow(static_cast<double>(theta), static_cast<double>(e)));
    }
    return r;
}

}  // namespace bd

using namespace bd;

extern "C" int bd_qkv_post(const float *src, int n, int64_t ld_src, int heads, int kv_heads, int head_dim,
                           const float *q_norm, const float *k_norm, float epsilon, float theta, int64_t pos0,
                           float *q_out, int64_t q_ld, uint16_t *k_cache_f16, uint16_t *v_cache_f16, int64_t kv_ld,
                           int32_t *flags, bd_stream_t stream) {
    // heads == 0: a k|v row block only (context rows), q pointers unused
    if (n < 1 || heads < 0 || kv_heads < 1 || head_dim < 2 || (head_dim & 1) || head_dim > 2 * kRopeMax || !src ||
        (heads > 0 && (!q_out || !q_norm)) || !k_cache_f16 || !v_cache_f16 || !k_norm)
        return BD_ERR_INVALID;
    const unsigned threads = static_cast<unsigned>((head_dim / 2 + 31) / 32 * 32);
    return launch_pdl(qkv_post_kernel, dim3(n, heads + 2 * kv_heads, 1), dim3(threads), 0, stream, src, ld_src, heads,
                      kv_heads, head_dim, q_norm, k_norm, epsilon, rope_table(theta, head_dim), pos0, q_out, q_ld,
                      reinterpret_cast<__half *>(k_cache_f16), reinterpret_cast<__half *>(v_cache_f16), kv_ld,
                      int64_t{0}, int64_t{0}, int64_t{0}, flags);
}

extern "C" int bd_context_kv_post(const float *src, int n, int64_t ld_src, int layers, int64_t layer_cols,
                                  int kv_heads, int head_dim, const float *k_norms, float epsilon, float theta,
                                  int64_t pos0, uint16_t *k_cache_f16, uint16_t *v_cache_f16, int64_t kv_ld,
                                  int64_t cache_layer_stride, int32_t *flags, bd_stream_t stream) {
    if (n < 1 || layers < 1 || layers > 65535 || kv_heads < 1 || head_dim < 2 || (head_dim & 1) ||
        head_dim > 2 * kRopeMax || !src || !k_norms || !k_cache_f16 || !v_cache_f16 ||
        layer_cols < 2 * kv_heads * static_cast<int64_t>(head_dim) ||
        ld_src < (layers - 1) * layer_cols + 2 * kv_heads * static_cast<int64_t>(head_dim) ||
        kv_ld < kv_heads * static_cast<int64_t>(head_dim) || cache_layer_stride < 0)
        return BD_ERR_INVALID;
    const unsigned threads = static_cast<unsigned>((head_dim / 2 + 31) / 32 * 32);
    return launch_pdl(qkv_post_kernel, dim3(n, 2 * kv_heads, layers), dim3(threads), 0, stream, src, ld_src, 0,
                      kv_heads, head_dim, static_cast<const float *>(nullptr), k_norms, epsilon,
                      rope_table(theta, head_dim), pos0, static_cast<float *>(nullptr), int64_t{0},
                      reinterpret_cast<__half *>(k_cache_f16), reinterpret_cast<__half *>(v_cache_f16), kv_ld,
                      layer_cols, static_cast<int64_t>(head_dim), cache_layer_stride, flags);
}

extern "C" int bd_embed_rows(const uint16_t *table, int64_t vocab, int64_t hidden, const int32_t *ids, int n,
                             float *out, int32_t *flags, bd_stream_t stream) {
    if (vocab < 1 || hidden < 1 || n < 1 || !table || !ids || !out) return BD_ERR_INVALID;
    return launch_pdl(embed_kernel, dim3(n), dim3(256), 0, stream, table, vocab, hidden, ids, out, flags);
}

extern "C" int bd_rms_rows(const float *x, int n, int64_t cols, int64_t ldx, const float *weight, float epsilon,
                           float *out, int64_t ldo, bd_stream_t stream) {
    if (n < 1 || cols < 1 || ldx < cols || ldo < cols || !x || !weight || !out) return BD_ERR_INVALID;
    return launch_pdl(rms_rows_kernel, dim3(n), dim3(256), 0, stream, x, cols, ldx, weight, epsilon, out, ldo);
}

extern "C" int bd_heads_post(const float *src, int n, int64_t ld_src, int64_t col0, int heads, int head_dim,
                             const float *norm_weight, float epsilon, int rope, float theta, int64_t pos0,
                             uint16_t *dst_f16, int64_t dst_ld, int32_t *flags, bd_stream_t stream) {
    if (n < 1 || heads < 1 || head_dim < 2 || (head_dim & 1) || head_dim > 2048 || !src || !dst_f16 ||
        (rope && head_dim > 2 * kRopeMax))
        return BD_ERR_INVALID;
    const unsigned threads = static_cast<unsigned>((head_dim / 2 + 31) / 32 * 32);
    return launch_pdl(heads_post_kernel, dim3(n, heads), dim3(threads), 0, stream, src, ld_src, col0, heads,
                      head_dim, norm_weight, epsilon, rope, rope_table(theta, head_dim), pos0,
                      reinterpret_cast<__half *>(dst_f16), dst_ld,
                      flags);
}

extern "C" int bd_round_submit(void *graph_exec, const void *host_rows, void *dev_rows, size_t row_bytes,
                               const int32_t *host_first, int32_t *dev_first, const int32_t *dev_drafted,
                               int32_t *host_drafted, int drafted, bd_stream_t stream) {
    if (!graph_exec || (row_bytes && (!host_rows || !dev_rows)) || (host_first && !dev_first) || drafted < 0 ||
        (drafted && (!dev_drafted || !host_drafted)))
        return BD_ERR_INVALID;
    if (row_bytes && cudaMemcpyAsync(dev_rows, host_rows, row_bytes, cudaMemcpyHostToDevice, stream) != cudaSuccess)
        return BD_ERR_LAUNCH;
    if (host_first &&
        cudaMemcpyAsync(dev_first, host_first, sizeof(int32_t), cudaMemcpyHostToDevice, stream) != cudaSuccess)
        return BD_ERR_LAUNCH;
    if (cudaGraphLaunch(static_cast<cudaGraphExec_t>(graph_exec), stream) != cudaSuccess) return BD_ERR_LAUNCH;
    if (drafted && cudaMemcpyAsync(host_drafted, dev_drafted, drafted * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                   stream) != cudaSuccess)
        return BD_ERR_LAUNCH;
    return cudaStreamSynchronize(stream) == cudaSuccess ? BD_OK : BD_ERR_LAUNCH;
}
