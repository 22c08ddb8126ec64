// Row-wise elementwise chains of the training forward and their backward, one
// launch each instead of torch's chains of small kernels:
//   rms_rows_*   rms(x, w) = x * rsqrt(mean(x^2) + eps) * w over the last axis
//                (w1a1_eagle/model.py:50-51): attn/ffn/encoder/output norms;
//   head_post_*  per (row, head) of d values: the head rms with its weight
//                (q_norm / k_norm), the rotate-half rotary of the row's position
//                (model.py:54-63), and optionally the fp16 storage rounding with
//                a straight-through gradient (cache_storage, model.py:98-102).
// The elementwise operations keep the reference's order and roundings (no
// contraction: every product and sum rounds as torch's separate kernels do);
// only the mean's summation order is this kernel's.  The weight gradients come
// as per-CTA partial rows summed afterwards in a fixed order.
#include "kernels.cuh"

namespace bd {

constexpr int kRowsThreads = 256;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, d));
    return v;
}

// CTA-wide sum in a fixed order (warps in order after a butterfly within each).
__device__ __forceinline__ float cta_sum(float v, float *scratch) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float total = 0.0f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) total = __fadd_rn(total, scratch[w]);
    return total;
}

// One CTA per row.
__global__ void __launch_bounds__(kRowsThreads) rms_rows_fwd_kernel(const float *__restrict__ x, int64_t cols,
                                                                  const float *__restrict__ w, float eps,
                                                                  float *__restrict__ out, float *__restrict__ inv) {
    __shared__ float scratch[kRowsThreads / 32];
    const float *xr = x + blockIdx.x * cols;
    float ss = 0.0f;
    for (int64_t k = threadIdx.x; k < cols; k += blockDim.x) ss = __fadd_rn(ss, __fmul_rn(xr[k], xr[k]));
    const float total = cta_sum(ss, scratch);
    const float r = rsqrtf(__fadd_rn(__fdiv_rn(total, static_cast<float>(cols)), eps));
    if (threadIdx.x == 0) inv[blockIdx.x] = r;
    float *o = out + blockIdx.x * cols;
    for (int64_t k = threadIdx.x; k < cols; k += blockDim.x) o[k] = __fmul_rn(__fmul_rn(xr[k], r), w[k]);
}

// The backward in two passes, so that every CTA has work at a few hundred rows:
//   rms_rows_dot_kernel   s[row] = sum_k dy w x (one warp per row);
//   rms_rows_grad_kernel  grid (column tiles of 256, chunks of kRmsChunk rows): per
//                         thread one column, dx = r u - (r^3 / n) x s, u = dy w, and
//                         its column's dw partial over the chunk = sum dy x r.
constexpr int kRmsChunk = 16;

__global__ void __launch_bounds__(kRowsThreads) rms_rows_dot_kernel(const float *__restrict__ x, int64_t rows,
                                                                   int64_t cols, const float *__restrict__ w,
                                                                   const float *__restrict__ dy,
                                                                   float *__restrict__ total) {
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (kRowsThreads / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const float *xr = x + row * cols, *g = dy + row * cols;
    float s = 0.0f;
    const bool vec = (cols & 3) == 0 && ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(dy) |
                                          reinterpret_cast<uintptr_t>(w)) & 15) == 0;
    if (vec) {  // 16-byte loads: lane l takes columns 4 (l + 32 i) .. 4 (l + 32 i) + 3
#pragma unroll 4
        for (int64_t k = 4 * lane; k < cols; k += 128) {
            const float4 gv = *reinterpret_cast<const float4 *>(g + k), wv = *reinterpret_cast<const float4 *>(w + k);
            const float4 xv = *reinterpret_cast<const float4 *>(xr + k);
            s = __fadd_rn(s, __fmul_rn(__fmul_rn(gv.x, wv.x), xv.x));
            s = __fadd_rn(s, __fmul_rn(__fmul_rn(gv.y, wv.y), xv.y));
            s = __fadd_rn(s, __fmul_rn(__fmul_rn(gv.z, wv.z), xv.z));
            s = __fadd_rn(s, __fmul_rn(__fmul_rn(gv.w, wv.w), xv.w));
        }
    } else {
#pragma unroll 4
        for (int64_t k = lane; k < cols; k += 32) s = __fadd_rn(s, __fmul_rn(__fmul_rn(g[k], w[k]), xr[k]));
    }
    s = warp_sum(s);
    if (lane == 0) total[row] = s;
}

__global__ void __launch_bounds__(kRowsThreads) rms_rows_grad_kernel(const float *__restrict__ x, int64_t rows,
                                                                    int64_t cols, const float *__restrict__ w,
                                                                    const float *__restrict__ inv,
                                                                    const float *__restrict__ dy,
                                                                    const float *__restrict__ total,
                                                                    float *__restrict__ dx,
                                                                    float *__restrict__ dw_part) {
    const int64_t k = static_cast<int64_t>(blockIdx.x) * kRowsThreads + threadIdx.x;
    if (k >= cols) return;
    const int64_t r0 = static_cast<int64_t>(blockIdx.y) * kRmsChunk;
    const float wk = w[k];
    float gv[kRmsChunk], xv[kRmsChunk];
#pragma unroll
    for (int j = 0; j < kRmsChunk; ++j) {  // the chunk's loads in flight together
        const int64_t row = r0 + j;
        gv[j] = row < rows ? dy[row * cols + k] : 0.0f;
        xv[j] = row < rows ? x[row * cols + k] : 0.0f;
    }
    float dw = 0.0f;
#pragma unroll
    for (int j = 0; j < kRmsChunk; ++j) {
        const int64_t row = r0 + j;
        if (row >= rows) break;
        const float r = inv[row];
        const float c = __fmul_rn(__fdiv_rn(__fmul_rn(__fmul_rn(r, r), r), static_cast<float>(cols)), total[row]);
        const float u = __fmul_rn(gv[j], wk);
        dx[row * cols + k] = __fsub_rn(__fmul_rn(r, u), __fmul_rn(c, xv[j]));
        dw = __fadd_rn(dw, __fmul_rn(__fmul_rn(gv[j], xv[j]), r));
    }
    dw_part[static_cast<int64_t>(blockIdx.y) * cols + k] = dw;
}

// The weight gradient: partial rows summed in a fixed order.  A CTA takes 32
// columns; its 8 warps take the partial rows p = w, w + 8, ... (increasing p),
// and the 8 sums of a column are then added in warp order, so narrow matrices
// with many partial rows (a head's 128 columns) still spread over many threads.
constexpr int kSumCols = 32, kSumGroups = kRowsThreads / kSumCols;

__global__ void __launch_bounds__(kRowsThreads) sum_partials_kernel(const float *__restrict__ part, int64_t nparts,
                                                                    int64_t cols, float *__restrict__ out) {
    __shared__ float sums[kSumGroups][kSumCols];
    const int c = threadIdx.x & (kSumCols - 1), grp = threadIdx.x / kSumCols;
    const int64_t k = static_cast<int64_t>(blockIdx.x) * kSumCols + c;
    float s = 0.0f;
    if (k < cols) {
#pragma unroll 8
        for (int64_t p = grp; p < nparts; p += kSumGroups) s = __fadd_rn(s, part[p * cols + k]);
    }
    sums[grp][c] = s;
    __syncthreads();
    if (grp == 0 && k < cols) {
        float t = sums[0][c];
#pragma unroll
        for (int i = 1; i < kSumGroups; ++i) t = __fadd_rn(t, sums[i][c]);
        out[k] = t;
    }
}

struct HeadPostArgs {
    const float *x;  // [rows][ld_x], head h at columns h * d
    int64_t ld_x, rows;
    int heads, d;
    const float *w;        // [d] head rms weight, or null: no rms
    float eps;
    const int64_t *pos;    // [rows] positions, or null: no rotary
    const float *freq;     // [d / 2] rotary frequencies
    int fp16;              // round the output through fp16 (straight-through gradient)
    float *out;            // [rows][heads][d]
    float *inv;            // [rows][heads] rms scale (forward writes it, backward reads it)
    const float *dy;       // backward: [rows][heads][d]
    float *dx;             // backward: [rows][ld_x] (head columns only)
    float *dw_part;        // backward: [grid][d]
    int32_t *flags;
};

// One warp per (row, head); lane l holds the pairs (e, e + d/2) for e = l, l + 32, ...
// (d <= 256).
constexpr int kHeadPairs = 4;

__global__ void __launch_bounds__(kRowsThreads) head_post_fwd_kernel(const HeadPostArgs a) {
    const int lane = threadIdx.x & 31;
    const int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= a.rows * a.heads) return;
    const int64_t row = item / a.heads;
    const int h = static_cast<int>(item % a.heads);
    const int half = a.d / 2;
    const float *xr = a.x + row * a.ld_x + static_cast<int64_t>(h) * a.d;
    float lo[kHeadPairs], hi[kHeadPairs];
    float ss = 0.0f;
#pragma unroll
    for (int i = 0; i < kHeadPairs; ++i) {
        const int e = lane + 32 * i;
        lo[i] = e < half ? xr[e] : 0.0f;
        hi[i] = e < half ? xr[e + half] : 0.0f;
    }
    // the mean of squares in element order within the lane, lanes by butterfly
#pragma unroll
    for (int i = 0; i < kHeadPairs; ++i) ss = __fadd_rn(ss, __fadd_rn(__fmul_rn(lo[i], lo[i]), __fmul_rn(hi[i], hi[i])));
    float r = 1.0f;
    if (a.w) {
        r = rsqrtf(__fadd_rn(__fdiv_rn(warp_sum(ss), static_cast<float>(a.d)), a.eps));
        if (lane == 0) a.inv[item] = r;
#pragma unroll
        for (int i = 0; i < kHeadPairs; ++i) {
            const int e = lane + 32 * i;
            if (e < half) {
                lo[i] = __fmul_rn(__fmul_rn(lo[i], r), a.w[e]);
                hi[i] = __fmul_rn(__fmul_rn(hi[i], r), a.w[e + half]);
            }
        }
    }
    bool bad = false;
    float *o = a.out + item * a.d;
#pragma unroll
    for (int i = 0; i < kHeadPairs; ++i) {
        const int e = lane + 32 * i;
        if (e >= half) continue;
        float y0 = lo[i], y1 = hi[i];
        if (a.pos) {
            // value * cos + cat(-second, first) * sin, angle = position * frequency
            const float angle = __fmul_rn(static_cast<float>(a.pos[row]), a.freq[e]);
            const float c = cosf(angle), s = sinf(angle);
            y0 = __fadd_rn(__fmul_rn(lo[i], c), __fmul_rn(-hi[i], s));
            y1 = __fadd_rn(__fmul_rn(hi[i], c), __fmul_rn(lo[i], s));
        }
        if (a.fp16) {
            y0 = __half2float(__float2half_rn(y0));
            y1 = __half2float(__float2half_rn(y1));
            bad |= !isfinite(y0) || !isfinite(y1);
        }
        o[e] = y0;
        o[e + half] = y1;
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) set_flag(a.flags, BD_FLAG_CACHE_OVERFLOW);
}

// Gradient of the forward above (the fp16 rounding passes it straight through).
// The loads of one (row, head) item: its gradient and input halves, the gradient
// rotated back through the rotary (dy_e = g_e c + g_{e+h} s, dy_{e+h} = g_{e+h} c - g_e s).
struct HeadItem {
    float gl[kHeadPairs], gh[kHeadPairs], xl[kHeadPairs], xh[kHeadPairs];
};

__device__ __forceinline__ void head_item_load(const HeadPostArgs &a, int64_t item, int lane, HeadItem &it) {
    const int half = a.d / 2;
    const int64_t row = item / a.heads;
    const int h = static_cast<int>(item % a.heads);
    const float *xr = a.x + row * a.ld_x + static_cast<int64_t>(h) * a.d;
    const float *g = a.dy + item * a.d;
#pragma unroll
    for (int i = 0; i < kHeadPairs; ++i) {
        const int e = lane + 32 * i;
        const bool live = e < half;
        it.gl[i] = live ? g[e] : 0.0f;
        it.gh[i] = live ? g[e + half] : 0.0f;
        it.xl[i] = live ? xr[e] : 0.0f;
        it.xh[i] = live ? xr[e + half] : 0.0f;
    }
}

__device__ __forceinline__ void head_item_finish(const HeadPostArgs &a, int64_t item, int lane, HeadItem &it,
                                                 float (&dwl)[kHeadPairs], float (&dwh)[kHeadPairs]) {
    const int half = a.d / 2;
    const int64_t row = item / a.heads;
    const int h = static_cast<int>(item % a.heads);
    if (a.pos) {
#pragma unroll
        for (int i = 0; i < kHeadPairs; ++i) {
            const int e = lane + 32 * i;
            if (e >= half) continue;
            const float angle = __fmul_rn(static_cast<float>(a.pos[row]), a.freq[e]);
            const float c = cosf(angle), s = sinf(angle);
            const float a0 = __fadd_rn(__fmul_rn(it.gl[i], c), __fmul_rn(it.gh[i], s));
            const float a1 = __fsub_rn(__fmul_rn(it.gh[i], c), __fmul_rn(it.gl[i], s));
            it.gl[i] = a0;
            it.gh[i] = a1;
        }
    }
    float *d = a.dx + row * a.ld_x + static_cast<int64_t>(h) * a.d;
    if (!a.w) {
#pragma unroll
        for (int i = 0; i < kHeadPairs; ++i) {
            const int e = lane + 32 * i;
            if (e < half) {
                d[e] = it.gl[i];
                d[e + half] = it.gh[i];
            }
        }
        return;
    }
    const float r = a.inv[item];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < kHeadPairs; ++i) {
        const int e = lane + 32 * i;
        if (e < half)
            s = __fadd_rn(s, __fadd_rn(__fmul_rn(__fmul_rn(it.gl[i], a.w[e]), it.xl[i]),
                                       __fmul_rn(__fmul_rn(it.gh[i], a.w[e + half]), it.xh[i])));
    }
    const float c = __fdiv_rn(__fmul_rn(__fmul_rn(r, r), r), static_cast<float>(a.d)) * warp_sum(s);
#pragma unroll
    for (int i = 0; i < kHeadPairs; ++i) {
        const int e = lane + 32 * i;
        if (e >= half) continue;
        d[e] = __fsub_rn(__fmul_rn(r, __fmul_rn(it.gl[i], a.w[e])), __fmul_rn(c, it.xl[i]));
        d[e + half] = __fsub_rn(__fmul_rn(r, __fmul_rn(it.gh[i], a.w[e + half])), __fmul_rn(c, it.xh[i]));
        dwl[i] = __fadd_rn(dwl[i], __fmul_rn(__fmul_rn(it.gl[i], it.xl[i]), r));
        dwh[i] = __fadd_rn(dwh[i], __fmul_rn(__fmul_rn(it.gh[i], it.xh[i]), r));
    }
}

// Items in pairs: both items' loads are issued before either item's stores (the
// gradient and output buffers may not be assumed apart by the compiler).
__global__ void __launch_bounds__(kRowsThreads) head_post_bwd_kernel(const HeadPostArgs a, int items_per_warp) {
    extern __shared__ float dws[];  // [warps][d]
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int half = a.d / 2;
    float dwl[kHeadPairs] = {}, dwh[kHeadPairs] = {};
    const int64_t first = (static_cast<int64_t>(blockIdx.x) * nwarps + warp) * items_per_warp;
    const int64_t items = a.rows * a.heads;
    const int64_t end = first + items_per_warp < items ? first + items_per_warp : items;
    for (int64_t item = first; item < end; item += 2) {
        HeadItem it0, it1;
        head_item_load(a, item, lane, it0);
        const bool two = item + 1 < end;
        if (two) head_item_load(a, item + 1, lane, it1);
        head_item_finish(a, item, lane, it0, dwl, dwh);
        if (two) head_item_finish(a, item + 1, lane, it1, dwl, dwh);
    }
    if (!a.w) return;
#pragma unroll
    for (int i = 0; i < kHeadPairs; ++i) {
        const int e = lane + 32 * i;
        if (e < half) {
            dws[warp * a.d + e] = dwl[i];
            dws[warp * a.d + e + half] = dwh[i];
        }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < a.d; e += blockDim.x) {
        float t = 0.0f;
        for (int w = 0; w < nwarps; ++w) t = __fadd_rn(t, dws[w * a.d + e]);
        a.dw_part[static_cast<int64_t>(blockIdx.x) * a.d + e] = t;
    }
}

static int rows_grid(int64_t items, int per) { return static_cast<int>((items + per - 1) / per); }

}  // namespace bd

using namespace bd;

extern "C" int bd_rms_forward(const float *x, int64_t rows, int64_t cols, const float *weight, float eps, float *out,
                           float *inv, bd_stream_t stream) {
    if (rows < 0 || cols < 1 || rows > 0x7fffffff) return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    if (!x || !weight || !out || !inv) return BD_ERR_INVALID;
    rms_rows_fwd_kernel<<<static_cast<unsigned>(rows), kRowsThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        x, cols, weight, eps, out, inv);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

// Scratch of the backward in floats: the dw partial rows (one per chunk of rows) and
// the per-row sums.
extern "C" int64_t bd_rms_partials(int64_t rows, int64_t cols) {
    return rows < 1 || cols < 1 ? 0 : (rows + kRmsChunk - 1) / kRmsChunk * cols + rows;
}

extern "C" int bd_rms_backward(const float *x, int64_t rows, int64_t cols, const float *weight, const float *inv,
                                    const float *dy, float *dx, float *dw_partials, float *dw, bd_stream_t stream) {
    if (rows < 0 || cols < 1 || rows > 0x7fffffff) return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    if (!x || !weight || !inv || !dy || !dx || !dw_partials || !dw) return BD_ERR_INVALID;
    const int64_t chunks = (rows + kRmsChunk - 1) / kRmsChunk;
    if (chunks > 65535) return BD_ERR_INVALID;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float *total = dw_partials + chunks * cols;
    rms_rows_dot_kernel<<<rows_grid(rows, kRowsThreads / 32), kRowsThreads, 0, st>>>(x, rows, cols, weight, dy,
                                                                                     total);
    BD_CHECK_LAUNCH();
    rms_rows_grad_kernel<<<dim3(rows_grid(cols, kRowsThreads), static_cast<unsigned>(chunks)), kRowsThreads, 0, st>>>(
        x, rows, cols, weight, inv, dy, total, dx, dw_partials);
    BD_CHECK_LAUNCH();
    sum_partials_kernel<<<rows_grid(cols, kSumCols), kRowsThreads, 0, st>>>(dw_partials, chunks, cols, dw);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

static bool head_args_ok(const HeadPostArgs &a) {
    return a.rows >= 0 && a.heads >= 1 && a.d >= 2 && a.d % 2 == 0 && a.d <= 2 * 32 * kHeadPairs &&
           a.ld_x >= static_cast<int64_t>(a.heads) * a.d && a.x && a.out && (!a.pos || a.freq) && (!a.w || a.inv);
}

extern "C" int bd_head_post(const float *x, int64_t ld_x, int64_t rows, int heads, int head_dim, const float *weight,
                            float eps, const int64_t *positions, const float *frequencies, int fp16, float *out,
                            float *inv, int32_t *flags, bd_stream_t stream) {
    HeadPostArgs a{};
    a.x = x;
    a.ld_x = ld_x;
    a.rows = rows;
    a.heads = heads;
    a.d = head_dim;
    a.w = weight;
    a.eps = eps;
    a.pos = positions;
    a.freq = frequencies;
    a.fp16 = fp16;
    a.out = out;
    a.inv = inv;
    a.flags = flags;
    if (!head_args_ok(a)) return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    const int64_t items = rows * heads;
    head_post_fwd_kernel<<<rows_grid(items, kRowsThreads / 32), kRowsThreads, 0, static_cast<cudaStream_t>(stream)>>>(a);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

// (row, head) items per warp of the backward: enough warps to fill the GPU, few
// partial rows for the weight gradient.
static int head_items_per_warp(int64_t items) { return items >= 148 * 64 ? 8 : 1; }

extern "C" int64_t bd_head_post_partials(int64_t rows, int heads) {
    if (rows < 1 || heads < 1) return 0;
    const int64_t items = rows * heads;
    return rows_grid(items, static_cast<int64_t>(kRowsThreads / 32) * head_items_per_warp(items));
}

extern "C" int bd_head_post_backward(const float *x, int64_t ld_x, int64_t rows, int heads, int head_dim,
                                     const float *weight, const float *inv, const int64_t *positions,
                                     const float *frequencies, const float *dy, float *dx, float *dw_partials,
                                     float *dw, bd_stream_t stream) {
    HeadPostArgs a{};
    a.x = x;
    a.ld_x = ld_x;
    a.rows = rows;
    a.heads = heads;
    a.d = head_dim;
    a.w = weight;
    a.inv = const_cast<float *>(inv);
    a.pos = positions;
    a.freq = frequencies;
    a.out = dx;  // checked as non-null below
    a.dy = dy;
    a.dx = dx;
    a.dw_part = dw_partials;
    if (!head_args_ok(a) || !dy || !dx || (weight && (!dw_partials || !dw))) return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int64_t items = rows * heads;
    const int per = head_items_per_warp(items);
    const int64_t grid = bd_head_post_partials(rows, heads);
    const size_t smem = static_cast<size_t>(kRowsThreads / 32) * head_dim * sizeof(float);
    head_post_bwd_kernel<<<static_cast<unsigned>(grid), kRowsThreads, smem, st>>>(a, per);
    BD_CHECK_LAUNCH();
    if (weight) {
        sum_partials_kernel<<<rows_grid(head_dim, kSumCols), kRowsThreads, 0, st>>>(dw_partials, grid, head_dim,
                                                                                       dw);
        BD_CHECK_LAUNCH();
    }
    return BD_OK;
}
