// bf16 matrix x small activation block (tokens <= 32): the attention projections,
// context fusion and the tied LM head of the drafter.  HBM-bound: every weight
// byte is read once, straight into registers, in a tile order where each lane's
// 16-byte load is exactly its m16n8k16 A fragment (W16 layout).  Activations
// are split into bf16 hi + lo planes (x ~= hi + lo to ~16 bits) laid out as B
// fragments (X16 layout), so the fp32 accumulation sees ~fp32-quality inputs
// for the cost of a second MMA the HBM stream hides.  Each CTA owns RB row
// blocks; its 8 warps split K and their partial sums are added in a fixed order
// through shared memory (deterministic).  Epilogues: store (+ residual) and a
// running per-token argmax (largest value, lowest row on ties) kept as 64-bit
// keys updated with atomicMax.
#include <algorithm>

#include "kernels.cuh"

namespace bd {

constexpr int kGemvUnroll = 4;  // K tiles per register stage

struct GemvArgs {
    const uint4 *w;              // W16 tiles
    int64_t rows, cols, nkt;     // O, K (unpadded), K tiles of 16
    const uint2 *x;              // X16 fragments: [plane][ntb][nkt][32]
    int64_t ntb;                 // token blocks of 8 in the X16 buffer
    int tokens;
    float *out;                  // [tokens][ld_out] or null
    int64_t ld_out;
    const float *residual;       // [tokens][ld_out] or null
    unsigned long long *argmax;  // [tokens] running keys or null
    int32_t *flags;
    int splits;                  // CTAs along K (blockIdx.y); > 1 needs partial + counters
    float *partial;              // [splits][gridDim.x][cells]
    int32_t *counters;           // [gridDim.x], zero on entry, left zero
};

__device__ __forceinline__ unsigned long long order_key(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | static_cast<unsigned long long>(~idx);
}

template <int RB>
__device__ __forceinline__ void gemv_issue(uint4 (&wa)[kGemvUnroll][RB], const uint4 *const (&wrow)[RB], int64_t kt,
                                           int64_t kt1) {
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u)
#pragma unroll
        for (int r = 0; r < RB; ++r)
            if (kt + u < kt1) wa[u][r] = ld_stream_u4(wrow[r] + (kt + u) * 32);
}

// One batch of kGemvUnroll K tiles: the activation fragments of all tiles are
// requested together (they are L2 hits, but each round trip is long), then the MMAs.
template <int NT, int RB>
__device__ __forceinline__ void gemv_compute(float (&acc)[RB][NT][4], const uint4 (&wa)[kGemvUnroll][RB],
                                             const uint2 *x, int64_t plane, int64_t nkt, int64_t kt, int64_t kt1,
                                             int lane) {
    uint2 xb[kGemvUnroll][2][NT];
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u)
        if (kt + u < kt1)
#pragma unroll
            for (int p = 0; p < 2; ++p)
#pragma unroll
                for (int n = 0; n < NT; ++n) xb[u][p][n] = __ldg(x + p * plane + (n * nkt + kt + u) * 32 + lane);
#pragma unroll
    for (int u = 0; u < kGemvUnroll; ++u) {
        if (kt + u < kt1) {
#pragma unroll
            for (int r = 0; r < RB; ++r)
#pragma unroll
                for (int p = 0; p < 2; ++p)
#pragma unroll
                    for (int n = 0; n < NT; ++n)
                        mma_bf16_16816(acc[r][n], wa[u][r].x, wa[u][r].y, wa[u][r].z, wa[u][r].w, xb[u][p][n].x,
                                       xb[u][p][n].y);
        }
    }
}

template <int NT, int RB, int W>
__global__ void __launch_bounds__(W * 32) gemv_kernel(const GemvArgs a) {
    constexpr int kGemvWarps = W, kGemvThreads = W * 32;
    __shared__ float red[kGemvWarps][RB * NT * 4][32];
    __shared__ unsigned long long best[32];
    __shared__ int last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t nrb = (a.rows + 15) / 16;
    const int64_t rb0 = static_cast<int64_t>(blockIdx.x) * RB;
    // this CTA's K range, split over its warps
    const int64_t ck0 = blockIdx.y * a.nkt / a.splits, ck1 = (blockIdx.y + 1) * a.nkt / a.splits;
    const int64_t kt0 = ck0 + warp * (ck1 - ck0) / kGemvWarps, kt1 = ck0 + (warp + 1) * (ck1 - ck0) / kGemvWarps;
    float acc[RB][NT][4];
#pragma unroll
    for (int r = 0; r < RB; ++r)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[r][n][i] = 0.0f;

    const uint4 *wrow[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) wrow[r] = a.w + (rb0 + r < nrb ? rb0 + r : nrb - 1) * a.nkt * 32 + lane;
    const int64_t plane = a.ntb * a.nkt * 32;

    // one register stage per warp; HBM latency is hidden by the many resident
    // warps (a second stage costs registers, hence occupancy, and measured slower)
    uint4 wa[kGemvUnroll][RB];
    gemv_issue<RB>(wa, wrow, kt0, kt1);  // weights are read-only: before the dependency wait
    grid_wait();
    grid_launch_dependents();
    if (threadIdx.x < 32) best[threadIdx.x] = 0ull;
    for (int64_t kt = kt0; kt < kt1; kt += kGemvUnroll) {
        gemv_compute<NT, RB>(acc, wa, a.x, plane, a.nkt, kt, kt1, lane);
        gemv_issue<RB>(wa, wrow, kt + kGemvUnroll, kt1);
    }
#pragma unroll
    for (int r = 0; r < RB; ++r)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) red[warp][(r * NT + n) * 4 + i][lane] = acc[r][n][i];
    __syncthreads();
    // every thread finishes cells (value slot v, lane l) summing warps 0..7 in order
    constexpr int CELLS = RB * NT * 4 * 32;
    float sums[(CELLS + kGemvThreads - 1) / kGemvThreads];
#pragma unroll
    for (int q = 0; q < (CELLS + kGemvThreads - 1) / kGemvThreads; ++q) {
        const int c = threadIdx.x + q * kGemvThreads;
        float s = 0.0f;
        if (c < CELLS) {
            const int l = c & 31, v = c >> 5;
            s = red[0][v][l];
#pragma unroll
            for (int w = 1; w < kGemvWarps; ++w) s = __fadd_rn(s, red[w][v][l]);
        }
        sums[q] = s;
    }
    if (a.splits > 1) {
        // K split over CTAs: partials meet in global memory; the last CTA of this
        // row group adds them in split order (deterministic) and finishes.
        float *mine = a.partial + (static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x) * CELLS;
#pragma unroll
        for (int q = 0; q < (CELLS + kGemvThreads - 1) / kGemvThreads; ++q) {
            const int c = threadIdx.x + q * kGemvThreads;
            if (c < CELLS) mine[c] = sums[q];
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) last = atomicAdd(a.counters + blockIdx.x, 1) == a.splits - 1;
        __syncthreads();
        if (!last) return;
        __threadfence();
#pragma unroll
        for (int q = 0; q < (CELLS + kGemvThreads - 1) / kGemvThreads; ++q) {
            const int c = threadIdx.x + q * kGemvThreads;
            float s = 0.0f;
            if (c < CELLS)
                for (int ks = 0; ks < a.splits; ++ks)
                    s = __fadd_rn(s, __ldcg(a.partial + (static_cast<int64_t>(ks) * gridDim.x + blockIdx.x) * CELLS + c));
            sums[q] = s;
        }
        if (threadIdx.x == 0) atomicExch(a.counters + blockIdx.x, 0);
    }
    bool bad = false;
#pragma unroll
    for (int q = 0; q < (CELLS + kGemvThreads - 1) / kGemvThreads; ++q) {
        const int c = threadIdx.x + q * kGemvThreads;
        if (c >= CELLS) continue;
        float s = sums[q];
        const int l = c & 31, v = c >> 5;
        const int i = v & 3, n = (v >> 2) % NT, r = (v >> 2) / NT;
        const int g = l >> 2, t = l & 3;
        const int64_t o = (rb0 + r) * 16 + g + 8 * (i >> 1);
        const int token = n * 8 + 2 * t + (i & 1);
        if (o >= a.rows || token >= a.tokens) continue;
        if (a.residual) s = __fadd_rn(a.residual[token * a.ld_out + o], s);
        if (a.out) a.out[token * a.ld_out + o] = s;
        if (a.argmax) {
            if (isfinite(s))
                atomicMax(best + token, order_key(s, static_cast<uint32_t>(o)));
            else
                bad = true;
        }
    }
    if (a.argmax) {
        if (__any_sync(0xffffffffu, bad) && lane == 0) set_flag(a.flags, BD_FLAG_NONFINITE_STATE);
        __syncthreads();
        if (threadIdx.x < a.tokens && best[threadIdx.x]) atomicMax(a.argmax + threadIdx.x, best[threadIdx.x]);
    }
}

// W16 tiles from fp32 or bf16 row-major weights; one thread per lane-slot (8 values).
template <typename T>
__global__ void tile_w16_kernel(const T *__restrict__ w, int64_t rows, int64_t cols, int64_t nkt,
                                uint16_t *__restrict__ out) {
    const int64_t nrb = (rows + 15) / 16;
    const int64_t total = nrb * nkt * 32;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int lane = static_cast<int>(i & 31);
        const int64_t rest = i >> 5;
        const int64_t kt = rest % nkt, rb = rest / nkt;
        const int g = lane >> 2, t = lane & 3;
        uint16_t v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const int64_t row = rb * 16 + g + 8 * ((e >> 1) & 1);
            const int64_t col = kt * 16 + 2 * t + (e & 1) + 8 * (e >> 2);
            float f = 0.0f;
            if (row < rows && col < cols) {
                if constexpr (sizeof(T) == 4)
                    f = static_cast<float>(w[row * cols + col]);
                else
                    f = __uint_as_float(static_cast<uint32_t>(reinterpret_cast<const uint16_t *>(w)[row * cols + col]) << 16);
            }
            v[e] = __bfloat16_as_ushort(__float2bfloat16_rn(f));
        }
        uint4 packed;
        packed.x = v[0] | (static_cast<uint32_t>(v[1]) << 16);
        packed.y = v[2] | (static_cast<uint32_t>(v[3]) << 16);
        packed.z = v[4] | (static_cast<uint32_t>(v[5]) << 16);
        packed.w = v[6] | (static_cast<uint32_t>(v[7]) << 16);
        reinterpret_cast<uint4 *>(out)[i] = packed;
    }
}

__device__ __forceinline__ float load_value(const float *row, int64_t k) { return row[k]; }
__device__ __forceinline__ float load_value(const uint16_t *row, int64_t k) {
    return __uint_as_float(static_cast<uint32_t>(row[k]) << 16);  // bf16 bits
}

// Row scale rsqrt(mean(x^2) + eps) of rms (model.py:50-51), by one 256-thread CTA.
template <typename T>
__device__ __forceinline__ float rms_scale(const T *row, int64_t cols, float eps, float *part) {
    float ss = 0.0f;
    for (int64_t k = threadIdx.x; k < cols; k += blockDim.x) {
        const float v = load_value(row, k);
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) total += part[w];
    return rsqrtf(total / static_cast<float>(cols) + eps);
}

// Pack the 4 columns k0 .. k0 + 3 of one token row into both X16 planes (from bf16
// rows without a weight the lo plane is zero: hi holds the value exactly).
template <typename T>
__device__ __forceinline__ void pack_four(const T *row, int64_t k0, int64_t cols, float scale,
                                          const float *weight, float *normed_row, int token, int64_t nkt,
                                          int64_t ntb, uint32_t *out, bool &bad) {
    float y[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int64_t k = k0 + j;
        y[j] = 0.0f;
        if (k < cols) {
            y[j] = load_value(row, k);
            if (weight) y[j] = y[j] * scale * weight[k];
            bad |= !isfinite(y[j]);
            if (normed_row) normed_row[k] = y[j];
        }
    }
    const int nt = token >> 3, g = token & 7;
    const int64_t kt = k0 >> 4;
    const int kk = static_cast<int>(k0 & 15);  // multiple of 4: pairs (kk, kk+1), (kk+2, kk+3)
    const int half = kk >> 3;
#pragma unroll
    for (int pr = 0; pr < 2; ++pr) {
        const int t = ((kk & 7) >> 1) + pr;
        const __nv_bfloat16 h0 = __float2bfloat16_rn(y[2 * pr]), h1 = __float2bfloat16_rn(y[2 * pr + 1]);
        const __nv_bfloat16 l0 = __float2bfloat16_rn(y[2 * pr] - __bfloat162float(h0));
        const __nv_bfloat16 l1 = __float2bfloat16_rn(y[2 * pr + 1] - __bfloat162float(h1));
        const int64_t off = ((nt * nkt + kt) * 32 + g * 4 + t) * 2 + half;  // in 32-bit words
        out[off] = __bfloat16_as_ushort(h0) | (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16);
        out[ntb * nkt * 32 * 2 + off] =
            __bfloat16_as_ushort(l0) | (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16);
    }
}

// X16 activation fragments (hi/lo bf16 planes) of rows of x, optionally
// rms-normalised first: y = x * rsqrt(mean(x^2) + eps) * weight (model.py:50-51).
// Grid (tokens, column slices of 1024): each thread packs 4 consecutive columns
// (two bf16 pairs per plane); columns >= cols are written as zeros.  With a
// weight every CTA recomputes its row's rms scale (the row is L2-resident).
template <typename T>
__global__ void __launch_bounds__(256) pack_x16_kernel(const T *__restrict__ x, int64_t cols, int64_t ldx,
                                                       int64_t nkt, int64_t ntb, const float *__restrict__ weight,
                                                       float eps, uint32_t *__restrict__ out, float *normed,
                                                       int64_t ld_normed, int32_t *flags) {
    __shared__ float part[8];
    grid_wait();
    grid_launch_dependents();
    const int token = blockIdx.x;
    const T *row = x + token * ldx;
    const float scale = weight ? rms_scale(row, cols, eps, part) : 1.0f;
    const int64_t k0 = static_cast<int64_t>(blockIdx.y) * 1024 + 4 * threadIdx.x;
    bool bad = false;
    if (k0 < nkt * 16)
        pack_four(row, k0, cols, scale, weight, normed ? normed + token * ld_normed : nullptr, token, nkt, ntb, out,
                  bad);
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_NONFINITE_STATE);
}

// Decode argmax keys into token ids and reset the keys for the next use.
__global__ void argmax_finish_kernel(unsigned long long *keys, int n, int32_t *out) {
    grid_wait();
    grid_launch_dependents();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const unsigned long long k = keys[i];
        out[i] = k ? static_cast<int32_t>(~static_cast<uint32_t>(k & 0xffffffffull)) : -1;
        keys[i] = 0ull;
    }
}

template <int NT, int RB, int W>
static int launch_gemv_t(const GemvArgs &a, cudaStream_t stream) {
    const int64_t nrb = (a.rows + 15) / 16;
    const unsigned grid = static_cast<unsigned>((nrb + RB - 1) / RB);
    return launch_pdl(gemv_kernel<NT, RB, W>, dim3(grid, a.splits), dim3(W * 32), 0, stream, a);
}

// Launch plan (measured on the drafter's shapes, 16 tokens, each GEMV behind its
// activation pack in a CUDA graph).  Every warp's chain of dependent register
// stages is what bounds these small, latency-bound products:
//  - vocabulary-sized heads (>= 8 row blocks per SM): two row blocks per 8-warp
//    CTA, so one K tile of activations serves both;
//  - >= 2 row blocks per SM (the q|k|v projection): the same, one wave;
//  - long rows (K >= 8192, the context fusion): one row block per 4-warp CTA and
//    K split over CTAs to fill every resident slot (shorter chains per warp);
//    the partial sums meet in the workspace;
//  - otherwise one row block per 8-warp CTA over whole rows.
// The workspace starts with a fixed block of counters (one per row group of a
// split matrix; zero on entry, left zero) followed by scratch for the partial
// sums, so one workspace serves calls of any shape in any order.
constexpr int64_t kGemvCounters = 4096;
constexpr size_t kGemvCounterBytes = kGemvCounters * sizeof(int32_t);

struct GemvPlan {
    int rb, warps, splits;
    int64_t groups;
};

template <int NT, int RB, int W>
static int gemv_occupancy_t() {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gemv_kernel<NT, RB, W>, W * 32, 0) != cudaSuccess || n < 1)
        n = 1;
    return n;
}

static int gemv_occupancy(int nt) {  // 4-warp, one-row-block CTAs resident per SM
    static int cache[5] = {};
    int &c = cache[nt];
    if (!c) {
        switch (nt) {
            case 1: c = gemv_occupancy_t<1, 1, 4>(); break;
            case 2: c = gemv_occupancy_t<2, 1, 4>(); break;
            case 3: c = gemv_occupancy_t<3, 1, 4>(); break;
            default: c = gemv_occupancy_t<4, 1, 4>(); break;
        }
    }
    return c;
}

static GemvPlan gemv_plan(int tokens, int64_t rows, int64_t cols, int sms) {
    const int nt = (tokens + 7) / 8;
    const int64_t nrb = (rows + 15) / 16, nkt = (cols + 15) / 16;
    GemvPlan p{};
    p.warps = 8;
    p.splits = 1;
    p.rb = nrb >= 2 * static_cast<int64_t>(sms) ? 2 : 1;
    p.groups = (nrb + p.rb - 1) / p.rb;
    if (p.rb == 1 && nkt >= 512 && p.groups <= kGemvCounters) {
        p.warps = 4;
        int64_t s = static_cast<int64_t>(gemv_occupancy(nt)) * sms / p.groups;
        const int64_t cap = nkt / (p.warps * kGemvUnroll);  // at least one full stage per warp
        if (s > cap) s = cap;
        p.splits = static_cast<int>(s < 1 ? 1 : s);
    }
    return p;
}

static int64_t gemv_cells(int tokens, const GemvPlan &p) { return static_cast<int64_t>(p.rb) * ((tokens + 7) / 8) * 4 * 32; }

static size_t gemv_counter_bytes(const GemvPlan &) { return kGemvCounterBytes; }

size_t gemv_workspace_bytes(int tokens, int64_t rows, int64_t cols, int sms) {
    const GemvPlan p = gemv_plan(tokens, rows, cols, sms);
    if (p.splits <= 1) return 0;
    return gemv_counter_bytes(p) +
           static_cast<size_t>(p.splits) * static_cast<size_t>(p.groups * gemv_cells(tokens, p)) * sizeof(float);
}

int launch_gemv(const GemvArgs &a, int rb, int warps, cudaStream_t stream) {
    const int nt = (a.tokens + 7) / 8;
    if (a.tokens < 1 || a.tokens > 32 || nt > a.ntb) return BD_ERR_INVALID;
    if (warps == 8 && rb == 1) {
        switch (nt) {
            case 1: return launch_gemv_t<1, 1, 8>(a, stream);
            case 2: return launch_gemv_t<2, 1, 8>(a, stream);
            case 3: return launch_gemv_t<3, 1, 8>(a, stream);
            default: return launch_gemv_t<4, 1, 8>(a, stream);
        }
    }
    if (warps == 8) {
        switch (nt) {
            case 1: return launch_gemv_t<1, 2, 8>(a, stream);
            case 2: return launch_gemv_t<2, 2, 8>(a, stream);
            case 3: return launch_gemv_t<3, 2, 8>(a, stream);
            default: return launch_gemv_t<4, 2, 8>(a, stream);
        }
    }
    switch (nt) {  // 4-warp CTAs: one row block, K split (long rows)
        case 1: return launch_gemv_t<1, 1, 4>(a, stream);
        case 2: return launch_gemv_t<2, 1, 4>(a, stream);
        case 3: return launch_gemv_t<3, 1, 4>(a, stream);
        default: return launch_gemv_t<4, 1, 4>(a, stream);
    }
}

}  // namespace bd

using namespace bd;

static int64_t nkt_of(int64_t cols) { return (cols + 15) / 16; }

extern "C" int64_t bd_w16_bytes(int64_t rows, int64_t cols) {
    if (rows < 0 || cols < 0) return -1;
    return (rows + 15) / 16 * nkt_of(cols) * 512;
}

extern "C" int bd_tile_w16(const void *w, int dtype_bits, int64_t rows, int64_t cols, void *out,
                           bd_stream_t stream) {
    if (rows < 1 || cols < 1 || !w || !out || (dtype_bits != 32 && dtype_bits != 16)) return BD_ERR_INVALID;
    const int64_t total = (rows + 15) / 16 * nkt_of(cols) * 32;
    const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, 148 * 32));
    if (dtype_bits == 32)
        tile_w16_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float *>(w), rows, cols, nkt_of(cols),
                                                        static_cast<uint16_t *>(out));
    else
        tile_w16_kernel<uint16_t><<<grid, 256, 0, stream>>>(static_cast<const uint16_t *>(w), rows, cols,
                                                           nkt_of(cols), static_cast<uint16_t *>(out));
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int64_t bd_x16_bytes(int tokens, int64_t cols) {
    if (tokens < 0 || cols < 0) return -1;
    return 2 * static_cast<int64_t>((tokens + 7) / 8) * nkt_of(cols) * 32 * 8;
}

extern "C" int bd_pack_x16(const float *x, int tokens, int64_t cols, int64_t ldx, const float *rms_weight,
                           float epsilon, void *out, float *normed, int64_t ld_normed, int32_t *flags,
                           bd_stream_t stream) {
    if (tokens < 1 || tokens > 32 || cols < 1 || ldx < cols || !x || !out) return BD_ERR_INVALID;
    const unsigned slices = static_cast<unsigned>((nkt_of(cols) * 16 + 1023) / 1024);
    return launch_pdl(pack_x16_kernel<float>, dim3(tokens, slices), dim3(256), 0, stream, x, cols, ldx, nkt_of(cols),
                      static_cast<int64_t>((tokens + 7) / 8), rms_weight, epsilon, static_cast<uint32_t *>(out),
                      normed, ld_normed, flags);
}

extern "C" int bd_pack_x16_bf16(const void *x, int tokens, int64_t cols, int64_t ldx, const float *rms_weight,
                                float epsilon, void *out, float *normed, int64_t ld_normed, int32_t *flags,
                                bd_stream_t stream) {
    if (tokens < 1 || tokens > 32 || cols < 1 || ldx < cols || !x || !out) return BD_ERR_INVALID;
    const unsigned slices = static_cast<unsigned>((nkt_of(cols) * 16 + 1023) / 1024);
    return launch_pdl(pack_x16_kernel<uint16_t>, dim3(tokens, slices), dim3(256), 0, stream,
                      static_cast<const uint16_t *>(x), cols, ldx, nkt_of(cols),
                      static_cast<int64_t>((tokens + 7) / 8), rms_weight, epsilon, static_cast<uint32_t *>(out),
                      normed, ld_normed, flags);
}

static int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0, v = 0;
        n = (cudaGetDevice(&dev) == cudaSuccess &&
             cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
                ? v
                : 148;
    }
    return n;
}

extern "C" size_t bd_gemv_workspace_bytes(int tokens, int64_t rows, int64_t cols) {
    if (tokens < 1 || rows < 1 || cols < 1) return 0;
    return gemv_workspace_bytes(tokens, rows, cols, sm_count());
}

extern "C" int bd_gemv_bf16(const void *w16, int64_t rows, int64_t cols, const void *x16, int tokens, float *out,
                            int64_t ld_out, const float *residual, unsigned long long *argmax_keys, int32_t *flags,
                            void *workspace, size_t workspace_bytes, bd_stream_t stream) {
    if (rows < 1 || cols < 1 || !w16 || !x16 || tokens < 1 || tokens > 32) return BD_ERR_INVALID;
    if (!out && !argmax_keys) return BD_ERR_INVALID;
    if ((out || residual) && ld_out < rows) return BD_ERR_INVALID;
    GemvArgs a{};
    a.splits = 1;
    const GemvPlan plan = gemv_plan(tokens, rows, cols, sm_count());
    const size_t need = gemv_workspace_bytes(tokens, rows, cols, sm_count());
    if (need && workspace && workspace_bytes >= need) {  // without a workspace the K split is skipped
        a.splits = plan.splits;
        a.counters = static_cast<int32_t *>(workspace);
        a.partial = reinterpret_cast<float *>(static_cast<char *>(workspace) + gemv_counter_bytes(plan));
    }
    a.w = static_cast<const uint4 *>(w16);
    a.rows = rows;
    a.cols = cols;
    a.nkt = nkt_of(cols);
    a.x = static_cast<const uint2 *>(x16);
    a.ntb = (tokens + 7) / 8;
    a.tokens = tokens;
    a.out = out;
    a.ld_out = ld_out;
    a.residual = residual;
    a.argmax = argmax_keys;
    a.flags = flags;
    return launch_gemv(a, plan.rb, plan.warps, stream);
}

extern "C" int bd_argmax_finish(unsigned long long *keys, int n, int32_t *out, bd_stream_t stream) {
    if (n < 1 || !keys || !out) return BD_ERR_INVALID;
    return launch_pdl(argmax_finish_kernel, dim3((n + 127) / 128), dim3(128), 0, stream, keys, n, out);
}
