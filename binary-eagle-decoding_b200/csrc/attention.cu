// Block-draft attention over the fp16 K/V cache (Layer.forward, w1a1_eagle/model.py:212-218):
// softmax(q k^T / sqrt(d), masked to |pos_q - pos_k| < window on windowed layers) v
// for up to 16 query slots per q head, grouped-query (q head h uses kv head
// h / (heads / kv_heads)).
//
// Split over keys (flash decoding): CTA (kv head, chunk of 256 keys) stages its
// K and V rows in shared memory with cp.async; warp w owns q head
// kv * groups + (w & 3), its 16 query rows and quarter (w >> 2) of the keys.  S = Q K^T and O = P V run on
// m16n8k16 fp16 MMAs with fp32 accumulation (K fragments by ldmatrix, V by
// ldmatrix.trans, P re-packed from the S accumulators).  The cached K and V are
// fp16 values, exact as MMA operands; the fp32 queries and probabilities are
// split into fp16 hi + lo halves (x = hi + lo to ~22 bits), two MMAs each, so
// the products keep fp32 precision (the reference attends with fp32 queries).  Each CTA writes its
// chunk's row maxima, row sums and un-normalised O; a combine kernel merges the
// chunks.  No waits between CTAs: partials meet only in the combine launch.
#include "kernels.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace bd {

constexpr int kKeys = 256;  // keys per chunk
// Padded fp16 row of a staged K/V row in shared memory (conflict-free ldmatrix).
template <int D>
constexpr int row_bytes() { return D * 2 + 16; }

struct AttnArgs {
    const float *q;         // [tokens][heads][d] fp32
    const __half *k, *v;    // [positions][kv_heads][d] (cache rows 0 .. keys-1)
    int tokens, heads, kv_heads, keys;
    int windowed;           // apply |pos_q - pos_k| < window
    int64_t anchor;         // position of query row 0
    int64_t window;
    int64_t stable_keys;    // keys [0, stable_keys) were not written by the immediately preceding kernel
    float scale;            // 1 / sqrt(d)
    int chunks;
    float *part_o;          // [chunks][heads][16][d]
    float *part_ml;         // [chunks][heads][16][2]
    float *out;             // [tokens][heads * d], or null when x16 is set
    uint16_t *x16;          // X16 fragments of the output rows (the GEMV's activation layout), or null
    int32_t *flags;
};

// 16 warps: warp w takes q head (w & 3) of the kv group and quarter (w >> 2) of
// the chunk's keys; the quarters of a head merge through shared memory (the
// staged K/V area, free once P V is done).  One CTA per SM.
constexpr int kAttnWarps = 16;
constexpr int kKeyParts = kAttnWarps / 4;
constexpr int kPartKeys = kKeys / kKeyParts;  // 64

template <int kDim>
constexpr size_t attn_smem_bytes() {
    // staged K and V rows; the key-part exchange (per head and part 1..3, 4 values
    // per lane for every one of the kDim/8 O fragments plus (m, l) of its two
    // rows) reuses them
    return 2 * static_cast<size_t>(kKeys) * row_bytes<kDim>();
}
static_assert(static_cast<size_t>(4) * (kKeyParts - 1) * (128 / 8 * 4 + 4) * 32 * sizeof(float) <=
                  2 * static_cast<size_t>(kKeys) * row_bytes<128>(),
              "the key-part exchange fits in the staged K/V area");

template <int kDim>
__global__ void __launch_bounds__(kAttnWarps * 32, 1) attn_chunk_kernel(const AttnArgs a) {
    constexpr int kRowBytes = row_bytes<kDim>();
    constexpr int kX = kDim / 8 * 4 + 4;  // exchanged floats per lane
    extern __shared__ __align__(16) char sm[];
    char *ks = sm;
    char *vs = sm + kKeys * kRowBytes;
    float *xch = reinterpret_cast<float *>(sm);  // [part - 1][head][kX][32], after P V
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int hw = warp & 3, kh = warp >> 2;  // head of the group, key part
    const int kvh = blockIdx.x, chunk = blockIdx.y;
    const int groups = a.heads / a.kv_heads;
    const int key0 = chunk * kKeys;
    const int nkeys = min(kKeys, a.keys - key0);
    // stage K and V rows of this chunk (rows past the end are zero); a chunk of
    // context keys the preceding kernel did not write starts loading before the
    // dependency wait, so the cache stream overlaps that kernel
    auto stage = [&]() {
        for (int i = threadIdx.x; i < kKeys * (kDim / 8); i += blockDim.x) {
            const int r = i / (kDim / 8), c = i % (kDim / 8);
            const bool live = r < nkeys;
            const int64_t src = (static_cast<int64_t>(key0 + (live ? r : 0)) * a.kv_heads + kvh) * kDim + c * 8;
            cp_async16(ks + r * kRowBytes + c * 16, a.k + src, live ? 16 : 0);
            cp_async16(vs + r * kRowBytes + c * 16, a.v + src, live ? 16 : 0);
        }
    };
    const bool early = static_cast<int64_t>(key0) + kKeys <= a.stable_keys;
    if (early) stage();
    grid_wait();
    grid_launch_dependents();
    if (!early) stage();
    // Q fragments of this warp's head: rows are query slots (A operand, row-major 16 x kDim)
    const int head = kvh * groups + hw;
    const bool head_live = hw < groups;
    uint32_t qa[kDim / 16][4], ql[kDim / 16][4];
#pragma unroll
    for (int s = 0; s < kDim / 16; ++s) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int row = g + 8 * (j & 1);
            const int col = s * 16 + 2 * t + 8 * (j >> 1);
            float2 x = make_float2(0.0f, 0.0f);
            if (head_live && row < a.tokens)
                x = *reinterpret_cast<const float2 *>(a.q + (static_cast<int64_t>(row) * a.heads + head) * kDim + col);
            split_half2(x.x, x.y, qa[s][j], ql[s][j]);
        }
    }
    cp_async_wait_all();
    __syncthreads();

    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
    float o_acc[kDim / 8][4];
#pragma unroll
    for (int n = 0; n < kDim / 8; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) o_acc[n][i] = 0.0f;
    // a key part with no live key (the short last chunk) keeps m = -inf, l = 0, O = 0:
    // exactly what its masked products would give, without the MMAs
    const int kbase = kh * kPartKeys;
    if (head_live && kbase < nkeys) {
        // S = Q K^T over this warp's 64 keys: 8 n-tiles of 8 keys
        float s_acc[kPartKeys / 8][4];
#pragma unroll
        for (int n = 0; n < kPartKeys / 8; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) s_acc[n][i] = 0.0f;
#pragma unroll
        for (int s2 = 0; s2 < kDim / 32; ++s2) {
#pragma unroll
            for (int n = 0; n < kPartKeys / 8; ++n) {
                // x4: matrices (d 0-7, 8-15) of k-step 2*s2 and (d 0-7, 8-15) of k-step 2*s2+1 for 8 keys
                uint32_t b[4];
                const int mi = lane >> 3, r = lane & 7;
                ldmatrix_x4(b, ks + (kbase + n * 8 + r) * kRowBytes + (s2 * 32 + mi * 8) * 2);
                mma_f16_16816(s_acc[n], qa[2 * s2][0], qa[2 * s2][1], qa[2 * s2][2], qa[2 * s2][3], b[0], b[1]);
                mma_f16_16816(s_acc[n], ql[2 * s2][0], ql[2 * s2][1], ql[2 * s2][2], ql[2 * s2][3], b[0], b[1]);
                mma_f16_16816(s_acc[n], qa[2 * s2 + 1][0], qa[2 * s2 + 1][1], qa[2 * s2 + 1][2], qa[2 * s2 + 1][3],
                              b[2], b[3]);
                mma_f16_16816(s_acc[n], ql[2 * s2 + 1][0], ql[2 * s2 + 1][1], ql[2 * s2 + 1][2], ql[2 * s2 + 1][3],
                              b[2], b[3]);
            }
        }
        // scale, mask, row maxima (rows g and g + 8 of this lane)
        const int kq0 = key0 + kbase + 2 * t;
#pragma unroll
        for (int n = 0; n < kPartKeys / 8; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int row = g + 8 * (i >> 1);
                const int key = kq0 + n * 8 + (i & 1);
                bool ok = key < a.keys && row < a.tokens;
                if (a.windowed) {
                    const int64_t dist = a.anchor + row - key;
                    ok = ok && (dist < a.window && -dist < a.window);
                }
                const float v = ok ? s_acc[n][i] * a.scale : -INFINITY;
                s_acc[n][i] = v;
                m[i >> 1] = fmaxf(m[i >> 1], v);
            }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            m[r] = fmaxf(m[r], __shfl_xor_sync(0xffffffffu, m[r], 1));
            m[r] = fmaxf(m[r], __shfl_xor_sync(0xffffffffu, m[r], 2));
        }
#pragma unroll
        for (int n = 0; n < kPartKeys / 8; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float mm = m[i >> 1];
                const float p = mm == -INFINITY ? 0.0f : __expf(s_acc[n][i] - mm);
                s_acc[n][i] = p;
                l[i >> 1] += p;
            }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            l[r] += __shfl_xor_sync(0xffffffffu, l[r], 1);
            l[r] += __shfl_xor_sync(0xffffffffu, l[r], 2);
        }
        // O = P V over the 64 keys: P re-packed from the S accumulators as A fragments
#pragma unroll
        for (int kk = 0; kk < kPartKeys / 16; ++kk) {
            uint32_t pa0, pa1, pa2, pa3, pl0, pl1, pl2, pl3;
            split_half2(s_acc[2 * kk][0], s_acc[2 * kk][1], pa0, pl0);
            split_half2(s_acc[2 * kk][2], s_acc[2 * kk][3], pa1, pl1);
            split_half2(s_acc[2 * kk + 1][0], s_acc[2 * kk + 1][1], pa2, pl2);
            split_half2(s_acc[2 * kk + 1][2], s_acc[2 * kk + 1][3], pa3, pl3);
#pragma unroll
            for (int n2 = 0; n2 < kDim / 16; ++n2) {
                uint32_t b[4];
                const int mi = lane >> 3, r = lane & 7;
                ldmatrix_x4_trans(b, vs + (kbase + kk * 16 + (mi & 1) * 8 + r) * kRowBytes + (n2 * 16 + (mi >> 1) * 8) * 2);
                mma_f16_16816(o_acc[2 * n2], pa0, pa1, pa2, pa3, b[0], b[1]);
                mma_f16_16816(o_acc[2 * n2], pl0, pl1, pl2, pl3, b[0], b[1]);
                mma_f16_16816(o_acc[2 * n2 + 1], pa0, pa1, pa2, pa3, b[2], b[3]);
                mma_f16_16816(o_acc[2 * n2 + 1], pl0, pl1, pl2, pl3, b[2], b[3]);
            }
        }
    }
    // key parts 1..3 hand their state to part 0 through shared memory (the staged
    // K/V area: every warp has finished P V at the barrier)
    __syncthreads();
    if (head_live && kh > 0) {
        float *x = xch + ((kh - 1) * 4 + hw) * kX * 32 + lane;
#pragma unroll
        for (int n = 0; n < kDim / 8; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) x[(n * 4 + i) * 32] = o_acc[n][i];
        x[(kX - 4) * 32] = m[0];
        x[(kX - 3) * 32] = m[1];
        x[(kX - 2) * 32] = l[0];
        x[(kX - 1) * 32] = l[1];
    }
    __syncthreads();
    if (!head_live || kh > 0) return;
    for (int part = 1; part < kKeyParts; ++part) {  // fixed order
        const float *x = xch + ((part - 1) * 4 + hw) * kX * 32 + lane;
        float f0[2], f1[2];
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const float m1 = x[(kX - 4 + r) * 32], l1 = x[(kX - 2 + r) * 32];
            const float mx = fmaxf(m[r], m1);
            f0[r] = mx == -INFINITY ? 0.0f : __expf(m[r] - mx);
            f1[r] = mx == -INFINITY ? 0.0f : __expf(m1 - mx);
            l[r] = l[r] * f0[r] + l1 * f1[r];
            m[r] = mx;
        }
#pragma unroll
        for (int n = 0; n < kDim / 8; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) o_acc[n][i] = o_acc[n][i] * f0[i >> 1] + x[(n * 4 + i) * 32] * f1[i >> 1];
    }
    // partials: un-normalised O, row max and row sum of this chunk
    float *po = a.part_o + ((static_cast<int64_t>(chunk) * a.heads + head) * 16) * kDim;
#pragma unroll
    for (int n = 0; n < kDim / 8; ++n) {
        *reinterpret_cast<float2 *>(po + g * kDim + n * 8 + 2 * t) = make_float2(o_acc[n][0], o_acc[n][1]);
        *reinterpret_cast<float2 *>(po + (g + 8) * kDim + n * 8 + 2 * t) = make_float2(o_acc[n][2], o_acc[n][3]);
    }
    if (t == 0) {
        float *pml = a.part_ml + ((static_cast<int64_t>(chunk) * a.heads + head) * 16) * 2;
        pml[g * 2] = m[0];
        pml[g * 2 + 1] = l[0];
        pml[(g + 8) * 2] = m[1];
        pml[(g + 8) * 2 + 1] = l[1];
    }
}

// out[token][head * d + j] = sum_c e^{m_c - M} O_c / sum_c e^{m_c - M} l_c.
// Grid (tokens, heads), d threads: chunk weights are computed once into shared
// memory, then every thread sums its column over the chunks with independent loads.
constexpr int kMaxChunks = 1024;
constexpr int kCombineBatch = 20;  // chunk partials per thread requested at once

template <int kDim>
__global__ void __launch_bounds__(kDim) attn_combine_kernel(const AttnArgs a) {
    __shared__ float wgt[kMaxChunks];
    __shared__ float red[kDim / 32];
    __shared__ float s_max, s_den;
    grid_wait();
    grid_launch_dependents();
    const int token = blockIdx.x, head = blockIdx.y, j = threadIdx.x;
    const int lane = j & 31, warp = j >> 5;
    // the first kCombineBatch chunks' O values are requested with the chunk maxima
    // and sums, so the combine costs about one L2 round trip
    const float *po = a.part_o + (static_cast<int64_t>(head) * 16 + token) * kDim + j;
    const int64_t stride = static_cast<int64_t>(a.heads) * 16 * kDim;
    float ov[kCombineBatch];
#pragma unroll
    for (int c = 0; c < kCombineBatch; ++c) ov[c] = c < a.chunks ? po[c * stride] : 0.0f;
    float mloc = -INFINITY;
    for (int c = j; c < a.chunks; c += kDim) {
        const float mc = a.part_ml[((static_cast<int64_t>(c) * a.heads + head) * 16 + token) * 2];
        wgt[c] = mc;
        mloc = fmaxf(mloc, mc);
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) mloc = fmaxf(mloc, __shfl_xor_sync(0xffffffffu, mloc, d));
    if (lane == 0) red[warp] = mloc;
    __syncthreads();
    if (j == 0) {
        float M = red[0];
#pragma unroll
        for (int w = 1; w < kDim / 32; ++w) M = fmaxf(M, red[w]);
        s_max = M;
    }
    __syncthreads();
    const float M = s_max;
    float dloc = 0.0f;
    for (int c = j; c < a.chunks; c += kDim) {
        const int64_t base = (static_cast<int64_t>(c) * a.heads + head) * 16 + token;
        const float mc = wgt[c];
        const float w = mc == -INFINITY ? 0.0f : __expf(mc - M);
        wgt[c] = w;
        dloc += w * a.part_ml[base * 2 + 1];
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) dloc += __shfl_xor_sync(0xffffffffu, dloc, d);
    __syncthreads();  // red is reused; wgt is complete
    if (lane == 0) red[warp] = dloc;
    __syncthreads();
    if (j == 0) {
        float den = 0.0f;
        for (int w = 0; w < kDim / 32; ++w) den += red[w];
        s_den = den;
    }
    __syncthreads();
    float num = 0.0f;
#pragma unroll
    for (int c = 0; c < kCombineBatch; ++c)
        if (c < a.chunks) num += wgt[c] * ov[c];
#pragma unroll 8
    for (int c = kCombineBatch; c < a.chunks; ++c) num += wgt[c] * po[c * stride];
    const float y = num / s_den;
    if (a.out) a.out[static_cast<int64_t>(token) * a.heads * kDim + head * kDim + j] = y;
    if (a.x16) {
        // the element's slot in both bf16 planes of the X16 layout (as bd_pack_x16 writes it)
        const int64_t cols = static_cast<int64_t>(a.heads) * kDim, nkt = cols / 16;
        const int64_t ntb = (a.tokens + 7) / 8;
        const int64_t col = static_cast<int64_t>(head) * kDim + j;
        const int kk = static_cast<int>(col & 15);
        const int64_t word = (((token >> 3) * nkt + (col >> 4)) * 32 + (token & 7) * 4 + ((kk & 7) >> 1)) * 2 + (kk >> 3);
        const int64_t slot = word * 2 + (kk & 1);
        const __nv_bfloat16 hi = __float2bfloat16_rn(y);
        const __nv_bfloat16 lo = __float2bfloat16_rn(y - __bfloat162float(hi));
        a.x16[slot] = __bfloat16_as_ushort(hi);
        a.x16[ntb * nkt * 32 * 4 + slot] = __bfloat16_as_ushort(lo);
        if (!isfinite(y)) set_flag(a.flags, BD_FLAG_NONFINITE_STATE);
    }
}

}  // namespace bd

using namespace bd;

extern "C" size_t bd_attention_workspace_bytes(int heads, int head_dim, int keys) {
    const int chunks = (keys + kKeys - 1) / kKeys;
    return static_cast<size_t>(chunks) * heads * 16 * (head_dim + 2) * sizeof(float) + 256;
}

template <int D>
static int launch_attention(const AttnArgs &a, int kv_heads, int tokens, int heads, cudaStream_t stream) {
    const size_t smem = attn_smem_bytes<D>();
    if (cudaFuncSetAttribute(attn_chunk_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
        return BD_ERR_LAUNCH;
    int st = launch_pdl(attn_chunk_kernel<D>, dim3(kv_heads, a.chunks), dim3(kAttnWarps * 32), smem, stream, a);
    if (st) return st;
    return launch_pdl(attn_combine_kernel<D>, dim3(tokens, heads), dim3(D), 0, stream, a);
}

static int attention_decode(const float *q, const uint16_t *k_cache, const uint16_t *v_cache, int tokens, int heads,
                            int kv_heads, int head_dim, int keys, int windowed, int64_t anchor, int64_t window,
                            int64_t stable_keys, float *out, void *x16, int32_t *flags, void *workspace,
                            size_t workspace_bytes, bd_stream_t stream) {
    if (tokens < 1 || tokens > 16 || (head_dim != 64 && head_dim != 128) || heads < 1 || kv_heads < 1 ||
        heads % kv_heads ||
        heads / kv_heads > 4 || keys < 1 || keys > kMaxChunks * kKeys || !q || !k_cache || !v_cache || (!out && !x16))
        return BD_ERR_INVALID;
    if (!workspace || workspace_bytes < bd_attention_workspace_bytes(heads, head_dim, keys)) return BD_ERR_WORKSPACE;
    AttnArgs a{};
    a.q = q;
    a.k = reinterpret_cast<const __half *>(k_cache);
    a.v = reinterpret_cast<const __half *>(v_cache);
    a.tokens = tokens;
    a.heads = heads;
    a.kv_heads = kv_heads;
    a.keys = keys;
    a.windowed = windowed;
    a.anchor = anchor;
    a.window = window;
    a.stable_keys = stable_keys < 0 ? 0 : stable_keys;
    a.scale = 1.0f / sqrtf(static_cast<float>(head_dim));
    a.chunks = (keys + kKeys - 1) / kKeys;
    a.part_ml = static_cast<float *>(workspace);
    a.part_o = a.part_ml + static_cast<size_t>(a.chunks) * heads * 16 * 2;
    a.out = out;
    a.x16 = static_cast<uint16_t *>(x16);
    a.flags = flags;
    return head_dim == 64 ? launch_attention<64>(a, kv_heads, tokens, heads, stream)
                          : launch_attention<128>(a, kv_heads, tokens, heads, stream);
}

extern "C" int bd_attention_decode(const float *q, const uint16_t *k_cache, const uint16_t *v_cache, int tokens,
                                   int heads, int kv_heads, int head_dim, int keys, int windowed, int64_t anchor,
                                   int64_t window, int64_t stable_keys, float *out, void *workspace,
                                   size_t workspace_bytes, bd_stream_t stream) {
    if (!out) return BD_ERR_INVALID;
    return attention_decode(q, k_cache, v_cache, tokens, heads, kv_heads, head_dim, keys, windowed, anchor, window,
                            stable_keys, out, nullptr, nullptr, workspace, workspace_bytes, stream);
}

extern "C" int bd_attention_decode_x16(const float *q, const uint16_t *k_cache, const uint16_t *v_cache, int tokens,
                                       int heads, int kv_heads, int head_dim, int keys, int windowed, int64_t anchor,
                                       int64_t window, int64_t stable_keys, void *x16, int32_t *flags,
                                       void *workspace, size_t workspace_bytes, bd_stream_t stream) {
    if (!x16) return BD_ERR_INVALID;
    return attention_decode(q, k_cache, v_cache, tokens, heads, kv_heads, head_dim, keys, windowed, anchor, window,
                            stable_keys, nullptr, x16, flags, workspace, workspace_bytes, stream);
}
