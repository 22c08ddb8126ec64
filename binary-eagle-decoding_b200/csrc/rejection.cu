// Temperature-1 speculative rejection sampling over vocabulary-sized bf16 rows.
//
// The reference has no implementation of its own (it runs llama.cpp's sampler;
// the only in-tree pin is the statistical check of native/verifier-test.cpp:43-80
// and the EOG break of benchmarks/native.py:19-38), so this file implements a
// deterministic contract that a CPU restatement reproduces bit for bit:
//   * uniforms: Philox4x32-10 (Salmon et al., SC'11), key = the 64-bit seed,
//     counter = (request, position, purpose, offset), u = (x0 >> 8) * 2^-24;
//   * e(x), x <= 0: x clamped at -86.5; k = rint(x log2 e) and f = x log2 e - k
//     each with one fused rounding; 2^f by a degree-5 polynomial with a unit
//     constant term (Horner in fused multiply-adds); p 2^k formed exactly by
//     adding k to the exponent bits;
//   * rows are cut into chunks of 16384 entries = 256 lanes x 8 vectors x 8
//     items (entry 8 (t + 256 j) + e is item e of vector j of lane t); a chunk
//     sum adds each lane's items over j sequentially, combines the 8 item sums
//     by a balanced tree and the 256 lane sums by a balanced tree of adjacent
//     pairs;
//   * softmax of a row: chunk c keeps m_c = its max and s_c = sum e(l - m_c);
//     m = max m_c and S = tree over 32 slots of s_c e(m_c - m); p(j) =
//     e(l_j - m) * rcp(S) with a correctly rounded reciprocal;
//   * accept draft d at position i iff u q(d) < p(d); an accepted EOG that is
//     not the last draft ends the round; on rejection sample from
//     max(0, p - q) (from p when that is zero everywhere), after all drafts
//     from e(l - m) of the bonus row, by an inverse-CDF search: chunk by the
//     sequential prefix of chunk sums, lane by a Hillis-Steele scan of the
//     chunk's lane sums, item by the lane's sequential prefix.
//
// Kernel 1 (one CTA per row chunk, all rows) reads every logit once and writes
// (m_c, s_c).  Kernel 2 (one CTA per request chunk) combines the row statistics,
// walks the drafts, sums its chunk of the sampling weights, and the last CTA of
// each request to finish (a counter, no waiting) picks the token.
#include "kernels.cuh"

namespace bd {

constexpr int kLanes = 256;
constexpr int kVectors = 8;
constexpr int kItems = 8;
constexpr int kChunk = kLanes * kVectors * kItems;  // 16384
constexpr int kMaxChunks = 32;
constexpr uint32_t kPadBits = 0xFF7FFF7Fu;  // two lowest finite bf16 values (padding of ragged chunks)

// ---------------------------------------------------------------- deterministic exp
__device__ __forceinline__ float ucf(uint32_t b) { return __uint_as_float(b); }

#define BD_EXP_FLOOR (-86.5f)
#define BD_LOG2E_BITS 0x3FB8AA3Bu
#define BD_MAGIC 12582912.0f  // 1.5 * 2^23

// Two lanes of e(x) in packed fp32x2 arithmetic (each lane rounds as the scalar form).
__device__ __forceinline__ float2 exp_pair(float2 x) {
    x.x = fmaxf(x.x, BD_EXP_FLOOR);
    x.y = fmaxf(x.y, BD_EXP_FLOOR);
    const float l2e = ucf(BD_LOG2E_BITS);
    const float2 l2 = make_float2(l2e, l2e);
    const float2 tm = __ffma2_rn(x, l2, make_float2(BD_MAGIC, BD_MAGIC));
    const float2 kf = __fadd2_rn(tm, make_float2(-BD_MAGIC, -BD_MAGIC));
    const float2 f = __ffma2_rn(x, l2, make_float2(-kf.x, -kf.y));
    float2 p = make_float2(ucf(0x3AAF6433u), ucf(0x3AAF6433u));
    p = __ffma2_rn(p, f, make_float2(ucf(0x3C1E5FB0u), ucf(0x3C1E5FB0u)));
    p = __ffma2_rn(p, f, make_float2(ucf(0x3D6357F7u), ucf(0x3D6357F7u)));
    p = __ffma2_rn(p, f, make_float2(ucf(0x3E75FD26u), ucf(0x3E75FD26u)));
    p = __ffma2_rn(p, f, make_float2(ucf(0x3F317218u), ucf(0x3F317218u)));
    p = __ffma2_rn(p, f, make_float2(1.0f, 1.0f));
    return make_float2(ucf(__float_as_uint(p.x) + (__float_as_uint(tm.x) << 23)),
                       ucf(__float_as_uint(p.y) + (__float_as_uint(tm.y) << 23)));
}

__device__ __forceinline__ float exp_one(float x) {
    x = fmaxf(x, BD_EXP_FLOOR);
    const float l2e = ucf(BD_LOG2E_BITS);
    const float tm = __fmaf_rn(x, l2e, BD_MAGIC);
    const float kf = __fadd_rn(tm, -BD_MAGIC);
    const float f = __fmaf_rn(x, l2e, -kf);
    float p = ucf(0x3AAF6433u);
    p = __fmaf_rn(p, f, ucf(0x3C1E5FB0u));
    p = __fmaf_rn(p, f, ucf(0x3D6357F7u));
    p = __fmaf_rn(p, f, ucf(0x3E75FD26u));
    p = __fmaf_rn(p, f, ucf(0x3F317218u));
    p = __fmaf_rn(p, f, 1.0f);
    return ucf(__float_as_uint(p) + (__float_as_uint(tm) << 23));
}

// ---------------------------------------------------------------- Philox4x32-10
__device__ __forceinline__ uint4 philox(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int i = 0; i < 10; ++i) {
        const uint32_t lo0 = 0xD2511F53u * c.x, hi0 = __umulhi(0xD2511F53u, c.x);
        const uint32_t lo1 = 0xCD9E8D57u * c.z, hi1 = __umulhi(0xCD9E8D57u, c.z);
        c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
    return c;
}

__device__ __forceinline__ float uniform01(unsigned long long seed, uint32_t request, uint32_t position,
                                           uint32_t purpose, uint32_t offset) {
    const uint4 r = philox(make_uint4(request, position, purpose, offset), static_cast<uint32_t>(seed),
                           static_cast<uint32_t>(seed >> 32));
    return __fmul_rn(static_cast<float>(r.x >> 8), ucf(0x33800000u));  // 2^-24
}

__device__ __forceinline__ float lo_f(uint32_t w) { return ucf(w << 16); }
__device__ __forceinline__ float hi_f(uint32_t w) { return ucf(w & 0xFFFF0000u); }

struct RejArgs {
    const uint16_t *target;   // [B][n+1][V]
    const uint16_t *draft;    // [B][n][V]
    const int32_t *drafts;    // [B][n]
    const int32_t *eog;
    int n_eog;
    int requests, n, chunks;
    int64_t vocab;
    unsigned long long seed;
    uint32_t offset;
    float2 *stats;      // [rows][chunks]: (m_c, s_c)
    float2 *parts;      // [requests][chunks]: (residual or bonus sum, p sum)
    float2 *lanes;      // [requests][chunks][256]: the same per lane
    int32_t *counter;   // [requests]
    int32_t *accepted, *next_token;
    int32_t *flags;
};

__device__ __forceinline__ const uint16_t *target_row(const RejArgs &a, int64_t b, int64_t i) {
    return a.target + (b * (a.n + 1) + i) * a.vocab;
}
__device__ __forceinline__ const uint16_t *draft_row(const RejArgs &a, int64_t b, int64_t i) {
    return a.draft + (b * a.n + i) * a.vocab;
}
// stats row index: target rows first (b (n+1) + i), then draft rows
__device__ __forceinline__ int64_t target_stat(const RejArgs &a, int64_t b, int64_t i) { return b * (a.n + 1) + i; }
__device__ __forceinline__ int64_t draft_stat(const RejArgs &a, int64_t b, int64_t i) {
    return static_cast<int64_t>(a.requests) * (a.n + 1) + b * a.n + i;
}

template <bool VEC>
__device__ __forceinline__ uint4 load_vector(const uint16_t *row, int64_t e0, int64_t vocab) {
    if (VEC) return e0 < vocab ? ld_stream_u4(row + e0) : make_uint4(kPadBits, kPadBits, kPadBits, kPadBits);
    uint32_t h[kItems];
#pragma unroll
    for (int e = 0; e < kItems; ++e) h[e] = e0 + e < vocab ? row[e0 + e] : 0xFF7Fu;
    return make_uint4(h[0] | (h[1] << 16), h[2] | (h[3] << 16), h[4] | (h[5] << 16), h[6] | (h[7] << 16));
}

// Lane t's 8 vectors of chunk c (entries 8 (t + 256 j) + e); entries past the
// vocabulary read as the lowest finite bf16.  VEC: rows are 16-byte aligned and
// vocab % 8 == 0, so a vector is wholly inside or outside the row.
template <bool VEC>
__device__ __forceinline__ void load_chunk(const uint16_t *row, int64_t c0, int64_t vocab, uint4 (&w)[kVectors]) {
#pragma unroll
    for (int j = 0; j < kVectors; ++j) w[j] = load_vector<VEC>(row, c0 + kItems * (threadIdx.x + kLanes * j), vocab);
}

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// Balanced adjacent-pair tree over the CTA's 256 lane values; every thread gets the total.
__device__ __forceinline__ float cta_tree(float v, float *scratch) {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, d));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = v;
    __syncthreads();
    const float w01 = __fadd_rn(scratch[0], scratch[1]), w23 = __fadd_rn(scratch[2], scratch[3]);
    const float w45 = __fadd_rn(scratch[4], scratch[5]), w67 = __fadd_rn(scratch[6], scratch[7]);
    return __fadd_rn(__fadd_rn(w01, w23), __fadd_rn(w45, w67));
}

__device__ __forceinline__ float item_tree(const float2 (&s)[4]) {
    return __fadd_rn(__fadd_rn(__fadd_rn(s[0].x, s[0].y), __fadd_rn(s[1].x, s[1].y)),
                     __fadd_rn(__fadd_rn(s[2].x, s[2].y), __fadd_rn(s[3].x, s[3].y)));
}

// ---------------------------------------------------------------- kernel 1: chunk statistics
// e(x) without the clamp: equal to exp_pair whenever every x >= -86.5.
__device__ __forceinline__ float2 exp_pair_unclamped(float2 x) {
    const float l2e = ucf(BD_LOG2E_BITS);
    const float2 l2 = make_float2(l2e, l2e);
    const float2 tm = __ffma2_rn(x, l2, make_float2(BD_MAGIC, BD_MAGIC));
    const float2 kf = __fadd2_rn(tm, make_float2(-BD_MAGIC, -BD_MAGIC));
    const float2 f = __ffma2_rn(x, l2, make_float2(-kf.x, -kf.y));
    float2 p = make_float2(ucf(0x3AAF6433u), ucf(0x3AAF6433u));
    p = __ffma2_rn(p, f, make_float2(ucf(0x3C1E5FB0u), ucf(0x3C1E5FB0u)));
    p = __ffma2_rn(p, f, make_float2(ucf(0x3D6357F7u), ucf(0x3D6357F7u)));
    p = __ffma2_rn(p, f, make_float2(ucf(0x3E75FD26u), ucf(0x3E75FD26u)));
    p = __ffma2_rn(p, f, make_float2(ucf(0x3F317218u), ucf(0x3F317218u)));
    p = __ffma2_rn(p, f, make_float2(1.0f, 1.0f));
    return make_float2(ucf(__float_as_uint(p.x) + (__float_as_uint(tm.x) << 23)),
                       ucf(__float_as_uint(p.y) + (__float_as_uint(tm.y) << 23)));
}

// (m_c, s_c) of one chunk; get(j) returns this lane's vector j (read twice: max
// pass, then exp pass).  Every thread of the CTA calls it.
template <class Get>
__device__ __forceinline__ void chunk_stats(const RejArgs &a, int64_t task, Get get, float *scratch, float *scratch2) {
    const int64_t c0 = (task % a.chunks) * kChunk;
    // max, min and the non-finite check on bf16 pairs (NaN-propagating max and min)
    __nv_bfloat162 mx = __halves2bfloat162(__ushort_as_bfloat16(0xFF7Fu), __ushort_as_bfloat16(0xFF7Fu));
    __nv_bfloat162 mn = __halves2bfloat162(__ushort_as_bfloat16(0x7F7Fu), __ushort_as_bfloat16(0x7F7Fu));
#pragma unroll
    for (int j = 0; j < kVectors; ++j)
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t u = word_of(get(j), q);
            const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162 *>(&u);
            mx = __hmax2_nan(mx, v);
            mn = __hmin2_nan(mn, v);
        }
    float m = fmaxf(__bfloat162float(mx.x), __bfloat162float(mx.y));
    float lo = fminf(__bfloat162float(mn.x), __bfloat162float(mn.y));
    const bool bad = !isfinite(__bfloat162float(mx.x)) || !isfinite(__bfloat162float(mx.y)) || !isfinite(lo);
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(a.flags, BD_FLAG_NONFINITE_LOGITS);
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
        lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, d));
    }
    __syncthreads();  // the previous chunk's reductions have read the scratch
    if ((threadIdx.x & 31) == 0) {
        scratch[threadIdx.x >> 5] = m;
        scratch2[threadIdx.x >> 5] = lo;
    }
    __syncthreads();
    m = scratch[0];
    lo = scratch2[0];
#pragma unroll
    for (int i = 1; i < kLanes / 32; ++i) {
        m = fmaxf(m, scratch[i]);
        lo = fminf(lo, scratch2[i]);
    }
    // s_c: per item sequential over the vectors, then the item and lane trees; the
    // clamp of e is an identity when the chunk's smallest entry is within 86.5 of m
    float2 acc[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) acc[q] = make_float2(0.0f, 0.0f);
    const float2 mm = make_float2(-m, -m);
    const bool full = c0 + kChunk <= a.vocab;
    if (full && __fsub_rn(lo, m) >= BD_EXP_FLOOR) {
#pragma unroll
        for (int j = 0; j < kVectors; ++j)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t u = word_of(get(j), q);
                acc[q] = __fadd2_rn(acc[q], exp_pair_unclamped(__fadd2_rn(make_float2(lo_f(u), hi_f(u)), mm)));
            }
    } else {
#pragma unroll
        for (int j = 0; j < kVectors; ++j) {
            const int64_t e0 = c0 + kItems * (threadIdx.x + kLanes * j);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t u = word_of(get(j), q);
                float2 e = exp_pair(__fadd2_rn(make_float2(lo_f(u), hi_f(u)), mm));
                if (e0 + 2 * q >= a.vocab) e.x = 0.0f;
                if (e0 + 2 * q + 1 >= a.vocab) e.y = 0.0f;
                acc[q] = __fadd2_rn(acc[q], e);
            }
        }
    }
    const float s = cta_tree(item_tree(acc), scratch);
    if (threadIdx.x == 0) a.stats[task] = make_float2(m, s);
}

// One CTA per (row, chunk): the chunk's 8 vectors per lane are loaded into
// registers once and reduced twice (max, then sum); four CTAs per SM.
template <bool VEC>
__global__ void __launch_bounds__(kLanes, VEC ? 4 : 1) rej_stats_kernel(const RejArgs a) {
    __shared__ float scratch[kLanes / 32], scratch2[kLanes / 32];
    const int64_t task = blockIdx.x;
    const int64_t g = task * kLanes + threadIdx.x;
    if (g < a.requests) a.counter[g] = 0;  // the sampling kernel's arrival counters
    const int64_t r = task / a.chunks;
    const int64_t tr = static_cast<int64_t>(a.requests) * (a.n + 1);
    const uint16_t *row = r < tr ? a.target + r * a.vocab : a.draft + (r - tr) * a.vocab;
    uint4 w[kVectors];
    load_chunk<VEC>(row, (task % a.chunks) * kChunk, a.vocab, w);
    chunk_stats(a, task, [&](int j) { return w[j]; }, scratch, scratch2);
}

// ---------------------------------------------------------------- kernel 2: decide and sample
// (m, S) of a row from its chunk statistics (one warp; lane l holds chunk l).
__device__ __forceinline__ float2 combine_row(const float2 *st_row, int chunks) {
    const int lane = threadIdx.x & 31;
    const float2 st = lane < chunks ? st_row[lane] : make_float2(-INFINITY, 0.0f);
    float m = st.x;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
    float v = lane < chunks ? __fmul_rn(st.y, exp_one(__fsub_rn(st.x, m))) : 0.0f;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, d));
    return make_float2(m, v);
}

struct PosStat {
    float mp, ip, mq, iq;  // row maxima and reciprocal softmax totals of the target and draft rows
    float lp, lq;          // target and draft logits of the drafted token
    int accept, eog, bad, pad;  // 40 bytes: the float2 statistics that follow stay 8-byte aligned
};

// Shared memory of the sampling kernel: positions, then the request's row statistics.
__host__ __device__ inline size_t sample_smem_bytes(int drafts, int chunks) {
    return (static_cast<size_t>(drafts) + 1) * sizeof(PosStat) +
           (2 * static_cast<size_t>(drafts) + 1) * chunks * sizeof(float2);
}

// Sampling weights of two entries (mode 0: e(l - m_p); 1: max(0, p - q); 2: p) and the p weights.
__device__ __forceinline__ void weights_pair(uint32_t up, uint32_t uq, int mode, const PosStat &ps, float2 &w,
                                             float2 &pw) {
    const float2 ep = exp_pair(__fadd2_rn(make_float2(lo_f(up), hi_f(up)), make_float2(-ps.mp, -ps.mp)));
    if (mode == 0) {
        w = ep;
        pw = ep;
        return;
    }
    pw = __fmul2_rn(ep, make_float2(ps.ip, ps.ip));
    if (mode == 2) {
        w = pw;
        return;
    }
    const float2 eq = exp_pair(__fadd2_rn(make_float2(lo_f(uq), hi_f(uq)), make_float2(-ps.mq, -ps.mq)));
    const float2 qw = __fmul2_rn(eq, make_float2(ps.iq, ps.iq));
    const float2 d = __fadd2_rn(pw, make_float2(-qw.x, -qw.y));
    w = make_float2(fmaxf(d.x, 0.0f), fmaxf(d.y, 0.0f));
}

// The 8 sampling weights (and p weights) of vector j of this lane; entries past the vocabulary weigh 0.
template <bool VEC>
__device__ __forceinline__ void vector_weights(const uint16_t *prow, const uint16_t *qrow, int64_t e0, int64_t vocab,
                                               int mode, const PosStat &ps, float2 (&w)[4], float2 (&pw)[4]) {
    const uint4 vp = load_vector<VEC>(prow, e0, vocab);
    const uint4 vq = mode == 1 ? load_vector<VEC>(qrow, e0, vocab) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        weights_pair(word_of(vp, q), word_of(vq, q), mode, ps, w[q], pw[q]);
        if (e0 + 2 * q >= vocab) w[q].x = pw[q].x = 0.0f;
        if (e0 + 2 * q + 1 >= vocab) w[q].y = pw[q].y = 0.0f;
    }
}

template <bool VEC>
__global__ void __launch_bounds__(kLanes, VEC ? 2 : 1) rej_sample_kernel(const RejArgs a) {
    extern __shared__ PosStat pos_stat[];  // [n + 1], then float2 [2n + 1][chunks]
    __shared__ float scratch[kLanes / 32];
    __shared__ float hs[kLanes];
    __shared__ float2 s_parts[kMaxChunks];
    __shared__ float s_items[kVectors * kItems];
    __shared__ int s_pos, s_mode, s_done, s_last, s_pick, s_lane_hit, s_lane_pos;
    __shared__ float s_target, s_base;
    const int64_t b = blockIdx.x / a.chunks;
    const int c = static_cast<int>(blockIdx.x % a.chunks);
    const int warp = threadIdx.x >> 5;
    float2 *st = reinterpret_cast<float2 *>(pos_stat + a.n + 1);
    // ---- the request's row statistics (target rows 0..n, then draft rows 0..n-1) and drafted logits
    {
        const int per = a.chunks;
        const int64_t t0 = target_stat(a, b, 0) * per, d0 = draft_stat(a, b, 0) * per;
        const int nt = (a.n + 1) * per, nd = a.n * per;
        for (int i = threadIdx.x; i < nt + nd; i += kLanes) st[i] = i < nt ? a.stats[t0 + i] : a.stats[d0 + i - nt];
        for (int i = threadIdx.x; i < a.n; i += kLanes) {
            const int d = a.drafts[b * a.n + i];
            const bool bad = d < 0 || d >= a.vocab;
            pos_stat[i].bad = bad;
            pos_stat[i].lp = bad ? 0.0f : bf16_bits_to_f32(target_row(a, b, i)[d]);
            pos_stat[i].lq = bad ? 0.0f : bf16_bits_to_f32(draft_row(a, b, i)[d]);
            int eog = 0;
            for (int e = 0; e < a.n_eog; ++e) eog |= a.eog[e] == d;
            pos_stat[i].eog = eog;
            if (bad && c == 0) set_flag(a.flags, BD_FLAG_BAD_TOKEN);
        }
    }
    __syncthreads();
    // ---- (m, S) of every row (warps over rows)
    for (int r = warp; r < 2 * a.n + 1; r += kLanes / 32) {
        const float2 ms = combine_row(st + static_cast<int64_t>(r) * a.chunks, a.chunks);
        if ((threadIdx.x & 31) == 0) {
            if (r <= a.n) {
                pos_stat[r].mp = ms.x;
                pos_stat[r].ip = __frcp_rn(ms.y);
            } else {
                pos_stat[r - a.n - 1].mq = ms.x;
                pos_stat[r - a.n - 1].iq = __frcp_rn(ms.y);
            }
        }
    }
    __syncthreads();
    // ---- every position's acceptance test
    for (int i = threadIdx.x; i < a.n; i += kLanes) {
        PosStat &q = pos_stat[i];
        int accept = 0;
        if (!q.bad) {
            const float p = __fmul_rn(exp_one(__fsub_rn(q.lp, q.mp)), q.ip);
            const float qq = __fmul_rn(exp_one(__fsub_rn(q.lq, q.mq)), q.iq);
            accept = __fmul_rn(uniform01(a.seed, static_cast<uint32_t>(b), i, 0, a.offset), qq) < p;
        }
        q.accept = accept;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int pos = a.n, mode = 0, done = 0;
        for (int i = 0; i < a.n; ++i) {
            if (pos_stat[i].accept) {
                if (pos_stat[i].eog && i + 1 < a.n) {
                    if (c == 0) {
                        a.accepted[b] = i;
                        a.next_token[b] = a.drafts[b * a.n + i];
                    }
                    done = 1;
                    break;
                }
                continue;
            }
            pos = i;
            mode = 1;
            break;
        }
        s_pos = pos;
        s_mode = mode;
        s_done = done;
    }
    __syncthreads();
    if (s_done) return;
    const int pos = s_pos;
    const int mode = s_mode;
    const PosStat ps = pos_stat[pos];
    const uint16_t *prow = target_row(a, b, pos);
    const uint16_t *qrow = mode ? draft_row(a, b, pos) : prow;
    // ---- this CTA's chunk: sums of the sampling weights and of p
    {
        const int64_t c0 = static_cast<int64_t>(c) * kChunk;
        uint4 vp[kVectors], vq[kVectors];
        load_chunk<VEC>(prow, c0, a.vocab, vp);
        if (mode == 1) load_chunk<VEC>(qrow, c0, a.vocab, vq);
        float2 acc[4], pacc[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[q] = pacc[q] = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int j = 0; j < kVectors; ++j) {
            const int64_t e0 = c0 + kItems * (threadIdx.x + kLanes * j);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float2 w, pw;
                weights_pair(word_of(vp[j], q), mode == 1 ? word_of(vq[j], q) : 0u, mode, ps, w, pw);
                if (e0 + 2 * q >= a.vocab) w.x = pw.x = 0.0f;
                if (e0 + 2 * q + 1 >= a.vocab) w.y = pw.y = 0.0f;
                acc[q] = __fadd2_rn(acc[q], w);
                pacc[q] = __fadd2_rn(pacc[q], pw);
            }
        }
        const float lw = item_tree(acc), lp = item_tree(pacc);
        a.lanes[(b * a.chunks + c) * kLanes + threadIdx.x] = make_float2(lw, lp);
        __threadfence();
        const float ws = cta_tree(lw, scratch);
        const float psum = mode ? cta_tree(lp, scratch) : ws;
        if (threadIdx.x == 0) {
            a.parts[b * a.chunks + c] = make_float2(ws, psum);
            __threadfence();
            s_last = atomicAdd(a.counter + b, 1) == a.chunks - 1;
        }
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        if (threadIdx.x < a.chunks) s_parts[threadIdx.x] = __ldcg(&a.parts[b * a.chunks + threadIdx.x]);
        __syncthreads();
    }
    // ---- last CTA of the request: pick the chunk, the lane and the item
    if (threadIdx.x == 0) {
        int m = mode;
        float run = 0.0f;
        for (int k = 0; k < a.chunks; ++k) run = __fadd_rn(run, s_parts[k].x);
        if (m == 1 && !(run > 0.0f)) m = 2;  // residual zero everywhere: sample from p
        const bool use_p = m == 2;
        float total = 0.0f;
        if (use_p)
            for (int k = 0; k < a.chunks; ++k) total = __fadd_rn(total, s_parts[k].y);
        else
            total = run;
        const float target = __fmul_rn(uniform01(a.seed, static_cast<uint32_t>(b), pos, 1, a.offset), total);
        float r = 0.0f, base = 0.0f;
        int pick = -1, last_pos = -1;
        for (int k = 0; k < a.chunks; ++k) {
            const float2 pk = s_parts[k];
            const float sk = use_p ? pk.y : pk.x;
            if (pick < 0 && __fadd_rn(r, sk) > target) {
                pick = k;
                base = r;
            }
            if (sk > 0.0f) last_pos = k;
            r = __fadd_rn(r, sk);
        }
        if (pick < 0) {
            pick = last_pos < 0 ? 0 : last_pos;
            base = 0.0f;
            for (int k = 0; k < pick; ++k) {
                const float2 pk = s_parts[k];
                base = __fadd_rn(base, use_p ? pk.y : pk.x);
            }
        }
        s_pick = pick;
        s_mode = m;
        s_target = target;
        s_base = base;
        s_lane_hit = kLanes;
        s_lane_pos = -1;
        a.counter[b] = 0;
    }
    __syncthreads();
    const int m = s_mode;
    const int64_t c0 = static_cast<int64_t>(s_pick) * kChunk;
    const float target = s_target, base = s_base;
    const float2 lane_sum = __ldcg(&a.lanes[(b * a.chunks + s_pick) * kLanes + threadIdx.x]);
    const float mine = m == 2 ? lane_sum.y : lane_sum.x;
    // Hillis-Steele inclusive scan of the lane sums (x[i] += x[i - d], d = 1, 2, 4, ...)
    hs[threadIdx.x] = mine;
    __syncthreads();
    for (int d = 1; d < kLanes; d <<= 1) {
        const float add = threadIdx.x >= d ? hs[threadIdx.x - d] : 0.0f;
        __syncthreads();
        if (threadIdx.x >= d) hs[threadIdx.x] = __fadd_rn(hs[threadIdx.x], add);
        __syncthreads();
    }
    if (__fadd_rn(base, hs[threadIdx.x]) > target) atomicMin(&s_lane_hit, static_cast<int>(threadIdx.x));
    if (mine > 0.0f) atomicMax(&s_lane_pos, static_cast<int>(threadIdx.x));
    __syncthreads();
    const int chosen = s_lane_hit < kLanes ? s_lane_hit : (s_lane_pos >= 0 ? s_lane_pos : 0);
    // the chosen lane's 64 weights: thread j fetches vector j
    if (threadIdx.x < kVectors) {
        float2 w[4], pw[4];
        vector_weights<VEC>(prow, qrow, c0 + kItems * (chosen + kLanes * static_cast<int>(threadIdx.x)), a.vocab, m,
                            ps, w, pw);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            s_items[threadIdx.x * kItems + 2 * q] = w[q].x;
            s_items[threadIdx.x * kItems + 2 * q + 1] = w[q].y;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const float excl = chosen == 0 ? 0.0f : hs[chosen - 1];
        int item = -1, last_pos = -1;
        float run = 0.0f;
        for (int i = 0; i < kVectors * kItems; ++i) {
            const float w = s_items[i];
            run = i ? __fadd_rn(run, w) : w;
            if (item < 0 && __fadd_rn(base, __fadd_rn(excl, run)) > target) item = i;
            if (w > 0.0f) last_pos = i;
        }
        if (item < 0) item = last_pos < 0 ? 0 : last_pos;
        int64_t idx = c0 + kItems * (chosen + kLanes * (item / kItems)) + item % kItems;
        if (idx > a.vocab - 1) idx = a.vocab - 1;
        a.accepted[b] = pos;
        a.next_token[b] = static_cast<int32_t>(idx);
    }
}

}  // namespace bd

using namespace bd;

namespace {
size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }
}  // namespace

namespace {
struct RejLayout {
    size_t stats, parts, lanes, counter, total;
};
RejLayout rej_layout(int requests, int drafts, int chunks) {
    const size_t rows = static_cast<size_t>(requests) * (2 * static_cast<size_t>(drafts) + 1);
    const size_t req_chunks = static_cast<size_t>(requests) * chunks;
    RejLayout l{};
    l.stats = 0;
    l.parts = l.stats + align256(rows * chunks * sizeof(float2));
    l.lanes = l.parts + align256(req_chunks * sizeof(float2));
    l.counter = l.lanes + align256(req_chunks * kLanes * sizeof(float2));
    l.total = l.counter + align256(static_cast<size_t>(requests) * sizeof(int32_t));
    return l;
}
}  // namespace

extern "C" size_t bd_rejection_workspace_bytes(int requests, int drafts, int64_t vocab) {
    if (requests < 0 || drafts < 0 || vocab < 1 || vocab > static_cast<int64_t>(kMaxChunks) * kChunk) return 0;
    return rej_layout(requests, drafts, static_cast<int>((vocab + kChunk - 1) / kChunk)).total;
}

extern "C" int bd_accept_rejection(const uint16_t *target_logits, const uint16_t *draft_logits, int requests,
                                   int drafts, int64_t vocab, const int32_t *draft_tokens, const int32_t *eog,
                                   int n_eog, unsigned long long seed, uint32_t offset, int32_t *accepted,
                                   int32_t *next_token, void *workspace, size_t workspace_bytes, int32_t *flags,
                                   bd_stream_t stream) {
    if (requests < 0 || drafts < 0 || vocab < 1 || n_eog < 0) return BD_ERR_INVALID;
    if (vocab > static_cast<int64_t>(kMaxChunks) * kChunk) return BD_ERR_INVALID;  // one chunk per warp lane
    if (requests == 0) return BD_OK;
    if (!target_logits || (drafts > 0 && (!draft_logits || !draft_tokens)) || (n_eog > 0 && !eog) || !accepted ||
        !next_token)
        return BD_ERR_INVALID;
    const int chunks = static_cast<int>((vocab + kChunk - 1) / kChunk);
    const RejLayout layout = rej_layout(requests, drafts, chunks);
    if (!workspace || workspace_bytes < layout.total) return BD_ERR_WORKSPACE;
    const size_t rows = static_cast<size_t>(requests) * (2 * static_cast<size_t>(drafts) + 1);
    if (rows * chunks > 0x7fffffffu || static_cast<size_t>(requests) * chunks > 0x7fffffffu) return BD_ERR_INVALID;
    const size_t pos_smem = sample_smem_bytes(drafts, chunks);
    if (pos_smem > 160 * 1024) return BD_ERR_TOO_LARGE;
    char *ws = static_cast<char *>(workspace);
    RejArgs a{};
    a.target = target_logits;
    a.draft = draft_logits;
    a.drafts = draft_tokens;
    a.eog = eog;
    a.n_eog = n_eog;
    a.requests = requests;
    a.n = drafts;
    a.chunks = chunks;
    a.vocab = vocab;
    a.seed = seed;
    a.offset = offset;
    a.stats = reinterpret_cast<float2 *>(ws + layout.stats);
    a.parts = reinterpret_cast<float2 *>(ws + layout.parts);
    a.lanes = reinterpret_cast<float2 *>(ws + layout.lanes);
    a.counter = reinterpret_cast<int32_t *>(ws + layout.counter);
    a.accepted = accepted;
    a.next_token = next_token;
    a.flags = flags;
    const bool vec = vocab % kItems == 0 && (reinterpret_cast<uintptr_t>(target_logits) & 15) == 0 &&
                     (drafts == 0 || (reinterpret_cast<uintptr_t>(draft_logits) & 15) == 0);
    // kernel 1: one CTA per (row, chunk); its threads also clear the request counters
    const size_t tasks = rows * chunks;
    const unsigned stat_blocks = static_cast<unsigned>(tasks);
    auto k2 = vec ? rej_sample_kernel<true> : rej_sample_kernel<false>;
    if (pos_smem > 48 * 1024 &&
        cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(pos_smem)) !=
            cudaSuccess)
        return BD_ERR_LAUNCH;
    if (vec)
        rej_stats_kernel<true><<<stat_blocks, kLanes, 0, stream>>>(a);
    else
        rej_stats_kernel<false><<<stat_blocks, kLanes, 0, stream>>>(a);
    BD_CHECK_LAUNCH();
    k2<<<static_cast<unsigned>(static_cast<size_t>(requests) * chunks), kLanes, pos_smem, stream>>>(a);
    BD_CHECK_LAUNCH();
    return BD_OK;
}
