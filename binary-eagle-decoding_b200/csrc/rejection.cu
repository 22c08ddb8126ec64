// Temperature-1 speculative rejection sampling over vocabulary-sized bf16 rows.
//
// The reference has no implementation of its own (it runs llama.cpp's sampler;
// the only in-tree pin is the statistical check of native/verifier-test.cpp:43-80
// and the EOG break of benchmarks/native.py:19-38), so this file implements a
// deterministic contract that a CPU restatement reproduces bit for bit:
//   * uniforms: Philox4x32-10 (Salmon et al., SC'11), key = the 64-bit seed,
//     counter = (request, position, purpose, offset), u = (x0 >> 8) * 2^-24;
//   * exp: Cody-Waite reduction by ln 2 and a degree-7 Taylor polynomial, every
//     step a separately rounded fp32 multiply or add (no contraction);
//   * softmax sums: tiles of 4096 entries = 512 lanes x 8 contiguous entries,
//     each lane adds its 8 sequentially, lane sums combine in a balanced tree of
//     adjacent pairs, tiles add sequentially;
//   * accept draft d at position i iff u * q(d) < p(d); an accepted EOG that is
//     not the last draft ends the round; on rejection sample from max(0, p - q),
//     after all drafts from p of the bonus row, by an inverse-CDF search over the
//     same tiles (Hillis-Steele scan of the chosen tile's lane sums).
// Kernel 1 computes every row's max, exp-sum and the probability of the drafted
// token; kernel 2 decides each request and samples its correction/bonus token.
#include "kernels.cuh"

namespace bd {

constexpr int kLanes = 512;
constexpr int kItems = 8;
constexpr int kTile = kLanes * kItems;

// ---------------------------------------------------------------- deterministic exp
__device__ __forceinline__ float exp_fixed(float x) {
    // constants as exact fp32 bit patterns: log2(e); ln 2 with its low 9 mantissa
    // bits cleared (15 significant bits, so k * hi is exact for |k| <= 512); the
    // fp32 rounding of the rest; Taylor coefficients 1/n! rounded to fp32
    const float kLog2e = __uint_as_float(0x3FB8AA3Bu);
    const float kLn2Hi = __uint_as_float(0x3F317200u);
    const float kLn2Lo = __uint_as_float(0x35BFBE8Eu);
    const float k = rintf(__fmul_rn(x, kLog2e));
    const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(k, kLn2Hi)), __fmul_rn(k, kLn2Lo));
    float p = __uint_as_float(0x39500D01u);                        // 1/7!
    p = __fadd_rn(__fmul_rn(p, r), __uint_as_float(0x3AB60B61u));  // 1/6!
    p = __fadd_rn(__fmul_rn(p, r), __uint_as_float(0x3C088889u));  // 1/5!
    p = __fadd_rn(__fmul_rn(p, r), __uint_as_float(0x3D2AAAABu));  // 1/4!
    p = __fadd_rn(__fmul_rn(p, r), __uint_as_float(0x3E2AAAABu));  // 1/3!
    p = __fadd_rn(__fmul_rn(p, r), 0.5f);
    p = __fadd_rn(__fmul_rn(p, r), 1.0f);
    p = __fadd_rn(__fmul_rn(p, r), 1.0f);
    const int ki = static_cast<int>(k);
    if (ki < -126) return 0.0f;
    const int kc = ki > 127 ? 127 : ki;
    return __fmul_rn(p, __uint_as_float(static_cast<uint32_t>(kc + 127) << 23));
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
    return __fmul_rn(static_cast<float>(r.x >> 8), __uint_as_float(0x33800000u));  // 2^-24
}

__device__ __forceinline__ float bf16f(uint16_t b) { return __uint_as_float(static_cast<uint32_t>(b) << 16); }

// Balanced adjacent-pair tree over the 512 lane values of a CTA; every thread gets the total.
__device__ __forceinline__ float tile_tree(float v, float *warp_part) {
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, d));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) warp_part[threadIdx.x >> 5] = v;
    __syncthreads();
    float w[kLanes / 32];
#pragma unroll
    for (int i = 0; i < kLanes / 32; ++i) w[i] = warp_part[i];
#pragma unroll
    for (int n = kLanes / 32; n > 1; n >>= 1)
#pragma unroll
        for (int i = 0; i < n / 2; ++i) w[i] = __fadd_rn(w[2 * i], w[2 * i + 1]);
    return w[0];
}

struct RejArgs {
    const uint16_t *target;   // [B][n+1][V]
    const uint16_t *draft;    // [B][n][V]
    const int32_t *drafts;    // [B][n]
    const int32_t *eog;
    int n_eog;
    int requests, n;
    int64_t vocab;
    unsigned long long seed;
    uint32_t offset;
    float *row_max, *row_sum, *row_prob;  // [B(n+1) + Bn]
    int32_t *accepted, *next_token;
    int32_t *flags;
};

// Row r < B(n+1): target row (request r / (n+1), position r % (n+1)); else draft row.
__device__ __forceinline__ const uint16_t *row_ptr(const RejArgs &a, int64_t r, int &request, int &position,
                                                   bool &is_target) {
    const int64_t tr = static_cast<int64_t>(a.requests) * (a.n + 1);
    if (r < tr) {
        request = static_cast<int>(r / (a.n + 1));
        position = static_cast<int>(r % (a.n + 1));
        is_target = true;
        return a.target + r * a.vocab;
    }
    const int64_t q = r - tr;
    request = static_cast<int>(q / a.n);
    position = static_cast<int>(q % a.n);
    is_target = false;
    return a.draft + q * a.vocab;
}

__global__ void __launch_bounds__(kLanes) rejection_stats_kernel(const RejArgs a) {
    __shared__ float part[kLanes / 32];
    __shared__ float s_running;
    const int64_t r = blockIdx.x;
    int request, position;
    bool is_target;
    const uint16_t *row = row_ptr(a, r, request, position, is_target);
    // pass 1: maximum, finiteness
    float m = -INFINITY;
    bool bad = false;
    for (int64_t i = threadIdx.x; i < a.vocab; i += kLanes) {
        const float f = bf16f(row[i]);
        bad |= !isfinite(f);
        m = fmaxf(m, f);
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = m;
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(a.flags, BD_FLAG_NONFINITE_LOGITS);
    __syncthreads();
    m = part[0];
#pragma unroll
    for (int w = 1; w < kLanes / 32; ++w) m = fmaxf(m, part[w]);
    // pass 2: tile sums of exp(l - m) in the contract's order
    if (threadIdx.x == 0) s_running = 0.0f;
    const int64_t tiles = (a.vocab + kTile - 1) / kTile;
    for (int64_t k = 0; k < tiles; ++k) {
        float lane = 0.0f;
#pragma unroll
        for (int e = 0; e < kItems; ++e) {
            const int64_t i = k * kTile + threadIdx.x * kItems + e;
            const float v = i < a.vocab ? exp_fixed(__fsub_rn(bf16f(row[i]), m)) : 0.0f;
            lane = e ? __fadd_rn(lane, v) : v;
        }
        const float tile = tile_tree(lane, part);
        if (threadIdx.x == 0) s_running = __fadd_rn(s_running, tile);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const float total = s_running;
        a.row_max[r] = m;
        a.row_sum[r] = total;
        // probability of the drafted token at this position (target rows past the last draft have none)
        float prob = 0.0f;
        if (position < a.n) {
            const int d = a.drafts[static_cast<int64_t>(request) * a.n + position];
            if (d < 0 || d >= a.vocab) {
                set_flag(a.flags, BD_FLAG_BAD_TOKEN);
            } else {
                prob = __fdiv_rn(exp_fixed(__fsub_rn(bf16f(row[d]), m)), total);
            }
        }
        a.row_prob[r] = prob;
    }
}

// Weight of entry j of the sampling distribution: residual max(0, p - q) or p.
__device__ __forceinline__ float sample_weight(const uint16_t *prow, const uint16_t *qrow, int64_t j, int64_t vocab,
                                               float pm, float ps, float qm, float qs, int mode) {
    if (j >= vocab) return 0.0f;
    const float ep = exp_fixed(__fsub_rn(bf16f(prow[j]), pm));
    if (mode == 0) return ep;                                 // bonus: unnormalised p
    const float p = __fdiv_rn(ep, ps);
    if (mode == 2) return p;                                  // residual was all zero: p
    const float q = __fdiv_rn(exp_fixed(__fsub_rn(bf16f(qrow[j]), qm)), qs);
    return fmaxf(__fsub_rn(p, q), 0.0f);                      // residual
}

__global__ void __launch_bounds__(kLanes) rejection_decide_kernel(const RejArgs a) {
    __shared__ float part[kLanes / 32];
    __shared__ float tile_sums[128];
    __shared__ float hs[kLanes];
    __shared__ int s_pos, s_mode, s_done, s_pick;
    __shared__ float s_target, s_running;
    const int b = blockIdx.x;
    const int64_t tr = static_cast<int64_t>(a.requests) * (a.n + 1);
    if (threadIdx.x == 0) {
        // walk the drafts (the acceptance rule of the contract)
        int pos = a.n, mode = 0, done = 0;
        for (int i = 0; i < a.n; ++i) {
            const int64_t prow = static_cast<int64_t>(b) * (a.n + 1) + i;
            const int64_t qrow = tr + static_cast<int64_t>(b) * a.n + i;
            const float p = a.row_prob[prow], q = a.row_prob[qrow];
            const float u = uniform01(a.seed, b, i, 0, a.offset);
            const int d = a.drafts[static_cast<int64_t>(b) * a.n + i];
            if (__fmul_rn(u, q) < p) {
                bool is_eog = false;
                for (int e = 0; e < a.n_eog; ++e) is_eog |= a.eog[e] == d;
                if (is_eog && i + 1 < a.n) {
                    a.accepted[b] = i;
                    a.next_token[b] = d;
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
    int mode = s_mode;
    const int64_t prow_i = static_cast<int64_t>(b) * (a.n + 1) + pos;
    const int64_t qrow_i = tr + static_cast<int64_t>(b) * a.n + (mode ? pos : 0);
    const uint16_t *prow = a.target + prow_i * a.vocab;
    const uint16_t *qrow = a.draft + (qrow_i - tr) * a.vocab;
    const float pm = a.row_max[prow_i], ps = a.row_sum[prow_i];
    const float qm = mode ? a.row_max[qrow_i] : 0.0f, qs = mode ? a.row_sum[qrow_i] : 1.0f;
    const int64_t tiles = (a.vocab + kTile - 1) / kTile;
    for (int attempt = 0; attempt < 2; ++attempt) {
        // tile sums of the weights, then the running total
        for (int64_t k = 0; k < tiles; ++k) {
            float lane = 0.0f;
#pragma unroll
            for (int e = 0; e < kItems; ++e) {
                const float v = sample_weight(prow, qrow, k * kTile + threadIdx.x * kItems + e, a.vocab, pm, ps, qm,
                                              qs, mode);
                lane = e ? __fadd_rn(lane, v) : v;
            }
            const float tile = tile_tree(lane, part);
            if (threadIdx.x == 0) tile_sums[k] = tile;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float run = 0.0f;
            for (int64_t k = 0; k < tiles; ++k) run = __fadd_rn(run, tile_sums[k]);
            s_running = run;
        }
        __syncthreads();
        if (mode == 1 && !(s_running > 0.0f)) {
            mode = 2;  // residual is all zero: sample from p (the contract's fallback)
            __syncthreads();
            continue;
        }
        break;
    }
    __syncthreads();  // every thread has read s_running before thread 0 reuses it
    if (threadIdx.x == 0) {
        const float u = uniform01(a.seed, b, pos, 1, a.offset);
        const float target = __fmul_rn(u, s_running);
        // tile: first with running + tile_sum > target, else last with a positive sum, else 0
        float run = 0.0f;
        int pick = -1, last_pos = -1;
        for (int64_t k = 0; k < tiles; ++k) {
            if (pick < 0 && __fadd_rn(run, tile_sums[k]) > target) pick = static_cast<int>(k);
            if (tile_sums[k] > 0.0f) last_pos = static_cast<int>(k);
            if (pick < 0) run = __fadd_rn(run, tile_sums[k]);
        }
        if (pick < 0) {
            pick = last_pos < 0 ? 0 : last_pos;
            run = 0.0f;
            for (int k = 0; k < pick; ++k) run = __fadd_rn(run, tile_sums[k]);
        }
        s_pick = pick;
        s_target = target;
        s_running = run;  // running sum before the picked tile
    }
    __syncthreads();
    const int64_t k = s_pick;
    const float target = s_target, base = s_running;
    float items[kItems], seq[kItems];
    float lane = 0.0f;
#pragma unroll
    for (int e = 0; e < kItems; ++e) {
        items[e] = sample_weight(prow, qrow, k * kTile + threadIdx.x * kItems + e, a.vocab, pm, ps, qm, qs, mode);
        lane = e ? __fadd_rn(lane, items[e]) : items[e];
        seq[e] = lane;
    }
    // Hillis-Steele inclusive scan of the lane sums (x[i] += x[i - d], d = 1, 2, 4, ...)
    hs[threadIdx.x] = lane;
    __syncthreads();
    for (int d = 1; d < kLanes; d <<= 1) {
        const float add = threadIdx.x >= d ? hs[threadIdx.x - d] : 0.0f;
        __syncthreads();
        if (threadIdx.x >= d) hs[threadIdx.x] = __fadd_rn(hs[threadIdx.x], add);
        __syncthreads();
    }
    // lane: smallest with base + incl > target, else largest with a positive lane sum, else 0
    const bool hit = __fadd_rn(base, hs[threadIdx.x]) > target;
    __shared__ int s_lane_hit, s_lane_pos;
    if (threadIdx.x == 0) {
        s_lane_hit = kLanes;
        s_lane_pos = -1;
    }
    __syncthreads();
    if (hit) atomicMin(&s_lane_hit, static_cast<int>(threadIdx.x));
    if (lane > 0.0f) atomicMax(&s_lane_pos, static_cast<int>(threadIdx.x));
    __syncthreads();
    const int chosen = s_lane_hit < kLanes ? s_lane_hit : (s_lane_pos >= 0 ? s_lane_pos : 0);
    if (static_cast<int>(threadIdx.x) == chosen) {
        const float excl = chosen == 0 ? 0.0f : hs[chosen - 1];
        int item = -1, last_pos = -1;
        for (int e = 0; e < kItems; ++e) {
            if (item < 0 && __fadd_rn(base, __fadd_rn(excl, seq[e])) > target) item = e;
            if (items[e] > 0.0f) last_pos = e;
        }
        if (item < 0) item = last_pos < 0 ? 0 : last_pos;
        int64_t idx = k * kTile + static_cast<int64_t>(chosen) * kItems + item;
        if (idx > a.vocab - 1) idx = a.vocab - 1;
        a.accepted[b] = pos;
        a.next_token[b] = static_cast<int32_t>(idx);
    }
}

}  // namespace bd

using namespace bd;

extern "C" size_t bd_rejection_workspace_bytes(int requests, int drafts) {
    const size_t rows = static_cast<size_t>(requests) * (2 * drafts + 1);
    return 3 * rows * sizeof(float) + 3 * 256;
}

extern "C" int bd_accept_rejection(const uint16_t *target_logits, const uint16_t *draft_logits, int requests,
                                   int drafts, int64_t vocab, const int32_t *draft_tokens, const int32_t *eog,
                                   int n_eog, unsigned long long seed, uint32_t offset, int32_t *accepted,
                                   int32_t *next_token, void *workspace, size_t workspace_bytes, int32_t *flags,
                                   bd_stream_t stream) {
    if (requests < 0 || drafts < 0 || vocab < 1 || vocab > 0x7fffffff || n_eog < 0) return BD_ERR_INVALID;
    if (vocab > static_cast<int64_t>(128) * kTile) return BD_ERR_INVALID;  // tile sums live in shared memory
    if (requests == 0) return BD_OK;
    if (!target_logits || (drafts > 0 && (!draft_logits || !draft_tokens)) || (n_eog > 0 && !eog) || !accepted ||
        !next_token)
        return BD_ERR_INVALID;
    if (!workspace || workspace_bytes < bd_rejection_workspace_bytes(requests, drafts)) return BD_ERR_WORKSPACE;
    const size_t rows = static_cast<size_t>(requests) * (2 * drafts + 1);
    const size_t stride = (rows * sizeof(float) + 255) & ~static_cast<size_t>(255);
    RejArgs a{};
    a.target = target_logits;
    a.draft = draft_logits;
    a.drafts = draft_tokens;
    a.eog = eog;
    a.n_eog = n_eog;
    a.requests = requests;
    a.n = drafts;
    a.vocab = vocab;
    a.seed = seed;
    a.offset = offset;
    a.row_max = static_cast<float *>(workspace);
    a.row_sum = reinterpret_cast<float *>(static_cast<char *>(workspace) + stride);
    a.row_prob = reinterpret_cast<float *>(static_cast<char *>(workspace) + 2 * stride);
    a.accepted = accepted;
    a.next_token = next_token;
    a.flags = flags;
    rejection_stats_kernel<<<static_cast<unsigned>(rows), kLanes, 0, stream>>>(a);
    BD_CHECK_LAUNCH();
    rejection_decide_kernel<<<static_cast<unsigned>(requests), kLanes, 0, stream>>>(a);
    BD_CHECK_LAUNCH();
    return BD_OK;
}
