// Block-draft acceptance over vocabulary-sized bf16 logit rows.
//
// Greedy: the grid streams all rows as equal contiguous ranges; each CTA folds
// the argmax of every row piece it covers (strict '>' so the lowest index wins
// ties, -0.0 == +0.0, non-finite logits flagged) into the row's 64-bit key with
// an atomic max (the key order makes the result independent of arrival order),
// and the last CTA to finish walks the drafts (benchmarks/verifier.py:107-113).
// Plain row argmax keeps one CTA per row.
#include <mutex>

#include "common.cuh"

namespace bd {

constexpr int kArgmaxThreads = 512;

// Orderable 64-bit key: larger value first, then smaller index.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
    uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(b) << 32) | static_cast<unsigned long long>(~idx);
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long k) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, d);
        k = o > k ? o : k;
    }
    return k;
}

struct GreedyArgs {
    const uint16_t *logits;
    int64_t rows, vocab;
    int32_t *targets;
    int32_t *flags;
    int positions;             // drafts + 1 rows per request (0: plain argmax)
    const int32_t *drafts;     // [requests][positions - 1]
    const int32_t *eog;
    int n_eog;
    int32_t *accepted, *next_token;
    int32_t *counters;         // [requests] (per-row kernel) or [1] (stream kernel), zero on entry, left zero
    unsigned long long *keys;  // [rows] argmax keys of the stream kernel, zero on entry, left zero
};

// Running maximum of one thread: indices arrive in increasing order, so a
// strict '>' keeps the lowest index of the maximum.  Non-finite values are
// found separately (packed NaN-propagating min/max) and never win.
struct RunMax {
    float v = -INFINITY;
    uint32_t i = 0xffffffffu;
    __device__ __forceinline__ void push(float f, uint32_t idx) {
        const bool up = f > v && f != INFINITY;
        v = up ? f : v;
        i = up ? idx : i;
    }
};

__device__ __forceinline__ void push_word(RunMax &m, __nv_bfloat162 &lo, __nv_bfloat162 &hi, uint32_t w,
                                          uint32_t idx) {
    m.push(__uint_as_float(w << 16), idx);
    m.push(__uint_as_float(w & 0xffff0000u), idx + 1);
    const __nv_bfloat162 pair = *reinterpret_cast<const __nv_bfloat162 *>(&w);
    hi = __hmax2_nan(hi, pair);
    lo = __hmin2_nan(lo, pair);
}

// Running maximum over 8-element vectors: the maximum of each vector comes from
// three packed bf16 max operations, and only the vector that holds the running
// maximum is remembered (its value and the index of its first element); the
// element index inside it is resolved once at the end (resolve_vec).  Indices
// arrive in increasing order, so a strict '>' keeps the first vector with the
// maximum.  A vector whose maximum is +inf (never a winner) goes through the
// exact per-element path instead; NaN maxima lose every comparison.
struct RunVec {
    float v = -INFINITY;
    uint32_t base = 0xffffffffu;
    const uint4 *at = nullptr;
};

__device__ __forceinline__ void push_vec(RunVec &m, RunMax &slow, __nv_bfloat162 &lo, __nv_bfloat162 &hi,
                                         const uint4 &v, const uint4 *at, uint32_t base) {
    const __nv_bfloat162 p0 = *reinterpret_cast<const __nv_bfloat162 *>(&v.x);
    const __nv_bfloat162 p1 = *reinterpret_cast<const __nv_bfloat162 *>(&v.y);
    const __nv_bfloat162 p2 = *reinterpret_cast<const __nv_bfloat162 *>(&v.z);
    const __nv_bfloat162 p3 = *reinterpret_cast<const __nv_bfloat162 *>(&v.w);
    const __nv_bfloat162 c = __hmax2(__hmax2(p0, p1), __hmax2(p2, p3));
    const float bm = fmaxf(__low2float(c), __high2float(c));
    if (bm > m.v) {
        if (bm != INFINITY) {
            m.v = bm;
            m.base = base;
            m.at = at;
        } else {
            push_word(slow, lo, hi, v.x, base);
            push_word(slow, lo, hi, v.y, base + 2);
            push_word(slow, lo, hi, v.z, base + 4);
            push_word(slow, lo, hi, v.w, base + 6);
            return;
        }
    }
    hi = __hmax2_nan(hi, __hmax2_nan(__hmax2_nan(p0, p1), __hmax2_nan(p2, p3)));
    lo = __hmin2_nan(lo, __hmin2_nan(__hmin2_nan(p0, p1), __hmin2_nan(p2, p3)));
}

// The key of a lane's best vector (its first element equal to the maximum) merged
// with the exact path's key.
__device__ __forceinline__ unsigned long long resolve_vec(const RunVec &m, const RunMax &slow) {
    unsigned long long best = slow.i == 0xffffffffu ? 0ull : argmax_key(slow.v, slow.i);
    if (m.base != 0xffffffffu) {
        const uint4 v = *m.at;  // re-read one 16-byte vector
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t j = 8;
#pragma unroll
        for (int k = 7; k >= 0; --k) {
            const uint32_t bits = (k & 1) ? (w[k >> 1] & 0xffff0000u) : (w[k >> 1] << 16);
            if (__uint_as_float(bits) == m.v) j = static_cast<uint32_t>(k);
        }
        const unsigned long long kv = argmax_key(m.v, m.base + j);
        best = kv > best ? kv : best;
    }
    return best;
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_greedy_kernel(const GreedyArgs a) {
    __shared__ unsigned long long part[kArgmaxThreads / 32];
    __shared__ int last;
    const int64_t row = blockIdx.x;
    const uint16_t *src = a.logits + row * a.vocab;
    RunMax m;
    __nv_bfloat162 hi = __float2bfloat162_rn(-1.0f), lo = __float2bfloat162_rn(1.0f);
    const bool vec = (a.vocab % 8) == 0 && (reinterpret_cast<uintptr_t>(src) & 15) == 0;
    if (vec) {
        const int64_t nvec = a.vocab / 8;
        const uint4 *p = reinterpret_cast<const uint4 *>(src);
        int64_t i = threadIdx.x;
        for (; i + 3 * kArgmaxThreads < nvec; i += 4 * kArgmaxThreads) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = ld_stream_u4(p + i + u * kArgmaxThreads);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const uint32_t base = static_cast<uint32_t>((i + u * kArgmaxThreads) * 8);
                push_word(m, lo, hi, v[u].x, base);
                push_word(m, lo, hi, v[u].y, base + 2);
                push_word(m, lo, hi, v[u].z, base + 4);
                push_word(m, lo, hi, v[u].w, base + 6);
            }
        }
        for (; i < nvec; i += kArgmaxThreads) {
            const uint4 v = ld_stream_u4(p + i);
            const uint32_t base = static_cast<uint32_t>(i * 8);
            push_word(m, lo, hi, v.x, base);
            push_word(m, lo, hi, v.y, base + 2);
            push_word(m, lo, hi, v.z, base + 4);
            push_word(m, lo, hi, v.w, base + 6);
        }
    } else {
        for (int64_t i = threadIdx.x; i < a.vocab; i += kArgmaxThreads) {
            const uint32_t w = src[i];
            m.push(__uint_as_float(w << 16), static_cast<uint32_t>(i));
            const __nv_bfloat162 pair = *reinterpret_cast<const __nv_bfloat162 *>(&w);
            hi = __hmax2_nan(hi, pair);
            lo = __hmin2_nan(lo, pair);
        }
    }
    const float2 hf = __bfloat1622float2(hi), lf = __bfloat1622float2(lo);
    const bool bad = !isfinite(hf.x) || !isfinite(hf.y) || !isfinite(lf.x) || !isfinite(lf.y);
    unsigned long long best = m.i == 0xffffffffu ? 0ull : argmax_key(m.v, m.i);
    best = warp_max_u64(best);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = best;
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(a.flags, BD_FLAG_NONFINITE_LOGITS);
    __syncthreads();
    if (threadIdx.x < 32) {
        unsigned long long k = threadIdx.x < kArgmaxThreads / 32 ? part[threadIdx.x] : 0ull;
        k = warp_max_u64(k);
        if (threadIdx.x == 0) {
            const int32_t idx = static_cast<int32_t>(~static_cast<uint32_t>(k & 0xffffffffull));
            a.targets[row] = idx;
            last = 0;
            if (a.positions > 0) {
                __threadfence();
                const int64_t request = row / a.positions;
                const int old = atomicAdd(a.counters + request, 1);
                last = old == a.positions - 1;
            }
        }
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    // the last row of this request: walk the drafts
    __threadfence();
    const int64_t request = row / a.positions;
    const int n = a.positions - 1;
    const int32_t *tg = a.targets + request * a.positions;
    const int32_t *dr = a.drafts + request * n;
    int acc = n;
    int nxt = __ldcg(tg + n);
    for (int i = 0; i < n; ++i) {
        const int t = __ldcg(tg + i);
        bool is_eog = false;
        for (int e = 0; e < a.n_eog; ++e) is_eog |= a.eog[e] == t;
        if (t != dr[i] || (is_eog && i + 1 < n)) {
            acc = i;
            nxt = t;
            break;
        }
    }
    a.accepted[request] = acc;
    a.next_token[request] = nxt;
    atomicExch(a.counters + request, 0);
}


constexpr int kStreamThreads = 512;

// Greedy acceptance as one balanced stream: the grid (sized to the resident CTA
// count) splits the rows' concatenated vectors into equal contiguous ranges; a
// CTA folds each row piece of its range into the row's 64-bit key with an
// atomic max (order-independent), and the last CTA to finish decodes every
// key and walks every request's drafts.  VEC: 8 entries per unit (16-byte
// loads), else one entry per unit.
template <bool VEC>
__global__ void __launch_bounds__(kStreamThreads) greedy_stream_kernel(const GreedyArgs a) {
    __shared__ unsigned long long part[kStreamThreads / 32];
    __shared__ int last;
    const int64_t per_row = VEC ? a.vocab / 8 : a.vocab;
    const int64_t total = a.rows * per_row;
    const int64_t q = total / gridDim.x, rmd = total % gridDim.x;
    const int64_t begin = q * blockIdx.x + min(static_cast<int64_t>(blockIdx.x), rmd);
    const int64_t end = begin + q + (static_cast<int64_t>(blockIdx.x) < rmd ? 1 : 0);
    __nv_bfloat162 hi = __float2bfloat162_rn(-1.0f), lo = __float2bfloat162_rn(1.0f);
    for (int64_t seg = begin; seg < end;) {
        const int64_t row = seg / per_row;
        const int64_t seg_end = min(end, (row + 1) * per_row);
        const int64_t row0 = row * per_row;
        RunMax m;
        RunVec mv;
        if (VEC) {
            const uint4 *p = reinterpret_cast<const uint4 *>(a.logits);
            int64_t u = seg + threadIdx.x;
            for (; u + 3 * kStreamThreads < seg_end; u += 4 * kStreamThreads) {
                uint4 v[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) v[k] = ld_stream_u4(p + u + k * kStreamThreads);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    push_vec(mv, m, lo, hi, v[k], p + u + k * kStreamThreads,
                             static_cast<uint32_t>((u + k * kStreamThreads - row0) * 8));
            }
            for (; u < seg_end; u += kStreamThreads)
                push_vec(mv, m, lo, hi, ld_stream_u4(p + u), p + u, static_cast<uint32_t>((u - row0) * 8));
        } else {
            for (int64_t u = seg + threadIdx.x; u < seg_end; u += kStreamThreads) {
                const uint32_t w = a.logits[u];
                m.push(__uint_as_float(w << 16), static_cast<uint32_t>(u - row0));
                const __nv_bfloat162 pair = *reinterpret_cast<const __nv_bfloat162 *>(&w);
                hi = __hmax2_nan(hi, pair);
                lo = __hmin2_nan(lo, pair);
            }
        }
        unsigned long long best = resolve_vec(mv, m);
        best = warp_max_u64(best);
        __syncthreads();  // the previous piece's reduction has read part[]
        if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = best;
        __syncthreads();
        if (threadIdx.x == 0) {
            unsigned long long k = part[0];
#pragma unroll
            for (int w = 1; w < kStreamThreads / 32; ++w) k = part[w] > k ? part[w] : k;
            if (k) atomicMax(a.keys + row, k);
        }
        seg = seg_end;
    }
    const float2 hf = __bfloat1622float2(hi), lf = __bfloat1622float2(lo);
    const bool bad = !isfinite(hf.x) || !isfinite(hf.y) || !isfinite(lf.x) || !isfinite(lf.y);
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(a.flags, BD_FLAG_NONFINITE_LOGITS);
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(a.counters, 1) == static_cast<int>(gridDim.x) - 1;
    }
    __syncthreads();
    if (!last) return;
    // the last CTA: decode (and clear) every key, then walk every request
    __threadfence();
    for (int64_t r = threadIdx.x; r < a.rows; r += kStreamThreads) {
        const unsigned long long k = atomicExch(a.keys + r, 0ull);
        a.targets[r] = static_cast<int32_t>(~static_cast<uint32_t>(k & 0xffffffffull));
    }
    __syncthreads();
    __threadfence_block();
    const int64_t requests = a.rows / a.positions;
    const int n = a.positions - 1;
    for (int64_t request = threadIdx.x; request < requests; request += kStreamThreads) {
        const int32_t *tg = a.targets + request * a.positions;
        const int32_t *dr = a.drafts + request * n;
        int acc = n;
        int nxt = tg[n];
        for (int i = 0; i < n; ++i) {
            const int t = tg[i];
            bool is_eog = false;
            for (int e = 0; e < a.n_eog; ++e) is_eog |= a.eog[e] == t;
            if (t != dr[i] || (is_eog && i + 1 < n)) {
                acc = i;
                nxt = t;
                break;
            }
        }
        a.accepted[request] = acc;
        a.next_token[request] = nxt;
    }
    if (threadIdx.x == 0) atomicExch(a.counters, 0);
}

}  // namespace bd

using namespace bd;

namespace {
size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

int launch_greedy_stream(GreedyArgs &a, bd_stream_t stream) {
    static std::mutex mu;
    static int grid[64][2] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BD_ERR_DEVICE;
    const bool vec = (a.vocab % 8) == 0 && (reinterpret_cast<uintptr_t>(a.logits) & 15) == 0;
    int g = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        int &cached = grid[dev][vec ? 1 : 0];
        if (!cached) {
            int sms = 0, per_sm = 0;
            if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
                cudaOccupancyMaxActiveBlocksPerMultiprocessor(
                    &per_sm, vec ? greedy_stream_kernel<true> : greedy_stream_kernel<false>, kStreamThreads, 0) !=
                    cudaSuccess)
                return BD_ERR_LAUNCH;
            cached = sms * (per_sm > 0 ? per_sm : 1);
        }
        g = cached;
    }
    const int64_t units = a.rows * (vec ? a.vocab / 8 : a.vocab);
    const int64_t min_units = vec ? 4 * kStreamThreads : 8 * kStreamThreads;  // at least a few loads per thread
    int64_t blocks = (units + min_units - 1) / min_units;
    if (blocks > g) blocks = g;
    if (blocks < 1) blocks = 1;
    if (vec)
        greedy_stream_kernel<true><<<static_cast<unsigned>(blocks), kStreamThreads, 0, stream>>>(a);
    else
        greedy_stream_kernel<false><<<static_cast<unsigned>(blocks), kStreamThreads, 0, stream>>>(a);
    BD_CHECK_LAUNCH();
    return BD_OK;
}
}  // namespace

extern "C" size_t bd_accept_workspace_bytes(int requests, int drafts) {
    if (requests < 0 || drafts < 0) return 0;
    const size_t rows = static_cast<size_t>(requests) * (drafts + 1);
    return align256(rows * sizeof(int32_t)) + align256(static_cast<size_t>(requests) * sizeof(int32_t)) +
           align256(rows * sizeof(unsigned long long));
}

extern "C" int bd_accept_greedy(const uint16_t *logits, int requests, int drafts, int64_t vocab,
                                const int32_t *draft_tokens, const int32_t *eog, int n_eog, int32_t *accepted,
                                int32_t *next_token, int32_t *targets, void *workspace, size_t workspace_bytes,
                                int32_t *flags, bd_stream_t stream) {
    if (requests < 0 || drafts < 0 || vocab < 1 || vocab > 0x7fffffff || n_eog < 0) return BD_ERR_INVALID;
    if (requests == 0) return BD_OK;
    if (!logits || (drafts > 0 && !draft_tokens) || (n_eog > 0 && !eog) || !accepted || !next_token)
        return BD_ERR_INVALID;
    if (!workspace || workspace_bytes < bd_accept_workspace_bytes(requests, drafts)) return BD_ERR_WORKSPACE;
    const size_t rows = static_cast<size_t>(requests) * (drafts + 1);
    char *ws = static_cast<char *>(workspace);
    GreedyArgs a{};
    a.logits = logits;
    a.rows = static_cast<int64_t>(rows);
    a.vocab = vocab;
    a.targets = targets ? targets : reinterpret_cast<int32_t *>(ws);
    a.flags = flags;
    a.positions = drafts + 1;
    a.drafts = draft_tokens;
    a.eog = eog;
    a.n_eog = n_eog;
    a.accepted = accepted;
    a.next_token = next_token;
    a.counters = reinterpret_cast<int32_t *>(ws + align256(rows * sizeof(int32_t)));
    a.keys = reinterpret_cast<unsigned long long *>(ws + align256(rows * sizeof(int32_t)) +
                                                    align256(static_cast<size_t>(requests) * sizeof(int32_t)));
    return launch_greedy_stream(a, stream);
}

// ---------------------------------------------------------------------------
// Greedy acceptance without any allocation.
//
// Some callers cannot allocate device memory at all: a verifier embedded in a
// host serving runtime that hands it only a stream and tensor pointers, where
// cudaMalloc is off limits on the decode thread (it can synchronise the whole
// device and stall every other stream), or a process whose device memory budget
// is fixed when it starts.  For them the per-request counters and the target
// argmax rows live in this fixed-size file-scope array instead of a
// caller-provided workspace.  Every GPU that loads the library holds it until
// the process exits.  All calls share it and it keeps the last call's contents:
// the counters are cleared by every call, and calls that overlap on the GPU
// (different streams, or different host threads) race on it.
constexpr int kNoAllocMaxRequests = 256;
constexpr int kNoAllocMaxPositions = 33;  // up to 32 drafts + the bonus row
// layout: counters [256] int32, argmax keys [256 x 33] u64, target rows [256 x 33] int32
constexpr size_t kNoAllocKeysOffset = kNoAllocMaxRequests * sizeof(int32_t);
constexpr size_t kNoAllocTargetsOffset =
    kNoAllocKeysOffset + static_cast<size_t>(kNoAllocMaxRequests) * kNoAllocMaxPositions * sizeof(unsigned long long);
static __device__ __align__(256) int32_t g_greedy_scratch[kNoAllocTargetsOffset / sizeof(int32_t) +
                                                          kNoAllocMaxRequests * kNoAllocMaxPositions];

// Device address of the scratch array on the current device.  In host code the
// symbol is only a host-side stand-in, so the address is looked up once per
// device (with that device current) and cached.
static int greedy_scratch(int32_t **out) {
    static std::mutex mu;
    static int32_t *address[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BD_ERR_DEVICE;
    std::lock_guard<std::mutex> lock(mu);
    if (!address[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_greedy_scratch) != cudaSuccess || !p) return BD_ERR_LAUNCH;
        address[dev] = static_cast<int32_t *>(p);
    }
    *out = address[dev];
    return BD_OK;
}

extern "C" int bd_accept_greedy_noalloc(const uint16_t *logits, int requests, int drafts, int64_t vocab,
                                        const int32_t *draft_tokens, const int32_t *eog, int n_eog,
                                        int32_t *accepted, int32_t *next_token, int32_t *targets, int32_t *flags,
                                        bd_stream_t stream) {
    if (requests < 0 || drafts < 0 || vocab < 1 || vocab > 0x7fffffff || n_eog < 0) return BD_ERR_INVALID;
    if (requests == 0) return BD_OK;
    if (!logits || (drafts > 0 && !draft_tokens) || (n_eog > 0 && !eog) || !accepted || !next_token)
        return BD_ERR_INVALID;
    if (requests > kNoAllocMaxRequests || drafts + 1 > kNoAllocMaxPositions) return BD_ERR_TOO_LARGE;
    int32_t *scratch = nullptr;
    if (int st = greedy_scratch(&scratch)) return st;
    const size_t rows = static_cast<size_t>(requests) * (drafts + 1);
    char *base = reinterpret_cast<char *>(scratch);
    // clear the counters and the keys this call uses (both are also left zero by every call)
    if (cudaMemsetAsync(base, 0, kNoAllocKeysOffset + rows * sizeof(unsigned long long), stream) != cudaSuccess)
        return BD_ERR_LAUNCH;
    GreedyArgs a{};
    a.logits = logits;
    a.rows = static_cast<int64_t>(rows);
    a.vocab = vocab;
    a.targets = targets ? targets : reinterpret_cast<int32_t *>(base + kNoAllocTargetsOffset);
    a.flags = flags;
    a.positions = drafts + 1;
    a.drafts = draft_tokens;
    a.eog = eog;
    a.n_eog = n_eog;
    a.accepted = accepted;
    a.next_token = next_token;
    a.counters = scratch;
    a.keys = reinterpret_cast<unsigned long long *>(base + kNoAllocKeysOffset);
    return launch_greedy_stream(a, stream);
}

extern "C" int bd_argmax_rows_bf16(const uint16_t *logits, int64_t rows, int64_t vocab, int32_t *out,
                                   int32_t *flags, bd_stream_t stream) {
    if (rows < 0 || vocab < 1 || vocab > 0x7fffffff) return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    if (!logits || !out) return BD_ERR_INVALID;
    GreedyArgs a{};
    a.logits = logits;
    a.rows = rows;
    a.vocab = vocab;
    a.targets = out;
    a.flags = flags;
    argmax_greedy_kernel<<<static_cast<unsigned>(rows), kArgmaxThreads, 0, stream>>>(a);
    BD_CHECK_LAUNCH();
    return BD_OK;
}
