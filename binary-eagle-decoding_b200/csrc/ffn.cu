// Decode-size (tokens <= 32) packed-sign projections on the integer tensor pipe.
//
// A CTA owns a rectangle of 512-byte sign units (row blocks x column pairs).
// Before waiting on the previous kernel (programmatic dependent launch) it
// streams its sign tiles -- read-only weights -- into shared memory with
// cp.async, together with the epilogue operands; after the wait it stages the
// activation codes (F8 B-fragment layout, frag_offset) for its column range.
// Warps then walk (row block, column pair) items: each lane expands its 16
// bytes of a unit into the 0/1 int8 A fragments of m16n8k32 MMAs (two
// instructions per register) and reads its B fragments with 16-byte shared
// loads.  With b in {0,1} (b = 1 for latent >= 0) the +-1 dot is
// D = 2 * D01 - sum(codes), exact in int32; partial sums meet in shared int32
// accumulators (order-free, exact), and the epilogue runs on all threads.
// Grids are sized on the host to a single wave of CTAs.
//
// Early-start invariant: before grid_wait() a kernel reads only weights and
// parameters; kernels call grid_launch_dependents() only after their own
// grid_wait(), so the kernel that started early can rely on every kernel
// before its predecessor having completed.  A kernel that writes sign tiles
// (the optimizer's re-pack) never triggers early starts.
#include <mutex>
#include <unordered_map>

#include "kernels.cuh"

namespace bd {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr size_t kSmemLimit = 220 * 1024;

// Stage `bytes` (multiple of 16) from global to shared with 16-byte cp.async.
__device__ __forceinline__ void stage(void *dst, const void *src, int64_t bytes) {
    char *d = static_cast<char *>(dst);
    const char *s = static_cast<const char *>(src);
    for (int64_t i = threadIdx.x * 16; i < bytes; i += kThreads * 16) cp_async16(d + i, s + i, 16);
}

// A fragments (0/1 bytes) of k-step q of chunk words (wa: row g, wb: row g + 8).
struct AFrag {
    uint32_t r[4];
    __device__ __forceinline__ AFrag(uint32_t wa, uint32_t wb, int q) {
        r[0] = (wa >> (2 * q)) & 0x01010101u;
        r[1] = (wb >> (2 * q)) & 0x01010101u;
        r[2] = (wa >> (2 * q + 1)) & 0x01010101u;
        r[3] = (wb >> (2 * q + 1)) & 0x01010101u;
    }
};

// Shape of one CTA's work, shared by both kernels.
struct Tile {
    int blocks;     // row blocks (pairs for gate/up) owned by this CTA
    int64_t block0; // first row block (pair)
    int cp0, ncpc;  // column-pair range [cp0, cp0 + ncpc)
};

// Shared-memory plan (byte offsets) of a CTA.
struct Plan {
    int M;          // matrices per block (2 for gate/up)
    int TP;         // padded tokens (8 NT)
    int planes;
    int64_t bits, codes, acc, params, sums, total;
    __host__ __device__ Plan(int m, int tp, int p, int blocks, int ncpc) : M(m), TP(tp), planes(p) {
        int64_t off = 0;
        bits = off;
        off += static_cast<int64_t>(blocks) * m * ncpc * 512;
        codes = off;
        off += static_cast<int64_t>(planes) * (tp / 8) * ncpc * 4 * 512;
        acc = off;
        off += static_cast<int64_t>(blocks) * m * 16 * tp * planes * 4;
        params = off;
        off += static_cast<int64_t>(blocks) * 16 * 5 * 4;
        sums = off;
        off += 2 * 32 * 4;
        total = off;
    }
};

// Per-item MMA: M matrices of row block `blk` at column pair `cp` (relative to
// the staged slice) against PLANES staged code planes.
template <int NT, int PLANES, int M>
__device__ __forceinline__ void item_mma(int (&acc)[M][PLANES][NT][4], const char *sm, const Plan &pl, int blk,
                                         int cpr, int ncpc, int lane) {
    uint4 w[M];
#pragma unroll
    for (int m = 0; m < M; ++m)
        w[m] = *reinterpret_cast<const uint4 *>(sm + pl.bits + ((blk * M + m) * ncpc + cpr) * 512 + lane * 16);
    const char *codes = sm + pl.codes;
    const int64_t plane_bytes = static_cast<int64_t>(NT) * ncpc * 4 * 512;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int qp = 0; qp < 2; ++qp) {
            const int sp = cpr * 4 + c * 2 + qp;
            uint4 b[PLANES][NT];
#pragma unroll
            for (int p = 0; p < PLANES; ++p)
#pragma unroll
                for (int nt = 0; nt < NT; ++nt)
                    b[p][nt] = *reinterpret_cast<const uint4 *>(codes + p * plane_bytes +
                                                                ((nt * ncpc * 4 + sp) * 32 + lane) * 16);
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {
                const int q = 2 * qp + qq;
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    const AFrag a(c ? w[m].z : w[m].x, c ? w[m].w : w[m].y, q);
#pragma unroll
                    for (int p = 0; p < PLANES; ++p)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
                            mma_s8_16832(acc[m][p][nt], a.r[0], a.r[1], a.r[2], a.r[3], qq ? b[p][nt].z : b[p][nt].x,
                                         qq ? b[p][nt].w : b[p][nt].y);
                }
            }
        }
    }
}

// Add a warp's register accumulators of block `blk` into the shared totals.
template <int NT, int PLANES, int M>
__device__ __forceinline__ void flush(int (&acc)[M][PLANES][NT][4], int *sacc, int blk, int lane) {
    const int g = lane >> 2, t = lane & 3;
    constexpr int TP = NT * 8;
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int p = 0; p < PLANES; ++p)
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int row = g + 8 * (i >> 1), token = n * 8 + 2 * t + (i & 1);
                    const int v = acc[m][p][n][i];
                    if (v) atomicAdd(sacc + (((blk * M + m) * PLANES + p) * 16 + row) * TP + token, v);
                    acc[m][p][n][i] = 0;
                }
}

// Walk this CTA's (block, column pair) items: warp w takes a contiguous share.
template <int NT, int PLANES, int M>
__device__ __forceinline__ void walk_items(const char *sm, int *sacc, const Plan &pl, const Tile &tile) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int items = tile.blocks * tile.ncpc;
    const int i0 = warp * items / kWarps, i1 = (warp + 1) * items / kWarps;
    int acc[M][PLANES][NT][4];
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int p = 0; p < PLANES; ++p)
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[m][p][n][i] = 0;
    int blk = i0 < i1 ? i0 / tile.ncpc : 0;
    for (int it = i0; it < i1; ++it) {
        const int b = it / tile.ncpc, cpr = it - b * tile.ncpc;
        if (b != blk) {
            flush<NT, PLANES, M>(acc, sacc, blk, lane);
            blk = b;
        }
        item_mma<NT, PLANES, M>(acc, sm, pl, b, cpr, tile.ncpc, lane);
    }
    if (i0 < i1) flush<NT, PLANES, M>(acc, sacc, blk, lane);
}

// Stage this CTA's sign tiles: for each owned block and matrix, ncpc contiguous units.
__device__ __forceinline__ void stage_bits(char *sm, const Plan &pl, const ProjArgs &a, const Tile &tile) {
    for (int b = 0; b < tile.blocks; ++b)
        for (int m = 0; m < pl.M; ++m) {
            const int64_t vrb = (tile.block0 + b) * pl.M + m;
            stage(sm + pl.bits + static_cast<int64_t>(b * pl.M + m) * tile.ncpc * 512,
                  a.bits + (vrb * a.ncp + tile.cp0) * 128, static_cast<int64_t>(tile.ncpc) * 512);
        }
}

// Stage the codes of columns [cp0, cp0 + ncpc) pairs for every n-tile and plane.
__device__ __forceinline__ void stage_codes(char *sm, const Plan &pl, const ProjArgs &a, const Tile &tile, int nt_count) {
    const int64_t nsp = a.ld / 64;
    for (int p = 0; p < pl.planes; ++p) {
        const int8_t *src = p ? a.codes1 : a.codes0;
        for (int nt = 0; nt < nt_count; ++nt)
            stage(sm + pl.codes + (static_cast<int64_t>(p) * nt_count + nt) * tile.ncpc * 4 * 512,
                  src + (nt * nsp + static_cast<int64_t>(tile.cp0) * 4) * 512, static_cast<int64_t>(tile.ncpc) * 4 * 512);
    }
}

// Exact +-1 dot from the 0/1 partial sums of all planes.
template <int PLANES>
__device__ __forceinline__ int pm_dot(int d0, int d1, int cs0, int cs1) {
    if (PLANES == 2) return 256 * (2 * d0 - cs0) + (2 * d1 - cs1);
    return 2 * d0 - cs0;
}

__device__ __forceinline__ int code_sum(const int32_t *sums, int nparts, int token) {
    int s = 0;
    for (int i = 0; i < nparts; ++i) s += sums[token * nparts + i];
    return s;
}

// --------------------------------------------------------------------------- gate/up pair kernel
template <int NT, int PLANES, int EPI>
__global__ void __launch_bounds__(kThreads) gateup_kernel(const ProjArgs a, int pairs_per_cta) {
    extern __shared__ __align__(16) char sm[];
    constexpr int TP = NT * 8;
    const int64_t npairs = (a.rows + 15) / 16;
    Tile tile;
    tile.block0 = static_cast<int64_t>(blockIdx.x) * pairs_per_cta;
    tile.blocks = static_cast<int>(min(static_cast<int64_t>(pairs_per_cta), npairs - tile.block0));
    tile.cp0 = 0;
    tile.ncpc = static_cast<int>(a.ncp);
    const Plan pl(2, TP, PLANES, pairs_per_cta, tile.ncpc);
    int *sacc = reinterpret_cast<int *>(sm + pl.acc);
    float *prm = reinterpret_cast<float *>(sm + pl.params);  // [5][pairs*16]: scale0 mid0 scale1 mid1 next_gain
    int *ssum = reinterpret_cast<int *>(sm + pl.sums);       // [2][32]: input code sums, next code sums

    // read-only operands first (weights and parameters)
    stage_bits(sm, pl, a, tile);
    const int rows_c = tile.blocks * 16;
    for (int i = threadIdx.x; i < rows_c; i += kThreads) {
        const int64_t o = tile.block0 * 16 + i;
        const bool live = o < a.rows;
        prm[0 * rows_c + i] = live ? __ldg(a.scale0 + o) : 0.0f;
        prm[1 * rows_c + i] = (live && a.mid0) ? __ldg(a.mid0 + o) : 0.0f;
        prm[2 * rows_c + i] = live ? __ldg(a.scale1 + o) : 0.0f;
        prm[3 * rows_c + i] = (live && a.mid1) ? __ldg(a.mid1 + o) : 0.0f;
        prm[4 * rows_c + i] = (live && a.next_gain) ? __ldg(a.next_gain + o) : 0.0f;
    }
    for (int i = threadIdx.x; i < tile.blocks * 2 * 16 * TP * PLANES; i += kThreads) sacc[i] = 0;
    grid_wait();
    grid_launch_dependents();
    stage_codes(sm, pl, a, tile, NT);
    if (threadIdx.x < 64) ssum[threadIdx.x] = 0;
    cp_async_wait_all();
    __syncthreads();
    if (threadIdx.x < TP) {
        ssum[threadIdx.x] = threadIdx.x < a.tokens ? code_sum(a.csum0, a.nparts, threadIdx.x) : 0;
        if (PLANES == 2) ssum[32 + threadIdx.x] = threadIdx.x < a.tokens ? code_sum(a.csum1, a.nparts, threadIdx.x) : 0;
    }
    walk_items<NT, PLANES, 2>(sm, sacc, pl, tile);
    __syncthreads();
    int lo_sum = 0, lo_token = -1;  // running per-token sum of the next projection's codes
    Quant qin, qnext;
    if (EPI == EPI_HE4) {
        qin.init(__ldg(a.bound), a.code_bits);
        qnext.init(__ldg(a.next_bound), 8);
    }
    // every thread owns (pair, token, row) elements, rows fastest
    const int elems = tile.blocks * TP * 16;  // (pair, token, row), rows fastest; TP is a constant
    bool bad = false;
    int *nsum = ssum + 32;  // next-code sums (HE4 only, where the second plane is unused)
    if (EPI == EPI_HE4 && threadIdx.x < 32) nsum[threadIdx.x] = 0;
    __syncthreads();
    for (int e = threadIdx.x; e < elems; e += kThreads) {
        const int row = e & 15;
        const int rest = e >> 4;
        const int token = rest % TP;
        const int b = rest / TP;
        const int64_t o = (tile.block0 + b) * 16 + row;
        if (o >= a.rows || token >= a.tokens) continue;
        const int r = b * 16 + row;
        const int cs0 = ssum[token];
        const int cs1 = PLANES == 2 ? ssum[32 + token] : 0;
        const int *g0 = sacc + (((b * 2 + 0) * PLANES + 0) * 16 + row) * TP + token;
        const int *u0 = sacc + (((b * 2 + 1) * PLANES + 0) * 16 + row) * TP + token;
        const int Dg = pm_dot<PLANES>(g0[0], PLANES == 2 ? g0[16 * TP] : 0, cs0, cs1);
        const int Du = pm_dot<PLANES>(u0[0], PLANES == 2 ? u0[16 * TP] : 0, cs0, cs1);
        float gv, uv;
        if (EPI == EPI_HE4) {
            gv = he4_value(Dg, prm[r], qin.step, cs0, prm[rows_c + r]);
            uv = he4_value(Du, prm[2 * rows_c + r], qin.step, cs0, prm[3 * rows_c + r]);
        } else if (EPI == EPI_W1) {
            const float rs = __ldg(a.row_scale + token);
            gv = __fmul_rn(__fmul_rn(static_cast<float>(Dg), rs), prm[r]);
            uv = __fmul_rn(__fmul_rn(static_cast<float>(Du), rs), prm[2 * rows_c + r]);
        } else {
            const float rs = __ldg(a.row_scale + token);
            gv = __fmul_rn(__fmul_rn(static_cast<float>(Dg), prm[r]), rs);
            uv = __fmul_rn(__fmul_rn(static_cast<float>(Du), prm[2 * rows_c + r]), rs);
        }
        const float h = __fmul_rn(silu(gv), uv);
        if (a.out) a.out[token * a.rows + o] = h;
        if (EPI == EPI_HE4) {
            const float gained = __fmul_rn(h, prm[4 * rows_c + r]);
            bad |= !isfinite(gained);
            const int code = qnext.code(gained);
            a.next_codes[frag_offset(token, o, a.next_ld / 64)] = static_cast<int8_t>(code);
            if (token != lo_token) {
                if (lo_token >= 0 && lo_sum) atomicAdd(nsum + lo_token, lo_sum);
                lo_token = token;
                lo_sum = 0;
            }
            lo_sum += code;
        }
    }
    if (EPI == EPI_HE4) {
        if (lo_token >= 0 && lo_sum) atomicAdd(nsum + lo_token, lo_sum);
        if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(a.flags, BD_FLAG_NONFINITE_INPUT);
        __syncthreads();
        if (threadIdx.x < a.tokens && nsum[threadIdx.x]) atomicAdd(a.next_csum + threadIdx.x, nsum[threadIdx.x]);
    }
}

// --------------------------------------------------------------------------- single-matrix kernel
template <int NT, int PLANES, int EPI>
__global__ void __launch_bounds__(kThreads) proj_kernel(const ProjArgs a, int blocks_per_cta) {
    extern __shared__ __align__(16) char sm[];
    __shared__ int last;
    constexpr int TP = NT * 8;
    const int64_t nrb = (a.rows + 15) / 16;
    const int ncp = static_cast<int>(a.ncp);
    Tile tile;
    tile.block0 = static_cast<int64_t>(blockIdx.x) * blocks_per_cta;
    tile.blocks = static_cast<int>(min(static_cast<int64_t>(blocks_per_cta), nrb - tile.block0));
    tile.cp0 = static_cast<int>(blockIdx.y) * ncp / a.kgroups;
    tile.ncpc = static_cast<int>(blockIdx.y + 1) * ncp / a.kgroups - tile.cp0;
    const int ncpc_max = (ncp + a.kgroups - 1) / a.kgroups;
    const Plan pl(1, TP, PLANES, blocks_per_cta, ncpc_max);
    int *sacc = reinterpret_cast<int *>(sm + pl.acc);
    float *prm = reinterpret_cast<float *>(sm + pl.params);  // [2][blocks*16]: scale0, mid0

    if (tile.ncpc > 0) stage_bits(sm, pl, a, tile);
    const int rows_c = tile.blocks * 16;
    for (int i = threadIdx.x; i < rows_c; i += kThreads) {
        const int64_t o = tile.block0 * 16 + i;
        const bool live = o < a.rows;
        prm[i] = live ? __ldg(a.scale0 + o) : 0.0f;
        prm[rows_c + i] = (live && a.mid0) ? __ldg(a.mid0 + o) : 0.0f;
    }
    for (int i = threadIdx.x; i < tile.blocks * 16 * TP * PLANES; i += kThreads) sacc[i] = 0;
    grid_wait();
    grid_launch_dependents();
    // The plan's regions are sized for ncpc_max; this CTA's slice (tile.ncpc,
    // possibly one pair shorter) is staged and walked with its own stride.
    if (tile.ncpc > 0) stage_codes(sm, pl, a, tile, NT);
    cp_async_wait_all();
    __syncthreads();
    if (tile.ncpc > 0) walk_items<NT, PLANES, 1>(sm, sacc, pl, tile);
    __syncthreads();
    const int elems = tile.blocks * 16 * TP * PLANES;  // accumulator cells of this CTA
    if (a.kgroups > 1) {
        const int64_t rows_pad = nrb * 16;
        for (int e = threadIdx.x; e < elems; e += kThreads) {
            const int token = e % TP;
            const int rest = e / TP;
            const int row = rest % 16;
            const int rest2 = rest / 16;
            const int p = rest2 % PLANES;
            const int b = rest2 / PLANES;
            const int v = sacc[e];
            if (v) atomicAdd(a.acc + (p * rows_pad + (tile.block0 + b) * 16 + row) * TP + token, v);
        }
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) last = atomicAdd(a.counters + blockIdx.x, 1) == a.kgroups - 1;
        __syncthreads();
        if (!last) return;
        __threadfence();
        for (int e = threadIdx.x; e < elems; e += kThreads) {
            const int token = e % TP;
            const int rest = e / TP;
            const int row = rest % 16;
            const int rest2 = rest / 16;
            const int p = rest2 % PLANES;
            const int b = rest2 / PLANES;
            sacc[e] = atomicExch(a.acc + (p * rows_pad + (tile.block0 + b) * 16 + row) * TP + token, 0);
        }
        if (threadIdx.x == 0) atomicExch(a.counters + blockIdx.x, 0);
        __syncthreads();
    }
    Quant qin;
    if (EPI == EPI_HE4) qin.init(__ldg(a.bound), a.code_bits);
    const int outs = tile.blocks * TP * 16;
    for (int e = threadIdx.x; e < outs; e += kThreads) {
        const int row = e & 15;
        const int rest = e >> 4;
        const int token = rest % TP;
        const int b = rest / TP;
        const int64_t o = (tile.block0 + b) * 16 + row;
        if (o >= a.rows || token >= a.tokens) continue;
        const int r = b * 16 + row;
        const int cs0 = code_sum(a.csum0, a.nparts, token);
        const int cs1 = PLANES == 2 ? code_sum(a.csum1, a.nparts, token) : 0;
        const int *c0 = sacc + ((b * PLANES + 0) * 16 + row) * TP + token;
        const int D = pm_dot<PLANES>(c0[0], PLANES == 2 ? c0[16 * TP] : 0, cs0, cs1);
        float y;
        if (EPI == EPI_HE4) {
            y = he4_value(D, prm[r], qin.step, cs0, prm[rows_c + r]);
        } else if (EPI == EPI_W1) {
            y = __fmul_rn(__fmul_rn(static_cast<float>(D), __ldg(a.row_scale + token)), prm[r]);
        } else {
            y = __fmul_rn(__fmul_rn(static_cast<float>(D), prm[r]), __ldg(a.row_scale + token));
        }
        if (a.residual) y = __fadd_rn(a.residual[token * a.rows + o], y);
        a.out[token * a.rows + o] = y;
        if (a.raw_dot) a.raw_dot[token * a.rows + o] = D;
    }
}

// --------------------------------------------------------------------------- launchers

static int sms_cached() {
    static int n = 0;
    if (!n) {
        int dev = 0, v = 0;
        if (cudaGetDevice(&dev) == cudaSuccess &&
            cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && v > 0)
            n = v;
        else
            n = 148;
    }
    return n;
}

// Resident CTAs per SM of `kern` with `smem` dynamic bytes (registers, threads
// and shared memory all counted by the occupancy calculator).
template <typename Kern>
static int ctas_per_sm(Kern kern, int64_t smem) {
    int n = 0;
    if (smem > static_cast<int64_t>(kSmemLimit)) return 0;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit)) !=
            cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, static_cast<size_t>(smem)) != cudaSuccess)
        return 0;
    return n;
}

// Launch plans depend only on (device, shape); the occupancy queries behind
// them cost microseconds each, so each launcher caches its plans.
struct PlanCache {
    std::mutex mu;
    std::unordered_map<uint64_t, uint64_t> plans;
    static uint64_t key(int64_t rows, int64_t ncp, bool split) {
        int dev = 0;
        cudaGetDevice(&dev);
        return (static_cast<uint64_t>(rows) << 24) ^ (static_cast<uint64_t>(ncp) << 4) ^
               (static_cast<uint64_t>(dev) << 1) ^ (split ? 1u : 0u);
    }
    bool get(uint64_t k, uint64_t &v) {
        std::lock_guard<std::mutex> g(mu);
        auto it = plans.find(k);
        if (it == plans.end()) return false;
        v = it->second;
        return true;
    }
    void put(uint64_t k, uint64_t v) {
        std::lock_guard<std::mutex> g(mu);
        plans[k] = v;
    }
};

template <int NT, int PLANES, int EPI>
static int launch_gateup_t(const ProjArgs &a, cudaStream_t stream) {
    const int64_t npairs = (a.rows + 15) / 16;
    const int sms = sms_cached();
    auto kern = gateup_kernel<NT, PLANES, EPI>;
    static PlanCache cache;
    const uint64_t key = PlanCache::key(a.rows, a.ncp, false);
    uint64_t cached = 0;
    int per = 0;
    if (cache.get(key, cached)) {
        per = static_cast<int>(cached);
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit)) !=
            cudaSuccess)
            return BD_ERR_LAUNCH;
    } else {
        // fewest pairs per CTA such that all CTAs are resident at once
        for (int p = 1; p <= 64; ++p) {
            const Plan pl(2, NT * 8, PLANES, p, static_cast<int>(a.ncp));
            const int occ = ctas_per_sm(kern, pl.total);
            if (occ == 0) break;
            per = p;
            if (static_cast<int64_t>(p) * occ * sms >= npairs) break;
        }
        if (per == 0) return BD_ERR_INVALID;
        cache.put(key, static_cast<uint64_t>(per));
    }
    const Plan pl(2, NT * 8, PLANES, per, static_cast<int>(a.ncp));
    const unsigned grid = static_cast<unsigned>((npairs + per - 1) / per);
    return launch_pdl(kern, dim3(grid), dim3(kThreads), static_cast<size_t>(pl.total), stream, a, per);
}

// Row blocks per CTA and K groups of a single-matrix projection: one resident
// wave, small CTAs, and a K split only where it buys parallelism (its global
// atomics and last-arriver epilogue cost time).
template <int NT, int PLANES, int EPI>
static int launch_proj_t(const ProjArgs &a0, cudaStream_t stream) {
    ProjArgs a = a0;
    const int64_t nrb = (a.rows + 15) / 16;
    const int sms = sms_cached();
    auto kern = proj_kernel<NT, PLANES, EPI>;
    int best_per = 0, best_kg = 1;
    double best_cost = 1e30;
    const int max_kg = a.acc && a.counters ? static_cast<int>(a.ncp) : 1;
    static PlanCache cache;
    const uint64_t key = PlanCache::key(a.rows, a.ncp, max_kg > 1);
    uint64_t cached = 0;
    const bool hit = cache.get(key, cached);
    if (hit) {
        best_per = static_cast<int>(cached >> 32);
        best_kg = static_cast<int>(cached & 0xffffffffu);
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemLimit)) !=
            cudaSuccess)
            return BD_ERR_LAUNCH;
    }
    for (int per = 1; per <= 16 && !hit; ++per) {
        for (int kg = 1; kg <= max_kg; ++kg) {
            const int ncpc = static_cast<int>((a.ncp + kg - 1) / kg);
            const Plan pl(1, NT * 8, PLANES, per, ncpc);
            const int occ = ctas_per_sm(kern, pl.total);
            if (occ == 0) continue;
            const int64_t ctas = (nrb + per - 1) / per * kg;
            const int64_t slots = static_cast<int64_t>(occ) * sms;
            const int64_t waves = (ctas + slots - 1) / slots;
            const double cost = waves * (per * ncpc + 6.0) + (kg > 1 ? 4.0 + 0.3 * per * kg : 0.0);
            if (cost < best_cost) {
                best_cost = cost;
                best_per = per;
                best_kg = kg;
            }
        }
    }
    if (best_per == 0) return BD_ERR_INVALID;
    if (!hit) cache.put(key, (static_cast<uint64_t>(best_per) << 32) | static_cast<uint64_t>(best_kg));
    a.blocks_per_cta = best_per;
    a.kgroups = best_kg;
    const int ncpc_max = static_cast<int>((a.ncp + a.kgroups - 1) / a.kgroups);
    const Plan pl(1, NT * 8, PLANES, best_per, ncpc_max);
    dim3 grid(static_cast<unsigned>((nrb + best_per - 1) / best_per), static_cast<unsigned>(a.kgroups));
    return launch_pdl(kern, grid, dim3(kThreads), static_cast<size_t>(pl.total), stream, a, best_per);
}

#define BD_DISPATCH_NT(fn, planes, epi)                                  \
    do {                                                                 \
        if (a.tokens <= 8) return fn<1, planes, epi>(a, stream);         \
        if (a.tokens <= 16) return fn<2, planes, epi>(a, stream);        \
        if (a.tokens <= 24) return fn<3, planes, epi>(a, stream);        \
        return fn<4, planes, epi>(a, stream);                            \
    } while (0)

int launch_gateup(const ProjArgs &a, int epi, cudaStream_t stream) {
    if (a.tokens < 1 || a.tokens > 32 || a.nparts < 1) return BD_ERR_INVALID;
    if (epi == EPI_HE4) BD_DISPATCH_NT(launch_gateup_t, 1, EPI_HE4);
    if (epi == EPI_W1) BD_DISPATCH_NT(launch_gateup_t, 2, EPI_W1);
    BD_DISPATCH_NT(launch_gateup_t, 1, EPI_W1A1);
}

int launch_proj(const ProjArgs &a, int epi, cudaStream_t stream) {
    if (a.tokens < 1 || a.tokens > 32 || a.nparts < 1) return BD_ERR_INVALID;
    if (epi == EPI_HE4) BD_DISPATCH_NT(launch_proj_t, 1, EPI_HE4);
    if (epi == EPI_W1) BD_DISPATCH_NT(launch_proj_t, 2, EPI_W1);
    BD_DISPATCH_NT(launch_proj_t, 1, EPI_W1A1);
}

// Kept for the callers' sake: the launcher plans the grid itself.
void plan_proj(ProjArgs &a, int) {
    a.kgroups = 1;
    a.blocks_per_cta = 1;
}

}  // namespace bd
