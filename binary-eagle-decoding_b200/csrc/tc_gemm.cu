// Large-M projections on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
//
// D[tokens x outs] = codes[tokens x K] . signs[outs x K]^T with int8 operands: codes are
// the quantizer's integers (HE4 A4/A8) or +-1 (W1A1), signs are +-1 (an "I8" copy of
// the latent signs, expanded once per latent version), so D is the exact +-1 dot in
// int32 (kind::i8, s32 accumulators) -- bit-identical to the reference's fp32
// linear of integers.  Both operands are 128-byte-swizzled K-major tiles loaded by
// TMA, each CTA loading its own tiles; K and the token / out edges beyond the tensors read as zeros.
//
// Persistent, warp-specialised CTA (one per SM): warp 0 issues TMA loads into a
// 4-stage ring, warp 1 owns TMEM (two accumulator buffers of BN columns) and issues
// tcgen05.mma (M = 128 tokens, N = BN outs, K = 32 per instruction) from one lane,
// warps 2-9 drain an accumulator with tcgen05.ld (warp w reads TMEM lanes
// 32 (w % 4) .., one half of the columns) and apply the fused epilogue while the next tile accumulates in
// the other buffer.  Every mbarrier wait is bounded; a timeout raises
// BD_FLAG_TIMEOUT and sets a CTA-wide abort flag that ends every role's loop.
// Before the CTA frees its TMEM and exits, the producer waits (bounded again)
// for the TMA loads it already issued to land in shared memory, and the MMA
// issuer commits its issued MMAs to a drain barrier and waits for that; if
// either of those waits also runs out, the tile data is lost (the flag already
// reports the failure) and the CTA exits anyway rather than hang.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "kernels.cuh"

namespace bd {

constexpr int kTcBM = 128, kTcBK = 128, kTcStages = 4;
constexpr uint32_t kTcSpin = 1u << 21;

enum TcEpi : int {
    TC_RAW = 0,           // out_i32 = D
    TC_HE4 = 1,           // y = he4_value(D, scale[o], step, sums[t], mid[o]) (+ residual)
    TC_W1A1 = 2,          // y = (D * scale[o]) * rs[t]
    TC_W1A1_SWIGLU = 3,   // N tile = 128 gate + 128 up rows: h = silu(gate) * up, W1A1 values
    TC_F32 = 4,           // bf16 operands (kind::f16), fp32 accumulators: out = D
    TC_STE = 5,           // bf16 operands: out = (D * step) * 1[|latent| <= window] (+ per-warp partial sums)
    TC_CE_STATS = 6,      // bf16 operands, D = logits: per (row, 128-column half tile) max and sum of exp; target logit
    TC_CE_GRAD = 7,       // bf16 operands, D = logits: dl = w * (exp(D - lse) - onehot) as bf16 hi + lo halves
};

// K elements per 128-byte shared-memory row (one TMA box width) of the operand type.
__host__ __device__ constexpr int tc_bf16(int epi) {
    return epi == TC_F32 || epi == TC_STE || epi == TC_CE_STATS || epi == TC_CE_GRAD;
}
__host__ __device__ constexpr int tc_bk(int epi) { return tc_bf16(epi) ? 64 : 128; }

struct TcArgs {
    int64_t M, N, K;       // tokens, outs (as the reference sees them), reduction length
    int64_t n_tiles;       // BN-column tiles of the (possibly interleaved) weight rows
    int64_t m_tiles;
    int64_t ld_out;        // output row stride (elements)
    const float *scale, *scale2, *mid, *bound, *row_scale, *residual;
    const int32_t *sums;
    int code_bits;
    float *out;
    int32_t *out_i32;
    int32_t *flags;
    int parts;              // bf16 kinds: the product is a sum of 1-3 (A, B) operand pairs (split-bf16
                            // halves), each a full K reduction, issued as one reduction of parts x K
    float *out_dot;         // TC_HE4: the exact integer dot as fp32 as well (optional)
    // TC_STE: the straight-through sign gradient of the latent [M][N] (row stride ld_latent)
    const float *latent;
    int64_t ld_latent;
    const float *window;    // learned window (device scalar) or null: window_value
    float window_value;
    float *partials;        // optional [tiles][8 warps][2]: sum of out^2, sum over |w| > window of D * step * sign(w)
    // TC_CE_STATS / TC_CE_GRAD (rows = labelled positions, columns = vocabulary)
    const int32_t *labels;  // [M]
    const float *row_w;     // [M] label weights (GRAD)
    const float *row_lse;   // [M] log-sum-exp of each row (GRAD)
    float *stats;           // [M][2 n_tiles][2]: max, sum of exp(D - max) per half tile (STATS)
    float *target;          // [M] the label's logit (STATS)
    __nv_bfloat16 *dl_hi, *dl_lo;  // [M][ld_out] (GRAD)
    // TC_F32 split over K: tiles [0, split_full) are whole units; each later tile is
    // `splits` units of one K slice each (the tiles of a last, partial wave, or all
    // of them when they are fewer than the SMs).  A sliced unit writes its fp32
    // partial tile, and per (tile, epilogue warp) the last slice to arrive adds them
    // in slice order (deterministic) into out.
    int splits;
    int64_t split_full;
    float *split_part;      // [tiles][splits][kTcBM][BN]
    int32_t *split_count;   // [tiles][8] at the start of the workspace, zero on entry and left zero
    void *split_ws;         // caller's workspace for the above (host side only), or null: no split
    size_t split_ws_bytes;
};

// K slices per tile of a TC_F32 product: the count that minimises the
// waves of (tile, slice) units per full-K tile time, plus 5 % of a tile time per
// slice for writing and adding the partial tiles; at least 4 k-blocks per slice,
// at most 8 slices, and the partial tiles within half of L2.
// The counters sit at a fixed place (the first kTcSplitCounts words) whatever the
// shape, so that a workspace shared by products of different shapes never sees an
// earlier call's partial sums where this call keeps its counters.
constexpr int64_t kTcSplitCounts = 2048;  // 8 per tile: up to 256 split tiles

static int tc_split_slices(int64_t tiles, int64_t nk, int sms) {
    if (tiles * 8 > kTcSplitCounts) return 1;
    int best = 1;
    double best_cost = static_cast<double>((tiles + sms - 1) / sms) + 0.05;
    for (int s = 2; s <= 8 && s <= nk / 4; ++s) {
        if (static_cast<double>(tiles) * s * kTcBM * 256 * sizeof(float) > 64.0 * (1 << 20)) break;
        const double cost = static_cast<double>((tiles * s + sms - 1) / sms) / s + 0.05 * s;
        if (cost < best_cost - 1e-9) {
            best = s;
            best_cost = cost;
        }
    }
    return best;
}
static size_t tc_split_bytes(int64_t tiles, int slices, int bn) {
    return kTcSplitCounts * sizeof(int32_t) + static_cast<size_t>(tiles) * slices * kTcBM * bn * sizeof(float);
}

// Which tiles are cut into how many K slices: with fewer tiles than SMs, all of
// them (tc_split_slices).  With more, none: cutting only the tiles of a last,
// partial wave (the kernel supports it: tiles [0, full) whole) measured 2 % faster
// at 320 tiles, no faster at 160 and 18 % slower at 512, so it is not used.
static void tc_split_plan(int64_t tiles, int64_t nk, int sms, int64_t &full, int &slices) {
    full = tiles;
    slices = 1;
    if (tiles < sms) {
        slices = tc_split_slices(tiles, nk, sms);
        if (slices > 1) full = 0;
    }
}

__device__ __forceinline__ uint32_t su32(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mb_init(uint64_t *b, uint32_t n) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(b)), "r"(n));
}
__device__ __forceinline__ void mb_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mb_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(b)) : "memory");
}
// Bounded parity wait: false after kTcSpin polls or once the CTA aborted.
__device__ __forceinline__ bool mb_wait(uint64_t *b, uint32_t parity, volatile int *abort) {
    for (uint32_t i = 0; i < kTcSpin; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(su32(b)), "r"(parity)
            : "memory");
        if (ok) return true;
        if ((i & 1023) == 1023 && *abort) return false;
    }
    *abort = 1;
    return false;
}
// Bounded wait used on the abort path only (ignores the abort flag).
__device__ __forceinline__ void mb_drain(uint64_t *b, uint32_t parity) {
    for (uint32_t i = 0; i < kTcSpin; ++i) {
        uint32_t ok;
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(su32(b)), "r"(parity)
            : "memory");
        if (ok) return;
    }
}
__device__ __forceinline__ void tma_2d(void *dst, const CUtensorMap *map, uint64_t *bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            su32(dst)),
        "l"(map), "r"(su32(bar)), "r"(c0), "r"(c1)
        : "memory");
}
// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t sdesc(const void *p) {
    const uint64_t a = su32(p);
    return ((a >> 4) & 0x3FFFull) | (1ull << 16) | (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}
// Instruction descriptor, kind::f16: f32 accumulators, bf16 A and B, K-major, N, M = 128.
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(kTcBM >> 4) << 24);
}
// Instruction descriptor, kind::i8: s32 accumulators, signed A and B, K-major, N, M = 128.
__host__ __device__ constexpr uint32_t idesc_i8(int n) {
    return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(kTcBM >> 4) << 24);
}

template <int BN, int EPI>
__global__ void __launch_bounds__(320, 1) tc_gemm_kernel(const TcArgs a, const __grid_constant__ CUtensorMap ma,
                                                         const __grid_constant__ CUtensorMap mb,
                                                         const __grid_constant__ CUtensorMap ma2,
                                                         const __grid_constant__ CUtensorMap mb2,
                                                         const __grid_constant__ CUtensorMap ma3,
                                                         const __grid_constant__ CUtensorMap mb3) {
    extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sa = smem;                                // stages x 16 KB (tokens)
    uint8_t *sb = smem + kTcStages * kTcBM * kTcBK;    // stages x BN x 128 B (weights)
    __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], acc_full[2], acc_empty[2], drain;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t tiles = a.m_tiles * a.n_tiles;
    constexpr int BKE = tc_bk(EPI);  // K elements per stage
    const int nk1 = static_cast<int>((a.K + BKE - 1) / BKE);
    const int nk = nk1 * (a.parts > 1 ? a.parts : 1);  // part p covers k-blocks [p nk1, (p + 1) nk1)
    const int S = (EPI == TC_F32 && a.splits > 1) ? a.splits : 1;  // K slices of a sliced tile (at most nk)
    const int64_t whole = S > 1 ? a.split_full : tiles;              // tiles done whole
    const int64_t units = whole + (tiles - whole) * S;
    // unit -> (tile, K slice, slices of that tile)
    auto unit_of = [&](int64_t u, int64_t &t, int &sp, int &us) {
        if (u < whole) {
            t = u;
            sp = 0;
            us = 1;
        } else {
            const int64_t v = u - whole;
            t = whole + v / S;
            sp = static_cast<int>(v % S);
            us = S;
        }
    };
    constexpr uint32_t kCols = 2 * BN;  // two accumulator buffers
    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            mb_init(&full[s], 1);
            mb_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mb_init(&acc_full[b], 1);
            mb_init(&acc_empty[b], 8);  // one arrive per epilogue warp
        }
        mb_init(&drain, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                     "n"(kCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            uint32_t it = 0;
            for (int64_t u = blockIdx.x; u < units && !abort_flag; u += gridDim.x) {
                int64_t t;
                int sp, us;
                unit_of(u, t, sp, us);
                const int m0 = static_cast<int>((t % a.m_tiles) * kTcBM);
                const int n0 = static_cast<int>((t / a.m_tiles) * BN);
                const int kb = sp * nk / us, ke = (sp + 1) * nk / us;
                for (int k = kb; k < ke; ++k, ++it) {
                    const int s = it % kTcStages;
                    if (it >= kTcStages && !mb_wait(&empty[s], ((it / kTcStages) - 1) & 1, &abort_flag)) break;
                    mb_expect_tx(&full[s], (kTcBM + BN) * kTcBK);
                    const int part = k / nk1, kc = k - part * nk1;
                    tma_2d(sa + s * kTcBM * kTcBK, part == 0 ? &ma : (part == 1 ? &ma2 : &ma3), &full[s], kc * BKE, m0);
                    tma_2d(sb + s * BN * kTcBK, part == 0 ? &mb : (part == 1 ? &mb2 : &mb3), &full[s], kc * BKE, n0);
                }
            }
            if (abort_flag) {  // let the loads already issued (stages it - S .. it - 1) land
                for (uint32_t j = it > static_cast<uint32_t>(kTcStages) ? it - kTcStages : 0; j < it; ++j)
                    mb_drain(&full[j % kTcStages], (j / kTcStages) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = tc_bf16(EPI) ? idesc_bf16(BN) : idesc_i8(BN);
            uint32_t it = 0, lt = 0;
            for (int64_t u = blockIdx.x; u < units && !abort_flag; u += gridDim.x, ++lt) {
                const uint32_t b = lt & 1;
                if (!mb_wait(&acc_empty[b], ((lt >> 1) & 1) ^ 1, &abort_flag)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t d = tmem + b * BN;
                bool ok = true;
                int64_t t;
                int sp, us;
                unit_of(u, t, sp, us);
                const int kb = sp * nk / us, ke = (sp + 1) * nk / us;
                for (int k = kb; k < ke; ++k, ++it) {
                    const int s = it % kTcStages;
                    if (!mb_wait(&full[s], (it / kTcStages) & 1, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint64_t da = sdesc(sa + s * kTcBM * kTcBK), db = sdesc(sb + s * BN * kTcBK);
#pragma unroll
                    for (int kk = 0; kk < kTcBK / 32; ++kk) {
                        const uint32_t accumulate = (k > kb || kk > 0) ? 1u : 0u;
                        // one instruction consumes 32 bytes of K (32 int8 or 16 bf16): descriptor +2
                        if (tc_bf16(EPI))
                            asm volatile(
                                "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
                                " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
                                "l"(da + static_cast<uint64_t>(2 * kk)), "l"(db + static_cast<uint64_t>(2 * kk)),
                                "r"(idesc), "r"(accumulate));
                        else
                            asm volatile(
                                "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
                                " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
                                "l"(da + static_cast<uint64_t>(2 * kk)), "l"(db + static_cast<uint64_t>(2 * kk)),
                                "r"(idesc), "r"(accumulate));
                    }
                    asm volatile(
                        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(&empty[s]))
                        : "memory");
                }
                asm volatile(
                    "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(&acc_full[b]))
                    : "memory");
                if (!ok) break;
            }
            if (abort_flag) {  // every MMA this thread issued completes before TMEM is freed
                asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 su32(&drain))
                             : "memory");
                mb_drain(&drain, 0);
            }
        }
    } else {  // epilogue warps 2..9: warp w drains TMEM lanes 32 (w % 4) .., column half (w - 2) / 4
        const int quarter = warp & 3, half = (warp - 2) >> 2;
        const int row_in_tile = quarter * 32 + lane;
        Quant q;
        if (EPI == TC_HE4 || (EPI == TC_STE && a.bound)) q.init(__ldg(a.bound), a.code_bits);
        const float ste_step = (EPI == TC_STE && a.bound) ? q.step : 1.0f;
        const float ste_window = EPI == TC_STE ? (a.window ? __ldg(a.window) : a.window_value) : 0.0f;
        constexpr int OUT_COLS = EPI == TC_W1A1_SWIGLU ? BN / 2 : BN;
        constexpr int HALF = OUT_COLS / 2;
        const bool vec_out = (a.ld_out & 3) == 0 && (reinterpret_cast<uintptr_t>(EPI == TC_RAW ? static_cast<void *>(a.out_i32)
                                                                                               : static_cast<void *>(a.out)) & 15) == 0;
        uint32_t lt = 0;
        for (int64_t u = blockIdx.x; u < units && !abort_flag; u += gridDim.x, ++lt) {
            int64_t t;
            int sp, us;
            unit_of(u, t, sp, us);
            const int64_t tt = t - whole;  // index among the sliced tiles
            // this unit's partial tile (split K): rows of this thread, its half of the columns
            float *part = us > 1 ? a.split_part + ((tt * S + sp) * kTcBM + row_in_tile) * BN + half * HALF : nullptr;
            const uint32_t b = lt & 1;
            if (!mb_wait(&acc_full[b], (lt >> 1) & 1, &abort_flag)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int64_t row = (t % a.m_tiles) * kTcBM + row_in_tile;
            const bool live_row = row < a.M;
            const float rs = (EPI == TC_W1A1 || EPI == TC_W1A1_SWIGLU) && live_row ? __ldg(a.row_scale + row) : 0.0f;
            const int cs = (EPI == TC_HE4 && live_row) ? __ldg(a.sums + row) : 0;
            // in the SwiGLU tile, columns [0, BN/2) are gate rows and [BN/2, BN) the up rows of
            // the same outputs (128-row blocks interleaved in the weight copy)
            const int64_t o_base = (EPI == TC_W1A1_SWIGLU ? (t / a.m_tiles) * (BN / 2) : (t / a.m_tiles) * BN) + half * HALF;
            float ss = 0.0f, sc = 0.0f;  // TC_STE partial sums of this thread, in column order
            const bool ce = EPI == TC_CE_STATS || EPI == TC_CE_GRAD;
            const int label = ce && live_row ? __ldg(a.labels + row) : -1;
            const float rw = EPI == TC_CE_GRAD && live_row ? __ldg(a.row_w + row) : 0.0f;
            const float lse = EPI == TC_CE_GRAD && live_row ? __ldg(a.row_lse + row) : 0.0f;
            float run_max = -INFINITY, run_sum = 0.0f;  // TC_CE_STATS, over this thread's half tile
            for (int c = 0; c < HALF; c += 16) {
                uint32_t v[16], u[16];
                const uint32_t taddr = tmem + b * BN + (static_cast<uint32_t>(quarter * 32) << 16) + half * HALF + c;
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                    : "r"(taddr));
                if (EPI == TC_W1A1_SWIGLU) {
                    asm volatile(
                        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                        : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
                          "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]),
                          "=r"(u[15])
                        : "r"(taddr + BN / 2));
                }
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                const int64_t o0 = o_base + c;
                if (!live_row || o0 >= a.N) continue;
                const bool full16 = o0 + 16 <= a.N;
                // per-column parameters: the same 16 values for every lane (broadcast loads)
                float s1[16], s2[16], md[16];
                if (EPI != TC_RAW && EPI != TC_F32 && EPI != TC_STE && EPI != TC_CE_STATS && EPI != TC_CE_GRAD) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const bool live = full16 || o0 + j < a.N;
                        s1[j] = live ? __ldg(a.scale + o0 + j) : 0.0f;
                        s2[j] = (EPI == TC_W1A1_SWIGLU && live) ? __ldg(a.scale2 + o0 + j) : 0.0f;
                        md[j] = (EPI == TC_HE4 && live) ? __ldg(a.mid + o0 + j) : 0.0f;
                    }
                }
                float y[16];
                int32_t di[16];
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int D = static_cast<int>(v[j]);
                    di[j] = D;
                    if (EPI == TC_F32) {
                        y[j] = __uint_as_float(v[j]);
                    } else if (EPI == TC_STE) {
                        y[j] = __fmul_rn(__uint_as_float(v[j]), ste_step);
                    } else if (EPI == TC_HE4) {
                        y[j] = he4_value(D, s1[j], q.step, cs, md[j]);
                    } else if (EPI == TC_W1A1) {
                        y[j] = __fmul_rn(__fmul_rn(static_cast<float>(D), s1[j]), rs);
                    } else if (EPI == TC_W1A1_SWIGLU) {
                        const float gv = __fmul_rn(__fmul_rn(static_cast<float>(D), s1[j]), rs);
                        const float uv = __fmul_rn(__fmul_rn(static_cast<float>(static_cast<int>(u[j])), s2[j]), rs);
                        y[j] = __fmul_rn(silu(gv), uv);
                    }
                }
                const int64_t idx = row * a.ld_out + o0;
                if (EPI == TC_F32 && us > 1) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        *reinterpret_cast<float4 *>(part + c + j) = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
                    continue;
                }
                if (EPI == TC_CE_STATS) {
                    // online max and sum of exp over the live columns of this chunk
                    float cmax = -INFINITY;
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (full16 || o0 + j < a.N) cmax = fmaxf(cmax, __uint_as_float(v[j]));
                    const float m = fmaxf(run_max, cmax);
                    float sum = run_max == -INFINITY ? 0.0f : run_sum * exp2f((run_max - m) * 1.4426950408889634f);
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (full16 || o0 + j < a.N) sum += exp2f((__uint_as_float(v[j]) - m) * 1.4426950408889634f);
                    run_max = m;
                    run_sum = sum;
                    if (label >= o0 && label < o0 + 16) a.target[row] = __uint_as_float(v[label - o0]);
                    continue;
                }
                if (EPI == TC_CE_GRAD) {
                    uint32_t hp[8] = {}, lp[8] = {};  // bf16 pairs, column 2 i in the low half
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const float p = exp2f((__uint_as_float(v[j]) - lse) * 1.4426950408889634f);
                        const float d = __fmul_rn(rw, o0 + j == label ? __fsub_rn(p, 1.0f) : p);
                        const __nv_bfloat16 h = __float2bfloat16_rn(d);
                        const __nv_bfloat16 l = __float2bfloat16_rn(__fsub_rn(d, __bfloat162float(h)));
                        hp[j >> 1] |= static_cast<uint32_t>(__bfloat16_as_ushort(h)) << (16 * (j & 1));
                        lp[j >> 1] |= static_cast<uint32_t>(__bfloat16_as_ushort(l)) << (16 * (j & 1));
                    }
                    if (full16 && (a.ld_out & 7) == 0) {
                        uint4 *ph = reinterpret_cast<uint4 *>(a.dl_hi + idx), *pl = reinterpret_cast<uint4 *>(a.dl_lo + idx);
                        ph[0] = make_uint4(hp[0], hp[1], hp[2], hp[3]);
                        ph[1] = make_uint4(hp[4], hp[5], hp[6], hp[7]);
                        pl[0] = make_uint4(lp[0], lp[1], lp[2], lp[3]);
                        pl[1] = make_uint4(lp[4], lp[5], lp[6], lp[7]);
                    } else {
                        uint16_t *qh = reinterpret_cast<uint16_t *>(a.dl_hi + idx);
                        uint16_t *ql = reinterpret_cast<uint16_t *>(a.dl_lo + idx);
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (o0 + j < a.N) {
                                qh[j] = static_cast<uint16_t>(hp[j >> 1] >> (16 * (j & 1)));
                                ql[j] = static_cast<uint16_t>(lp[j >> 1] >> (16 * (j & 1)));
                            }
                    }
                    continue;
                }
                if (EPI == TC_STE) {
                    // mask by the straight-through window; the two sums the update needs
                    const float *lat = a.latent + row * a.ld_latent + o0;
                    float wl[16];
                    if (full16 && (a.ld_latent & 3) == 0 && (reinterpret_cast<uintptr_t>(a.latent) & 15) == 0) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4) {
                            const float4 q4 = __ldg(reinterpret_cast<const float4 *>(lat + j));
                            wl[j] = q4.x;
                            wl[j + 1] = q4.y;
                            wl[j + 2] = q4.z;
                            wl[j + 3] = q4.w;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j) wl[j] = (full16 || o0 + j < a.N) ? __ldg(lat + j) : 0.0f;
                    }
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        if (!(full16 || o0 + j < a.N)) continue;
                        const float w = wl[j];
                        const bool inside = fabsf(w) <= ste_window;
                        if (!inside) sc = __fadd_rn(sc, w >= 0.0f ? y[j] : -y[j]);
                        y[j] = inside ? y[j] : 0.0f;
                        ss = __fadd_rn(ss, __fmul_rn(y[j], y[j]));
                    }
                }
                if (EPI == TC_HE4 && a.out_dot) {
                    if (full16 && vec_out && (reinterpret_cast<uintptr_t>(a.out_dot) & 15) == 0) {
#pragma unroll
                        for (int j = 0; j < 16; j += 4)
                            *reinterpret_cast<float4 *>(a.out_dot + idx + j) =
                                make_float4(static_cast<float>(di[j]), static_cast<float>(di[j + 1]),
                                            static_cast<float>(di[j + 2]), static_cast<float>(di[j + 3]));
                    } else {
#pragma unroll
                        for (int j = 0; j < 16; ++j)
                            if (full16 || o0 + j < a.N) a.out_dot[idx + j] = static_cast<float>(di[j]);
                    }
                }
                if (EPI == TC_HE4 && a.residual) {
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        if (full16 || o0 + j < a.N) y[j] = __fadd_rn(a.residual[idx + j], y[j]);
                }
                if (full16 && vec_out) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4) {
                        if (EPI == TC_RAW)
                            *reinterpret_cast<int4 *>(a.out_i32 + idx + j) = make_int4(di[j], di[j + 1], di[j + 2], di[j + 3]);
                        else
                            *reinterpret_cast<float4 *>(a.out + idx + j) = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
                    }
                } else {
                    for (int j = 0; j < 16 && o0 + j < a.N; ++j) {
                        if (EPI == TC_RAW)
                            a.out_i32[idx + j] = di[j];
                        else
                            a.out[idx + j] = y[j];
                    }
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mb_arrive(&acc_empty[b]);
            if (EPI == TC_F32 && us > 1) {
                // the last split of this (tile, warp region) to arrive sums the partials in slice
                // order; no thread waits on another CTA
                __threadfence();
                __syncwarp();
                int old = 0;
                int32_t *count = a.split_count + tt * 8 + (warp - 2);
                if (lane == 0) old = atomicAdd(count, 1);
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old == S - 1) {
                    __threadfence();
                    const float *p0 = a.split_part + (tt * S * kTcBM + row_in_tile) * BN + half * HALF;
                    for (int c = 0; c < HALF && live_row; c += 16) {
                        const int64_t o0 = o_base + c;
                        if (o0 >= a.N) break;
                        float y[16];
#pragma unroll
                        for (int j = 0; j < 16; ++j) y[j] = 0.0f;
                        for (int s = 0; s < S; ++s) {
                            const float *src = p0 + static_cast<int64_t>(s) * kTcBM * BN + c;
#pragma unroll
                            for (int j = 0; j < 16; j += 4) {
                                const float4 v4 = __ldcg(reinterpret_cast<const float4 *>(src + j));
                                y[j] = __fadd_rn(y[j], v4.x);
                                y[j + 1] = __fadd_rn(y[j + 1], v4.y);
                                y[j + 2] = __fadd_rn(y[j + 2], v4.z);
                                y[j + 3] = __fadd_rn(y[j + 3], v4.w);
                            }
                        }
                        const int64_t idx = row * a.ld_out + o0;
                        if (o0 + 16 <= a.N && vec_out) {
#pragma unroll
                            for (int j = 0; j < 16; j += 4)
                                *reinterpret_cast<float4 *>(a.out + idx + j) = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
                        } else {
                            for (int j = 0; j < 16 && o0 + j < a.N; ++j) a.out[idx + j] = y[j];
                        }
                    }
                    if (lane == 0) *count = 0;
                }
            }
            if (EPI == TC_CE_STATS && live_row) {
                float *st = a.stats + (row * (2 * a.n_tiles) + (t / a.m_tiles) * 2 + half) * 2;
                st[0] = run_max;
                st[1] = run_sum;
            }
            if (EPI == TC_STE && a.partials) {  // fixed butterfly: deterministic per (tile, warp)
#pragma unroll
                for (int d = 16; d > 0; d >>= 1) {
                    ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, d));
                    sc = __fadd_rn(sc, __shfl_xor_sync(0xffffffffu, sc, d));
                }
                if (lane == 0) {
                    a.partials[(t * 8 + (warp - 2)) * 2 + 0] = ss;
                    a.partials[(t * 8 + (warp - 2)) * 2 + 1] = sc;
                }
            }
        }
    }
    if (abort_flag && threadIdx.x == 0) set_flag(a.flags, BD_FLAG_TIMEOUT);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(kCols));
    }
}

// ------------------------------------------------------------------ SM pairs (TC_F32)
// A cluster of two CTAs computes a 256 x 256 output tile with tcgen05.mma.cta_group::2:
// CTA r of the pair loads rows [128 r, 128 r + 128) of the tile's A and of its B (its
// half of the 256 output columns) into its own shared memory; the even CTA issues the
// MMAs, which read both CTAs' halves and leave each CTA's 128 rows x 256 columns of
// accumulators in its own TMEM.  A stage is 32 KB per CTA instead of 48 KB, so six
// stages fit: twice the MACs in flight of the single-CTA kernel.  Both CTAs' TMA loads
// complete on the even CTA's full barrier (which expects both halves); the MMA
// commits arrive on both CTAs' empty and accumulator barriers; both CTAs' epilogue
// warps arrive on the even CTA's accumulator-empty barrier.  Every wait is bounded.
constexpr int kPairStages = 6;

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// The even CTA's copy of a shared-memory object of this CTA (same offset).
__device__ __forceinline__ uint32_t even_cta_addr(const void *p) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(out) : "r"(su32(p)));
    return out;
}
__device__ __forceinline__ void cluster_sync_pair() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_2d_pair(void *dst, const CUtensorMap *map, uint32_t bar_even, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4}], [%2];" ::"r"(su32(dst)),
        "l"(map), "r"(bar_even), "r"(c0), "r"(c1)
        : "memory");
}
// Instruction descriptor, kind::f16, bf16 operands, f32 accumulators, K-major, M = 256 (a pair), N.
__host__ __device__ constexpr uint32_t idesc_bf16_pair(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (256u >> 4 << 24);
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(320, 1)
    tc_pair_kernel(const TcArgs a, const __grid_constant__ CUtensorMap ma, const __grid_constant__ CUtensorMap mb,
                   const __grid_constant__ CUtensorMap ma2, const __grid_constant__ CUtensorMap mb2,
                   const __grid_constant__ CUtensorMap ma3, const __grid_constant__ CUtensorMap mb3) {
    constexpr int BN = 256, HALF_ROWS = 128;
    constexpr uint32_t kStageBytes = (HALF_ROWS + HALF_ROWS) * kTcBK;  // this CTA's A and B halves
    extern __shared__ __align__(1024) uint8_t tc_smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(tc_smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sa = smem;                                   // stages x 16 KB: A rows of this CTA
    uint8_t *sb = smem + kPairStages * HALF_ROWS * kTcBK;  // stages x 16 KB: B rows of this CTA
    __shared__ __align__(8) uint64_t full[kPairStages], empty[kPairStages], acc_full[2], acc_empty[2], drain;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int64_t pair = blockIdx.x >> 1, pairs = gridDim.x >> 1;
    const int64_t pm = (a.M + 2 * HALF_ROWS - 1) / (2 * HALF_ROWS);  // 256-row tiles
    const int64_t tiles = pm * a.n_tiles;
    const int nk1 = static_cast<int>((a.K + 63) / 64);
    const int nk = nk1 * (a.parts > 1 ? a.parts : 1);
    constexpr uint32_t kCols = 2 * BN;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kPairStages; ++s) {
            mb_init(&full[s], 1);
            mb_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mb_init(&acc_full[b], 1);
            mb_init(&acc_empty[b], 16);  // every epilogue warp of both CTAs (used on the even CTA)
        }
        mb_init(&drain, 1);
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base)),
                     "n"(kCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    __syncthreads();
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    cluster_sync_pair();  // both CTAs' barriers and TMEM exist before either uses the other's
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base;

    if (warp == 0) {
        if (lane == 0) {  // TMA producer (both CTAs): this CTA's halves, completing on the even CTA's barrier
            uint32_t it = 0;
            for (int64_t t = pair; t < tiles && !abort_flag; t += pairs) {
                const int m0 = static_cast<int>((t % pm) * 2 * HALF_ROWS + rank * HALF_ROWS);
                const int n0 = static_cast<int>((t / pm) * BN + rank * HALF_ROWS);
                for (int k = 0; k < nk; ++k, ++it) {
                    const int s = it % kPairStages;
                    if (it >= kPairStages && !mb_wait(&empty[s], ((it / kPairStages) - 1) & 1, &abort_flag)) break;
                    if (rank == 0) mb_expect_tx(&full[s], 2 * kStageBytes);
                    const int part = k / nk1, kc = k - part * nk1;
                    const uint32_t bar = even_cta_addr(&full[s]);
                    tma_2d_pair(sa + s * HALF_ROWS * kTcBK, part == 0 ? &ma : (part == 1 ? &ma2 : &ma3), bar, kc * 64, m0);
                    tma_2d_pair(sb + s * HALF_ROWS * kTcBK, part == 0 ? &mb : (part == 1 ? &mb2 : &mb3), bar, kc * 64, n0);
                }
            }
            if (abort_flag && rank == 0) {  // the loads of both halves of the stages issued land first
                for (uint32_t j = it > static_cast<uint32_t>(kPairStages) ? it - kPairStages : 0; j < it; ++j)
                    mb_drain(&full[j % kPairStages], (j / kPairStages) & 1);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {  // MMA issuer: the even CTA only
            constexpr uint32_t idesc = idesc_bf16_pair(BN);
            uint32_t it = 0, lt = 0;
            for (int64_t t = pair; t < tiles && !abort_flag; t += pairs, ++lt) {
                const uint32_t b = lt & 1;
                if (!mb_wait(&acc_empty[b], ((lt >> 1) & 1) ^ 1, &abort_flag)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t d = tmem + b * BN;
                bool ok = true;
                for (int k = 0; k < nk; ++k, ++it) {
                    const int s = it % kPairStages;
                    if (!mb_wait(&full[s], (it / kPairStages) & 1, &abort_flag)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                    const uint64_t da = sdesc(sa + s * HALF_ROWS * kTcBK), db = sdesc(sb + s * HALF_ROWS * kTcBK);
#pragma unroll
                    for (int kk = 0; kk < kTcBK / 32; ++kk) {
                        const uint32_t accumulate = (k > 0 || kk > 0) ? 1u : 0u;
                        asm volatile(
                            "{\n .reg .pred p;\n setp.ne.u32 p, %4, 0;\n"
                            " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
                            "l"(da + static_cast<uint64_t>(2 * kk)), "l"(db + static_cast<uint64_t>(2 * kk)),
                            "r"(idesc), "r"(accumulate));
                    }
                    asm volatile(
                        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], "
                        "%1;" ::"r"(su32(&empty[s])),
                        "h"(static_cast<uint16_t>(3))
                        : "memory");
                }
                asm volatile(
                    "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                        su32(&acc_full[b])),
                    "h"(static_cast<uint16_t>(3))
                    : "memory");
                if (!ok) break;
            }
            if (abort_flag) {  // every MMA issued completes before either CTA frees TMEM or leaves
                asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                                 su32(&drain))
                             : "memory");
                mb_drain(&drain, 0);
            }
        }
    } else {  // epilogue warps 2..9 of both CTAs: TMEM lanes 32 (w % 4) .., column half (w - 2) / 4
        const int quarter = warp & 3, half = (warp - 2) >> 2;
        const int row_in_tile = quarter * 32 + lane;
        constexpr int HALF = BN / 2;
        const bool vec_out = (a.ld_out & 3) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0;
        const uint32_t empty_even[2] = {even_cta_addr(&acc_empty[0]), even_cta_addr(&acc_empty[1])};
        uint32_t lt = 0;
        for (int64_t t = pair; t < tiles && !abort_flag; t += pairs, ++lt) {
            const uint32_t b = lt & 1;
            if (!mb_wait(&acc_full[b], (lt >> 1) & 1, &abort_flag)) break;
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int64_t row = (t % pm) * 2 * HALF_ROWS + rank * HALF_ROWS + row_in_tile;
            const bool live_row = row < a.M;
            const int64_t o_base = (t / pm) * BN + half * HALF;
            for (int c = 0; c < HALF; c += 16) {
                uint32_t v[16];
                const uint32_t taddr = tmem + b * BN + (static_cast<uint32_t>(quarter * 32) << 16) + half * HALF + c;
                asm volatile(
                    "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                    : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
                      "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
                    : "r"(taddr));
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
                const int64_t o0 = o_base + c;
                if (!live_row || o0 >= a.N) continue;
                const int64_t idx = row * a.ld_out + o0;
                if (o0 + 16 <= a.N && vec_out) {
#pragma unroll
                    for (int j = 0; j < 16; j += 4)
                        *reinterpret_cast<float4 *>(a.out + idx + j) =
                            make_float4(__uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                                        __uint_as_float(v[j + 3]));
                } else {
                    for (int j = 0; j < 16 && o0 + j < a.N; ++j) a.out[idx + j] = __uint_as_float(v[j]);
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(empty_even[b])
                             : "memory");
        }
    }
    if (abort_flag && threadIdx.x == 0) set_flag(a.flags, BD_FLAG_TIMEOUT);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    cluster_sync_pair();  // no CTA frees TMEM or leaves while the pair's MMAs or loads may touch it
    if (warp == 1) {
        __syncwarp();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "n"(kCols));
    }
}

// ------------------------------------------------------------------ host side

static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// 2-D int8 (bf16 = false) or bf16 tensor [rows, cols] with row stride ld bytes
// (multiple of 16), boxes of box_rows x 128 bytes, 128-byte swizzle; reads past
// the tensor return zeros.
static bool make_i8_map(CUtensorMap *m, const void *ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                        bool bf16 = false) {
    auto enc = tensor_map_encoder();
    if (!enc || (reinterpret_cast<uintptr_t>(ptr) & 15) || (ld & 15)) return false;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(bf16 ? 64 : kTcBK), static_cast<cuuint32_t>(box_rows)};
    cuuint32_t es[2] = {1, 1};
    return enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8, 2,
               const_cast<void *>(ptr), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static int sms_tc() {
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

// Operands of a product of up to three parts: D = sum_p A_p . B_p^T (parts 2 and 3
// optional; every A_p has the row stride ld_codes, every B_p the stride ld_w).
struct TcParts {
    const int8_t *a2 = nullptr, *b2 = nullptr, *a3 = nullptr, *b3 = nullptr;
};

template <int BN, int EPI>
static int launch_tc_t(TcArgs a, const int8_t *codes, int64_t ld_codes, const int8_t *weights, int64_t w_rows,
                       int64_t ld_w, cudaStream_t stream, const TcParts &more = TcParts{}) {
    CUtensorMap ma, mb, ma2, mb2, ma3, mb3;
    const bool bf16 = tc_bf16(EPI);
    a.parts = more.a3 ? 3 : (more.a2 ? 2 : 1);
    if (!make_i8_map(&ma, codes, a.M, a.K, ld_codes, kTcBM, bf16) ||
        !make_i8_map(&mb, weights, w_rows, a.K, ld_w, BN, bf16) ||
        !make_i8_map(&ma2, more.a2 ? more.a2 : codes, a.M, a.K, ld_codes, kTcBM, bf16) ||
        !make_i8_map(&mb2, more.b2 ? more.b2 : weights, w_rows, a.K, ld_w, BN, bf16) ||
        !make_i8_map(&ma3, more.a3 ? more.a3 : codes, a.M, a.K, ld_codes, kTcBM, bf16) ||
        !make_i8_map(&mb3, more.b3 ? more.b3 : weights, w_rows, a.K, ld_w, BN, bf16))
        return BD_ERR_ALIGNMENT;
    a.m_tiles = (a.M + kTcBM - 1) / kTcBM;
    a.n_tiles = (w_rows + BN - 1) / BN;
    const size_t smem = static_cast<size_t>(kTcStages) * (kTcBM + BN) * kTcBK + 1024;
    auto kern = tc_gemm_kernel<BN, EPI>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
        return BD_ERR_LAUNCH;
    const int64_t tiles = a.m_tiles * a.n_tiles;
    a.splits = 1;
    a.split_full = tiles;
    if (EPI == TC_F32 && a.split_ws && (reinterpret_cast<uintptr_t>(a.split_ws) & 255) == 0) {
        const int64_t nk = (a.K + tc_bk(EPI) - 1) / tc_bk(EPI) * a.parts;
        int64_t full = tiles;
        int s = 1;
        tc_split_plan(tiles, nk, sms_tc(), full, s);
        if (s > 1 && tc_split_bytes(tiles - full, s, BN) <= a.split_ws_bytes) {
            a.splits = s;
            a.split_full = full;
            a.split_count = static_cast<int32_t *>(a.split_ws);
            a.split_part = reinterpret_cast<float *>(static_cast<char *>(a.split_ws) + kTcSplitCounts * sizeof(int32_t));
        }
    }
    const int64_t units = a.splits > 1 ? a.split_full + (tiles - a.split_full) * a.splits : tiles;
    if (EPI == TC_F32 && a.splits == 1 && BN == 256 && a.M >= 512 && tiles >= sms_tc()) {
        // SM pairs for products that fill the GPU: 256-row tiles, A and B halves per CTA
        // (the tensor maps' boxes are 128 rows); measured 4-8 % faster than single CTAs
        // at 2048-4096 rows
        CUtensorMap pb, pb2, pb3;
        if (!make_i8_map(&pb, weights, w_rows, a.K, ld_w, kTcBM, bf16) ||
            !make_i8_map(&pb2, more.b2 ? more.b2 : weights, w_rows, a.K, ld_w, kTcBM, bf16) ||
            !make_i8_map(&pb3, more.b3 ? more.b3 : weights, w_rows, a.K, ld_w, kTcBM, bf16))
            return BD_ERR_ALIGNMENT;
        const size_t psmem = static_cast<size_t>(kPairStages) * 2 * kTcBM * kTcBK + 1024;
        if (cudaFuncSetAttribute(tc_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(psmem)) !=
            cudaSuccess)
            return BD_ERR_LAUNCH;
        const int64_t ptiles = (a.M + 255) / 256 * a.n_tiles;
        const unsigned pgrid = static_cast<unsigned>(2 * std::min<int64_t>(ptiles, sms_tc() / 2));
        tc_pair_kernel<<<pgrid, 320, psmem, stream>>>(a, ma, pb, ma2, pb2, ma3, pb3);
        BD_CHECK_LAUNCH();
        return BD_OK;
    }
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>(units, sms_tc()));
    kern<<<grid, 320, smem, stream>>>(a, ma, mb, ma2, mb2, ma3, mb3);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

int64_t tc_tiles(int64_t m, int64_t n) { return (m + kTcBM - 1) / kTcBM * ((n + 255) / 256); }

int launch_tc_gemm(int epi, const TcArgs &a, const int8_t *codes, int64_t ld_codes, const int8_t *weights,
                   int64_t w_rows, int64_t ld_w, cudaStream_t stream, const TcParts &more = TcParts{}) {
    if (a.M < 1 || a.N < 1 || a.K < 1) return BD_ERR_INVALID;
    if ((more.a2 || more.a3) && !tc_bf16(epi)) return BD_ERR_INVALID;
    if (more.a3 && !more.a2) return BD_ERR_INVALID;
    switch (epi) {
        case TC_RAW:
            return launch_tc_t<256, TC_RAW>(a, codes, ld_codes, weights, w_rows, ld_w, stream);
        case TC_HE4:
            return launch_tc_t<256, TC_HE4>(a, codes, ld_codes, weights, w_rows, ld_w, stream);
        case TC_W1A1:
            return launch_tc_t<256, TC_W1A1>(a, codes, ld_codes, weights, w_rows, ld_w, stream);
        case TC_W1A1_SWIGLU:
            return launch_tc_t<256, TC_W1A1_SWIGLU>(a, codes, ld_codes, weights, w_rows, ld_w, stream);
        case TC_F32:
            return launch_tc_t<256, TC_F32>(a, codes, ld_codes, weights, w_rows, ld_w, stream, more);
        case TC_STE:
            return launch_tc_t<256, TC_STE>(a, codes, ld_codes, weights, w_rows, ld_w, stream, more);
        case TC_CE_STATS:
            return launch_tc_t<256, TC_CE_STATS>(a, codes, ld_codes, weights, w_rows, ld_w, stream, more);
        case TC_CE_GRAD:
            return launch_tc_t<256, TC_CE_GRAD>(a, codes, ld_codes, weights, w_rows, ld_w, stream, more);
        default:
            return BD_ERR_INVALID;
    }
}

// ------------------------------------------------------------------ I8 sign copies

// One thread per 16 consecutive columns of one (padded) row: 16 latents in (four
// 16-byte loads when the row stride allows), one 16-byte store of +-1 / 0 out.
__global__ void tile_i8_kernel(const float *__restrict__ latent, int64_t rows, int64_t cols, int64_t ld,
                               int8_t *__restrict__ out, int stride, int offset, int32_t *flags) {
    const int64_t rows_pad = (rows + kTcBM - 1) / kTcBM * kTcBM;
    const int64_t groups = ld / 16;
    const int64_t total = rows_pad * groups;
    const bool vec = (cols & 3) == 0 && (reinterpret_cast<uintptr_t>(latent) & 15) == 0;
    bool bad = false;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / groups, k0 = (i - r * groups) * 16;
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        if (r < rows) {
            const float *src = latent + r * cols + k0;
            float x[16];
            if (vec && k0 + 16 <= cols) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 f = __ldg(reinterpret_cast<const float4 *>(src) + q);
                    x[4 * q] = f.x;
                    x[4 * q + 1] = f.y;
                    x[4 * q + 2] = f.z;
                    x[4 * q + 3] = f.w;
                }
            } else {
#pragma unroll
                for (int e = 0; e < 16; ++e) x[e] = k0 + e < cols ? src[e] : 0.0f;
            }
#pragma unroll
            for (int e = 0; e < 16; ++e) {
                if (k0 + e < cols) {
                    bad |= !isfinite(x[e]);
                    w[e >> 2] |= static_cast<uint32_t>(x[e] >= 0.0f ? 0x01u : 0xFFu) << (8 * (e & 3));
                }
            }
        }
        const int64_t orow = ((r / kTcBM) * stride + offset) * kTcBM + (r % kTcBM);
        *reinterpret_cast<uint4 *>(out + orow * ld + k0) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_NONFINITE_LATENT);
}

int64_t i8_ld(int64_t cols) { return (cols + 15) / 16 * 16; }

}  // namespace bd

using namespace bd;

extern "C" int64_t bd_i8_ld(int64_t cols) { return cols < 1 ? 0 : i8_ld(cols); }

extern "C" int64_t bd_i8_bytes(int64_t rows, int64_t cols) {
    if (rows < 0 || cols < 0) return -1;
    return (rows + kTcBM - 1) / kTcBM * kTcBM * i8_ld(cols);
}

extern "C" int bd_tile_signs_i8(const float *latent, int64_t rows, int64_t cols, int8_t *out, int block_stride,
                                int block_offset, int32_t *flags, bd_stream_t stream) {
    if (rows < 0 || cols < 1 || block_stride < 1 || block_offset < 0 || block_offset >= block_stride)
        return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    if (!latent || !out) return BD_ERR_INVALID;
    const int64_t ld = i8_ld(cols);
    const int64_t total = (rows + kTcBM - 1) / kTcBM * kTcBM * (ld / 16);
    int64_t grid = (total + 255) / 256;
    if (grid > 148 * 16) grid = 148 * 16;
    tile_i8_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(latent, rows, cols, ld, out, block_stride,
                                                                    block_offset, flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_gemm_bf16(const uint16_t *a, int64_t m, int64_t k, int64_t lda, const uint16_t *b, int64_t n,
                            int64_t ldb, float *c, int64_t ldc, void *workspace, size_t workspace_bytes,
                            bd_stream_t stream) {
    if (m < 1 || k < 1 || n < 1 || lda < k || ldb < k || ldc < n || !a || !b || !c) return BD_ERR_INVALID;
    TcArgs t{};
    t.M = m;
    t.N = n;
    t.K = k;
    t.ld_out = ldc;
    t.out = c;
    t.split_ws = workspace;
    t.split_ws_bytes = workspace_bytes;
    // strides in bytes for the tensor maps (multiples of 16: lda, ldb multiples of 8)
    return launch_tc_gemm(TC_F32, t, reinterpret_cast<const int8_t *>(a), lda * 2,
                          reinterpret_cast<const int8_t *>(b), n, ldb * 2, static_cast<cudaStream_t>(stream));
}

extern "C" int bd_gemm_i8(const int8_t *codes, int64_t tokens, int64_t k, const int8_t *signs_i8, int64_t outs,
                          int32_t *dots, bd_stream_t stream) {
    if (tokens < 1 || k < 1 || outs < 1 || !codes || !signs_i8 || !dots) return BD_ERR_INVALID;
    TcArgs a{};
    a.M = tokens;
    a.N = outs;
    a.K = k;
    a.ld_out = outs;
    a.out_i32 = dots;
    return launch_tc_gemm(TC_RAW, a, codes, i8_ld(k), signs_i8, outs, i8_ld(k), stream);
}

// ------------------------------------------------------------------ W1A1 SwiGLU at any token count

struct LargePieces {
    int8_t *codes_x, *codes_h;
    int32_t *sums;
    float *mean_x, *mean_h, *hidden;
    size_t bytes;
};

static LargePieces carve_large(void *ws, int64_t tokens, int64_t hidden, int64_t inter) {
    char *base = static_cast<char *>(ws);
    size_t off = 0;
    auto take = [&](size_t n) {
        off = (off + 255) & ~static_cast<size_t>(255);
        char *p = base ? base + off : nullptr;
        off += n;
        return p;
    };
    LargePieces p{};
    p.codes_x = reinterpret_cast<int8_t *>(take(static_cast<size_t>(tokens) * i8_ld(hidden)));
    p.codes_h = reinterpret_cast<int8_t *>(take(static_cast<size_t>(tokens) * i8_ld(inter)));
    p.sums = reinterpret_cast<int32_t *>(take(static_cast<size_t>(tokens) * sizeof(int32_t)));
    p.mean_x = reinterpret_cast<float *>(take(static_cast<size_t>(tokens) * sizeof(float)));
    p.mean_h = reinterpret_cast<float *>(take(static_cast<size_t>(tokens) * sizeof(float)));
    p.hidden = reinterpret_cast<float *>(take(static_cast<size_t>(tokens) * inter * sizeof(float)));
    p.bytes = off;
    return p;
}

extern "C" size_t bd_ffn_large_workspace_bytes(int64_t tokens, int64_t hidden, int64_t inter) {
    return carve_large(nullptr, tokens, hidden, inter).bytes;
}

extern "C" int bd_ffn_w1a1_large(const bd_ffn_large_args *p, bd_stream_t stream) {
    if (!p || p->tokens < 1 || p->hidden < 1 || p->inter < 1 || p->tokens > 0x7fffffff) return BD_ERR_INVALID;
    if (!p->x || !p->y || !p->signs_gate_up_i8 || !p->signs_down_i8 || !p->scale_gate || !p->scale_up ||
        !p->scale_down)
        return BD_ERR_INVALID;
    const LargePieces w = carve_large(p->workspace, p->tokens, p->hidden, p->inter);
    if (!p->workspace || w.bytes > p->workspace_bytes) return BD_ERR_WORKSPACE;
    const int64_t T = p->tokens, H = p->hidden, F = p->inter;
    float *hidden = p->hidden_out ? p->hidden_out : w.hidden;
    int st = launch_binarize(p->x, T, H, i8_ld(H), w.codes_x, w.sums, w.mean_x, nullptr, 0, p->flags, stream, -1);
    if (st) return st;
    TcArgs g{};
    g.M = T;
    g.N = F;
    g.K = H;
    g.ld_out = F;
    g.scale = p->scale_gate;
    g.scale2 = p->scale_up;
    g.row_scale = w.mean_x;
    g.out = hidden;
    g.flags = p->flags;
    st = launch_tc_gemm(TC_W1A1_SWIGLU, g, w.codes_x, i8_ld(H), p->signs_gate_up_i8, 2 * ((F + kTcBM - 1) / kTcBM) * kTcBM,
                        i8_ld(H), stream);
    if (st) return st;
    st = launch_binarize(hidden, T, F, i8_ld(F), w.codes_h, w.sums, w.mean_h, nullptr, 0, p->flags, stream, -1);
    if (st) return st;
    TcArgs d{};
    d.M = T;
    d.N = H;
    d.K = F;
    d.ld_out = H;
    d.scale = p->scale_down;
    d.row_scale = w.mean_h;
    d.out = p->y;
    d.flags = p->flags;
    return launch_tc_gemm(TC_W1A1, d, w.codes_h, i8_ld(F), p->signs_down_i8, H, i8_ld(F), stream);
}

// ------------------------------------------------------------------ training-size HE4 projection and its
// straight-through gradients on tcgen05 (w1a1_eagle/model.py:71-73, 128-150)

extern "C" int bd_projection_he4_tc(const int8_t *codes, int64_t ld_codes, const int32_t *code_sums, int64_t tokens,
                                    int64_t in_features, const int8_t *signs_i8, int64_t out_features,
                                    const float *scale, const float *midpoint, const float *bound, int bits,
                                    const float *residual, float *y, float *dot, int32_t *flags, bd_stream_t stream) {
    if (tokens < 1 || in_features < 1 || out_features < 1 || (bits != 4 && bits != 8) || ld_codes < in_features ||
        tokens > 0x7fffffff)
        return BD_ERR_INVALID;
    if (!codes || !code_sums || !signs_i8 || !scale || !midpoint || !bound || !y) return BD_ERR_INVALID;
    TcArgs a{};
    a.M = tokens;
    a.N = out_features;
    a.K = in_features;
    a.ld_out = out_features;
    a.scale = scale;
    a.mid = midpoint;
    a.bound = bound;
    a.code_bits = bits;
    a.sums = code_sums;
    a.residual = residual;
    a.out = y;
    a.out_dot = dot;
    a.flags = flags;
    return launch_tc_gemm(TC_HE4, a, codes, ld_codes, signs_i8, out_features, i8_ld(in_features), stream);
}

extern "C" size_t bd_gemm_split_workspace_bytes(int64_t m, int64_t n, int64_t k, int parts) {
    if (m < 1 || n < 1 || k < 1 || parts < 1 || parts > 3) return 0;
    const int64_t tiles = tc_tiles(m, n);
    int64_t full = tiles;
    int s = 1;
    tc_split_plan(tiles, (k + 63) / 64 * parts, sms_tc(), full, s);
    return s > 1 ? tc_split_bytes(tiles - full, s, 256) : 0;
}

extern "C" int bd_gemm_bf16_split(const uint16_t *a_hi, const uint16_t *a_lo, int64_t m, int64_t k, int64_t lda,
                                  const uint16_t *b, int64_t n, int64_t ldb, float *c, int64_t ldc, void *workspace,
                                  size_t workspace_bytes, bd_stream_t stream) {
    if (m < 1 || k < 1 || n < 1 || lda < k || ldb < k || ldc < n || !a_hi || !b || !c) return BD_ERR_INVALID;
    TcArgs t{};
    t.M = m;
    t.N = n;
    t.K = k;
    t.ld_out = ldc;
    t.out = c;
    t.split_ws = workspace;
    t.split_ws_bytes = workspace_bytes;
    TcParts more;
    if (a_lo) {
        more.a2 = reinterpret_cast<const int8_t *>(a_lo);
        more.b2 = reinterpret_cast<const int8_t *>(b);
    }
    return launch_tc_gemm(TC_F32, t, reinterpret_cast<const int8_t *>(a_hi), lda * 2,
                          reinterpret_cast<const int8_t *>(b), n, ldb * 2, static_cast<cudaStream_t>(stream), more);
}

extern "C" int bd_gemm_bf16_split3(const uint16_t *a_hi, const uint16_t *a_lo, int64_t m, int64_t k, int64_t lda,
                                   const uint16_t *b_hi, const uint16_t *b_lo, int64_t n, int64_t ldb, float *c,
                                   int64_t ldc, void *workspace, size_t workspace_bytes, bd_stream_t stream) {
    if (m < 1 || k < 1 || n < 1 || lda < k || ldb < k || ldc < n || !a_hi || !a_lo || !b_hi || !c)
        return BD_ERR_INVALID;
    TcArgs t{};
    t.M = m;
    t.N = n;
    t.K = k;
    t.ld_out = ldc;
    t.out = c;
    t.split_ws = workspace;
    t.split_ws_bytes = workspace_bytes;
    TcParts more;
    more.a2 = reinterpret_cast<const int8_t *>(a_lo);
    more.b2 = reinterpret_cast<const int8_t *>(b_hi);
    if (b_lo) {
        more.a3 = reinterpret_cast<const int8_t *>(a_hi);
        more.b3 = reinterpret_cast<const int8_t *>(b_lo);
    }
    return launch_tc_gemm(TC_F32, t, reinterpret_cast<const int8_t *>(a_hi), lda * 2,
                          reinterpret_cast<const int8_t *>(b_hi), n, ldb * 2, static_cast<cudaStream_t>(stream), more);
}

extern "C" int64_t bd_ste_weight_grad_partials(int64_t out_features, int64_t in_features) {
    if (out_features < 1 || in_features < 1) return 0;
    return tc_tiles(out_features, in_features) * 8 * 2;
}

extern "C" int bd_ste_weight_grad(const uint16_t *grad_t_hi, const uint16_t *grad_t_lo, int64_t out_features,
                                  int64_t tokens, int64_t ld_t, const uint16_t *codes_t, int64_t in_features,
                                  const float *latent, const float *window, float window_value, const float *bound,
                                  int bits, float *d_latent, float *partials, int32_t *flags, bd_stream_t stream) {
    if (out_features < 1 || tokens < 1 || in_features < 1 || ld_t < tokens || (bound && bits != 4 && bits != 8) ||
        (!window && !(window_value >= 0.0f)))
        return BD_ERR_INVALID;
    if (!grad_t_hi || !codes_t || !latent || !d_latent) return BD_ERR_INVALID;
    TcArgs a{};
    a.M = out_features;
    a.N = in_features;
    a.K = tokens;
    a.ld_out = in_features;
    a.bound = bound;
    a.code_bits = bits;
    a.latent = latent;
    a.ld_latent = in_features;
    a.window = window;
    a.window_value = window_value;
    a.partials = partials;
    a.out = d_latent;
    a.flags = flags;
    TcParts more;
    if (grad_t_lo) {
        more.a2 = reinterpret_cast<const int8_t *>(grad_t_lo);
        more.b2 = reinterpret_cast<const int8_t *>(codes_t);
    }
    return launch_tc_gemm(TC_STE, a, reinterpret_cast<const int8_t *>(grad_t_hi), ld_t * 2,
                          reinterpret_cast<const int8_t *>(codes_t), in_features, ld_t * 2, stream, more);
}

// ------------------------------------------------------------------ fused cross-entropy head
// (w1a1_eagle/numerical/worker.py:315-363: cross_entropy(linear(head, vocabulary)) per label,
// weighted and summed); the logits are never written: one pass keeps per-row softmax
// statistics, a second recomputes them into the gradient in place.

__global__ void ce_reduce_kernel(const float *__restrict__ stats, const float *__restrict__ target, int64_t rows,
                                 int64_t nsplit, const float *__restrict__ weights, float *__restrict__ lse_out,
                                 float *__restrict__ loss_rows, int32_t *flags) {
    const int warp = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5), lane = threadIdx.x & 31;
    if (warp >= rows) return;
    const float *st = stats + static_cast<int64_t>(warp) * nsplit * 2;
    float m = -INFINITY;
    for (int64_t i = lane; i < nsplit; i += 32) m = fmaxf(m, st[2 * i]);
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
    float s = 0.0f;
    for (int64_t i = lane; i < nsplit; i += 32) {
        const float mi = st[2 * i];
        if (mi != -INFINITY) s = __fadd_rn(s, __fmul_rn(st[2 * i + 1], exp2f((mi - m) * 1.4426950408889634f)));
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, d));
    if (lane == 0) {
        const float lse = __fadd_rn(m, logf(s));
        const float loss = __fsub_rn(lse, target[warp]);
        if (!isfinite(loss)) set_flag(flags, BD_FLAG_NONFINITE_LOSS);
        lse_out[warp] = lse;
        loss_rows[warp] = __fmul_rn(weights[warp], loss);
    }
}

// total = sum of loss_rows in a fixed order (one block)
__global__ void ce_total_kernel(const float *__restrict__ loss_rows, int64_t rows, float *__restrict__ total) {
    __shared__ float part[256];
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < rows; i += 256) s = __fadd_rn(s, loss_rows[i]);
    part[threadIdx.x] = s;
    __syncthreads();
    for (int w = 128; w > 0; w >>= 1) {
        if (threadIdx.x < w) part[threadIdx.x] = __fadd_rn(part[threadIdx.x], part[threadIdx.x + w]);
        __syncthreads();
    }
    if (threadIdx.x == 0) total[0] = part[0];
}

extern "C" int64_t bd_loss_head_stats_count(int64_t rows, int64_t vocab) {
    if (rows < 1 || vocab < 1) return 0;
    return rows * 2 * ((vocab + 255) / 256) * 2;
}

extern "C" int bd_loss_head_forward(const uint16_t *h_hi, const uint16_t *h_lo, int64_t rows, int64_t hidden,
                                    int64_t ld_h, const uint16_t *v_hi, const uint16_t *v_lo, int64_t vocab,
                                    const int32_t *labels, const float *weights, float *stats, float *target,
                                    float *lse, float *loss_rows, float *loss, int32_t *flags, bd_stream_t stream) {
    if (rows < 1 || hidden < 1 || vocab < 1 || ld_h < hidden || (ld_h & 7) || !h_hi || !h_lo || !v_hi || !labels ||
        !weights || !stats || !target || !lse || !loss_rows || !loss)
        return BD_ERR_INVALID;
    TcArgs a{};
    a.M = rows;
    a.N = vocab;
    a.K = hidden;
    a.ld_out = vocab;
    a.labels = labels;
    a.stats = stats;
    a.target = target;
    a.flags = flags;
    TcParts more;
    more.a2 = reinterpret_cast<const int8_t *>(h_lo);
    more.b2 = reinterpret_cast<const int8_t *>(v_hi);
    if (v_lo) {
        more.a3 = reinterpret_cast<const int8_t *>(h_hi);
        more.b3 = reinterpret_cast<const int8_t *>(v_lo);
    }
    int st = launch_tc_gemm(TC_CE_STATS, a, reinterpret_cast<const int8_t *>(h_hi), ld_h * 2,
                            reinterpret_cast<const int8_t *>(v_hi), vocab, ld_h * 2, stream, more);
    if (st) return st;
    const int64_t nsplit = 2 * ((vocab + 255) / 256);
    ce_reduce_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, stream>>>(stats, target, rows, nsplit, weights,
                                                                                 lse, loss_rows, flags);
    BD_CHECK_LAUNCH();
    ce_total_kernel<<<1, 256, 0, stream>>>(loss_rows, rows, loss);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_loss_head_grad(const uint16_t *h_hi, const uint16_t *h_lo, int64_t rows, int64_t hidden,
                                 int64_t ld_h, const uint16_t *v_hi, const uint16_t *v_lo, int64_t vocab,
                                 const int32_t *labels, const float *weights, const float *lse, uint16_t *dl_hi,
                                 uint16_t *dl_lo, int64_t ld_dl, bd_stream_t stream) {
    if (rows < 1 || hidden < 1 || vocab < 1 || ld_h < hidden || (ld_h & 7) || ld_dl < vocab || (ld_dl & 7) || !h_hi ||
        !h_lo || !v_hi || !labels || !weights || !lse || !dl_hi || !dl_lo)
        return BD_ERR_INVALID;
    TcArgs a{};
    a.M = rows;
    a.N = vocab;
    a.K = hidden;
    a.ld_out = ld_dl;
    a.labels = labels;
    a.row_w = weights;
    a.row_lse = lse;
    a.dl_hi = reinterpret_cast<__nv_bfloat16 *>(dl_hi);
    a.dl_lo = reinterpret_cast<__nv_bfloat16 *>(dl_lo);
    TcParts more;
    more.a2 = reinterpret_cast<const int8_t *>(h_lo);
    more.b2 = reinterpret_cast<const int8_t *>(v_hi);
    if (v_lo) {
        more.a3 = reinterpret_cast<const int8_t *>(h_hi);
        more.b3 = reinterpret_cast<const int8_t *>(v_lo);
    }
    return launch_tc_gemm(TC_CE_GRAD, a, reinterpret_cast<const int8_t *>(h_hi), ld_h * 2,
                          reinterpret_cast<const int8_t *>(v_hi), vocab, ld_h * 2, stream, more);
}
