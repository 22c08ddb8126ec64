// Training-size block attention of Layer.group (w1a1_eagle/model.py:225-270):
// W windows of k <= 16 slots, grouped-query heads (g = heads / kv_heads <= 4
// query heads per kv head), each slot attending to the shared context keys its
// mask allows and to its window's own slots, one softmax over both parts; the
// forward and its backward (dQ, dK, dV of the context and of the slots).
//
// Operands are prepared on the host side as fp16 rows of DP (the head dim
// rounded up to 16, 32, 64 or 128) in head-major tiles:
//   qh, ql    [kv_heads][W][g][16][DP]  query hi + lo halves (x = hi + lo to ~22 bits)
//   doh, dol  [kv_heads][W][g][16][DP]  output gradient, times a power of two (dscale), hi + lo
//   kc, vc    [kv_heads][Lp][DP]        context keys / values (fp16 values, exact), Lp = L rounded up to 64
//   ks, vs    [kv_heads][W][16][DP]     the windows' slot keys / values
//   mctx      [W][16][Lp] uint8         context mask rows (slot, key); padding rows and keys 0
//   mslot     [16][16] uint8            slot-to-slot mask; padding 0
// so every product runs on fp16 m16n8k16 tensor-core MMAs with fp32
// accumulation: a product with one exact fp16 operand takes two MMAs (hi and lo
// of the other), one with neither exact three (hi hi, hi lo, lo hi).
//
// train_attn_fwd_kernel   CTA (window, kv head), 8 warps = 4 query heads x 2
//                         halves of the key tiles (64 keys each: the context
//                         tiles, then one tile of the window's slots); online
//                         softmax per half, halves merged through shared
//                         memory.  Writes O and the row log-sum-exp.
// train_attn_bwd_kv_kernel CTA (key tile, kv head), 4 warps of 16 keys: loops
//                         over the query tiles that see the tile (the windows
//                         that see a context tile, split over 4 CTAs whose
//                         partial sums are added in order afterwards; its own
//                         window for a slot tile), recomputes P^T from the saved
//                         log-sum-exp and accumulates dV = P^T dO and
//                         dK = dS^T Q in registers.
// train_attn_bwd_q_kernel CTA (window, kv head) like the forward: recomputes P
//                         and dP = dO V^T per key tile and accumulates dQ = dS K.
// Fully masked (query tile, key tile) pairs are skipped.  Every output element
// is written by one thread in a fixed order: no atomics, deterministic.
#include "kernels.cuh"

namespace bd {

constexpr int kTKeys = 64;  // keys per tile

struct TrainAttnArgs {
    const __half *qh, *ql, *doh, *dol;
    const __half *kc, *vc, *ks, *vs;
    const uint8_t *mctx, *mslot;
    const float *lse_in, *dr;  // [kv_heads][W][g][16]: saved log-sum-exp; rowsum(dO' * O)
    const float *unscale;      // 1 / dscale (device scalar)
    uint8_t *live;             // [W][Lp / 64 + 1]: does the window see any key of the tile (the forward
                               // writes it when not null; the dK/dV backward skips unseen tiles with it)
    float *o, *lse;            // forward outputs: [W][k][kv_heads][g][D], [kv_heads][W][g][16]
    float *dq;                 // [W][k][kv_heads][g][D]
    float *dkc, *dvc;          // [L][kv_heads][D]
    float *dks, *dvs;          // [W][k][kv_heads][D]
    float *kv_part;            // [2][kKvSplit][L][kv_heads][D]: the context dK, dV of each window share
    int W, k, kvh, g, D, L, Lp;
    float scale;               // 1 / sqrt(head_dim)
};

template <int DP>
constexpr int trow() { return DP * 2 + 16; }  // padded staged row (conflict-free ldmatrix)

// Key tile `tile` of (window w, kv head h) into K and V rows (64 x trow) and its
// mask rows (16 slots x 64 keys); rows and keys past the live ones are zero.
template <int DP>
__device__ __forceinline__ void stage_key_tile(const TrainAttnArgs &a, int h, int w, int tile, char *ks, char *vs,
                                               uint8_t *mk, int tid, int nthreads) {
    constexpr int RB = trow<DP>(), CH = DP * 2 / 16;
    const int nctx = a.Lp / kTKeys;
    for (int i = tid; i < kTKeys * CH; i += nthreads) {
        const int r = i / CH, c = i % CH;
        const __half *sk = a.ks, *sv = a.vs;
        int bytes = 0;
        if (tile < nctx) {
            const int64_t row = static_cast<int64_t>(h) * a.Lp + static_cast<int64_t>(tile) * kTKeys + r;
            sk = a.kc + row * DP + c * 8;
            sv = a.vc + row * DP + c * 8;
            bytes = 16;
        } else if (tile == nctx && r < 16) {
            const int64_t row = (static_cast<int64_t>(h) * a.W + w) * 16 + r;
            sk = a.ks + row * DP + c * 8;
            sv = a.vs + row * DP + c * 8;
            bytes = 16;
        }
        cp_async16(ks + r * RB + c * 16, sk, bytes);
        cp_async16(vs + r * RB + c * 16, sv, bytes);
    }
    for (int i = tid; i < 16 * 4; i += nthreads) {
        const int s = i >> 2, c = i & 3;
        const uint8_t *src = a.mslot;
        int bytes = 0;
        if (tile < nctx) {
            src = a.mctx + (static_cast<int64_t>(w) * 16 + s) * a.Lp + static_cast<int64_t>(tile) * kTKeys + c * 16;
            bytes = 16;
        } else if (tile == nctx && c == 0) {
            src = a.mslot + s * 16;
            bytes = 16;
        }
        cp_async16(mk + s * 64 + c * 16, src, bytes);
    }
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// A fragment (16 rows x 16 columns of fp16, row-major in shared memory, row pitch RB)
__device__ __forceinline__ void lda16(uint32_t (&r)[4], const char *base, int RB, int col, int lane) {
    ldmatrix_x4(r, base + (lane & 15) * RB + (col + (lane >> 4) * 8) * 2);
}

// S (16 rows x 64 keys) += A (16 x DP, from qa rows) . K^T for both halves of A.
template <int DP>
__device__ __forceinline__ void rows_times_keys(float (&acc)[8][4], const char *ah, const char *al, const char *keys,
                                                int lane) {
    constexpr int RB = trow<DP>();
#pragma unroll
    for (int s2 = 0; s2 < DP / 32; ++s2) {
        uint32_t h0[4], l0[4], h1[4], l1[4];
        lda16(h0, ah, RB, s2 * 32, lane);
        lda16(l0, al, RB, s2 * 32, lane);
        lda16(h1, ah, RB, s2 * 32 + 16, lane);
        lda16(l1, al, RB, s2 * 32 + 16, lane);
#pragma unroll
        for (int n = 0; n < 8; ++n) {
            uint32_t b[4];
            ldmatrix_x4(b, keys + (n * 8 + (lane & 7)) * RB + (s2 * 32 + (lane >> 3) * 8) * 2);
            mma_f16_16816(acc[n], h0[0], h0[1], h0[2], h0[3], b[0], b[1]);
            mma_f16_16816(acc[n], l0[0], l0[1], l0[2], l0[3], b[0], b[1]);
            mma_f16_16816(acc[n], h1[0], h1[1], h1[2], h1[3], b[2], b[3]);
            mma_f16_16816(acc[n], l1[0], l1[1], l1[2], l1[3], b[2], b[3]);
        }
    }
}
// The DP = 16 case has one k-step.
template <>
__device__ __forceinline__ void rows_times_keys<16>(float (&acc)[8][4], const char *ah, const char *al,
                                                    const char *keys, int lane) {
    constexpr int RB = trow<16>();
    uint32_t h0[4], l0[4];
    lda16(h0, ah, RB, 0, lane);
    lda16(l0, al, RB, 0, lane);
#pragma unroll
    for (int n = 0; n < 8; ++n) {
        uint32_t b[4];
        // x4 over 8 keys: matrices (k 0-7), (k 8-15) twice; only the first two are used
        ldmatrix_x4(b, keys + (n * 8 + (lane & 7)) * RB + ((lane >> 3) & 1) * 16);
        mma_f16_16816(acc[n], h0[0], h0[1], h0[2], h0[3], b[0], b[1]);
        mma_f16_16816(acc[n], l0[0], l0[1], l0[2], l0[3], b[0], b[1]);
    }
}

// acc (16 rows x DP) += P (16 x 64 keys, fp32 C fragments) . V (64 keys x DP rows),
// P as fp16 hi + lo (V exact).
template <int DP>
__device__ __forceinline__ void probs_times_values(float (&acc)[DP / 8][4], const float (&p)[8][4], const char *vals,
                                                   int lane) {
    constexpr int RB = trow<DP>();
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
        uint32_t a0, a1, a2, a3, l0, l1, l2, l3;
        split_half2(p[2 * kk][0], p[2 * kk][1], a0, l0);
        split_half2(p[2 * kk][2], p[2 * kk][3], a1, l1);
        split_half2(p[2 * kk + 1][0], p[2 * kk + 1][1], a2, l2);
        split_half2(p[2 * kk + 1][2], p[2 * kk + 1][3], a3, l3);
#pragma unroll
        for (int n2 = 0; n2 < DP / 16; ++n2) {
            uint32_t b[4];
            const int mi = lane >> 3, r = lane & 7;
            ldmatrix_x4_trans(b, vals + (kk * 16 + (mi & 1) * 8 + r) * RB + (n2 * 16 + (mi >> 1) * 8) * 2);
            mma_f16_16816(acc[2 * n2], a0, a1, a2, a3, b[0], b[1]);
            mma_f16_16816(acc[2 * n2], l0, l1, l2, l3, b[0], b[1]);
            mma_f16_16816(acc[2 * n2 + 1], a0, a1, a2, a3, b[2], b[3]);
            mma_f16_16816(acc[2 * n2 + 1], l0, l1, l2, l3, b[2], b[3]);
        }
    }
}

__device__ __forceinline__ bool tile_any(const uint8_t *mk, int lane) {
    const uint4 *m = reinterpret_cast<const uint4 *>(mk);
    const uint4 x = m[2 * lane], y = m[2 * lane + 1];
    return __any_sync(0xffffffffu, (x.x | x.y | x.z | x.w | y.x | y.y | y.z | y.w) != 0u);
}

// Stage this CTA's query-side rows (four heads x 16 rows x DP, hi and lo) into
// shared memory: src [kv_heads][W][g][16][DP].
template <int DP>
__device__ __forceinline__ void stage_rows(const TrainAttnArgs &a, const __half *hi, const __half *lo, int h, int w,
                                           char *dst_hi, char *dst_lo, int tid, int nthreads) {
    constexpr int RB = trow<DP>(), CH = DP * 2 / 16;
    for (int i = tid; i < 4 * 16 * CH; i += nthreads) {
        const int j = i / (16 * CH), r = (i / CH) % 16, c = i % CH;
        const bool live = j < a.g;
        const int64_t row = ((static_cast<int64_t>(h) * a.W + w) * a.g + (live ? j : 0)) * 16 + r;
        cp_async16(dst_hi + (j * 16 + r) * RB + c * 16, hi + row * DP + c * 8, live ? 16 : 0);
        cp_async16(dst_lo + (j * 16 + r) * RB + c * 16, lo + row * DP + c * 8, live ? 16 : 0);
    }
}

template <int DP>
constexpr size_t fwd_smem() {
    // [2 stages][2 halves] x (K + V tiles) + masks, then the query rows (hi, lo)
    return static_cast<size_t>(8) * kTKeys * trow<DP>() + 4 * 1024 + static_cast<size_t>(2) * 64 * trow<DP>();
}

template <int DP>
__global__ void __launch_bounds__(256, 1) train_attn_fwd_kernel(const TrainAttnArgs a) {
    constexpr int RB = trow<DP>(), KV = kTKeys * RB, NO = DP / 8;
    extern __shared__ __align__(16) char sm[];
    uint8_t *mbase = reinterpret_cast<uint8_t *>(sm + 8 * KV);
    char *qs_hi = sm + 8 * KV + 4 * 1024, *qs_lo = qs_hi + 64 * RB;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int hw = warp & 3, kh = warp >> 2;
    const int w = blockIdx.x, h = blockIdx.y;
    const bool head_live = hw < a.g;
    const int ntiles = a.Lp / kTKeys + 1;
    const int iters = (ntiles + 1) / 2;
    auto kbuf = [&](int st, int half) { return sm + ((st * 2 + half) * 2) * KV; };
    auto vbuf = [&](int st, int half) { return sm + ((st * 2 + half) * 2 + 1) * KV; };
    auto mbuf = [&](int st, int half) { return mbase + (st * 2 + half) * 1024; };

    stage_rows<DP>(a, a.qh, a.ql, h, w, qs_hi, qs_lo, threadIdx.x, blockDim.x);
    for (int half = 0; half < 2; ++half)
        stage_key_tile<DP>(a, h, w, half, kbuf(0, half), vbuf(0, half), mbuf(0, half), threadIdx.x, blockDim.x);
    cp_async_commit();

    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.0f, 0.0f};
    float o[NO][4];
#pragma unroll
    for (int n = 0; n < NO; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) o[n][i] = 0.0f;
    for (int it = 0; it < iters; ++it) {
        const int st = it & 1;
        if (it + 1 < iters) {
            for (int half = 0; half < 2; ++half)
                stage_key_tile<DP>(a, h, w, 2 * (it + 1) + half, kbuf(st ^ 1, half), vbuf(st ^ 1, half),
                                   mbuf(st ^ 1, half), threadIdx.x, blockDim.x);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const int tile = 2 * it + kh;
        const uint8_t *mk = mbuf(st, kh);
        const bool seen = head_live && tile < ntiles && tile_any(mk, lane);
        if (a.live && h == 0 && hw == 0 && lane == 0 && tile < ntiles) a.live[static_cast<int64_t>(w) * ntiles + tile] = seen;
        if (seen) {
            float s[8][4];
#pragma unroll
            for (int n = 0; n < 8; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) s[n][i] = 0.0f;
            rows_times_keys<DP>(s, qs_hi + hw * 16 * RB, qs_lo + hw * 16 * RB, kbuf(st, kh), lane);
            float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int n = 0; n < 8; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int row = g + 8 * (i >> 1), key = n * 8 + 2 * t + (i & 1);
                    const float v = mk[row * 64 + key] ? s[n][i] * a.scale : -INFINITY;
                    s[n][i] = v;
                    tmax[i >> 1] = fmaxf(tmax[i >> 1], v);
                }
            float corr[2];
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 1));
                tmax[r] = fmaxf(tmax[r], __shfl_xor_sync(0xffffffffu, tmax[r], 2));
                const float mn = fmaxf(m[r], tmax[r]);
                corr[r] = (m[r] == -INFINITY) ? (mn == -INFINITY ? 1.0f : 0.0f) : __expf(m[r] - mn);
                m[r] = mn;
            }
            float ls[2] = {0.0f, 0.0f};
#pragma unroll
            for (int n = 0; n < 8; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const float mm = m[i >> 1];
                    const float p = s[n][i] == -INFINITY ? 0.0f : __expf(s[n][i] - mm);
                    s[n][i] = p;
                    ls[i >> 1] += p;
                }
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 1);
                ls[r] += __shfl_xor_sync(0xffffffffu, ls[r], 2);
                l[r] = l[r] * corr[r] + ls[r];
            }
#pragma unroll
            for (int n = 0; n < NO; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) o[n][i] *= corr[i >> 1];
            probs_times_values<DP>(o, s, vbuf(st, kh), lane);
        }
        __syncthreads();  // the stage is refilled next iteration
    }
    // half 1 hands (O, m, l) to half 0 through the key-tile area
    constexpr int X = NO * 4 + 4;
    float *xch = reinterpret_cast<float *>(sm) + (hw * X) * 32 + lane;
    if (head_live && kh == 1) {
#pragma unroll
        for (int n = 0; n < NO; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) xch[(n * 4 + i) * 32] = o[n][i];
        xch[(X - 4) * 32] = m[0];
        xch[(X - 3) * 32] = m[1];
        xch[(X - 2) * 32] = l[0];
        xch[(X - 1) * 32] = l[1];
    }
    __syncthreads();
    if (!head_live || kh == 1) return;
    float f0[2], f1[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const float m1 = xch[(X - 4 + r) * 32], l1 = xch[(X - 2 + r) * 32];
        const float mx = fmaxf(m[r], m1);
        f0[r] = m[r] == -INFINITY ? 0.0f : __expf(m[r] - mx);
        f1[r] = m1 == -INFINITY ? 0.0f : __expf(m1 - mx);
        l[r] = l[r] * f0[r] + l1 * f1[r];
        m[r] = mx;
    }
    float inv[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) inv[r] = l[r] > 0.0f ? 1.0f / l[r] : 0.0f;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int slot = g + 8 * r;
        if (slot >= a.k) continue;
        float *dst = a.o + ((((static_cast<int64_t>(w) * a.k + slot) * a.kvh + h) * a.g + hw) * a.D);
#pragma unroll
        for (int n = 0; n < NO; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int col = n * 8 + 2 * t + e;
                if (col < a.D) dst[col] = (o[n][2 * r + e] * f0[r] + xch[(n * 4 + 2 * r + e) * 32] * f1[r]) * inv[r];
            }
        if (t == 0)
            a.lse[((static_cast<int64_t>(h) * a.W + w) * a.g + hw) * 16 + slot] =
                l[r] > 0.0f ? m[r] + __logf(l[r]) : INFINITY;
    }
}

// ------------------------------------------------------------------ backward: dK, dV

constexpr int kLiveList = 4096;  // windows listed per context tile (more: every window is staged)
constexpr int kKvSplit = 4;      // CTAs per context key tile, each over a contiguous share of its windows

template <int DP>
constexpr size_t kv_smem() {
    // K and V tiles, then [2 stages] x (q hi, q lo, dO hi, dO lo rows, mask, lse, dr), then the window list
    return static_cast<size_t>(2) * kTKeys * trow<DP>() + 2 * (static_cast<size_t>(4) * 16 * trow<DP>() + 1024 + 128) +
           kLiveList * sizeof(uint16_t);
}

// dst (16 keys x DP, C fragments) += src^T (16 keys x 16 rows, C fragments of two n-tiles) . R (16 rows x DP),
// both sides hi + lo: three MMAs (hi hi, hi lo, lo hi).
template <int DP>
__device__ __forceinline__ void keys_times_rows(float (&acc)[DP / 8][4], const float (&c)[2][4], const char *rh,
                                                const char *rl, int lane) {
    constexpr int RB = trow<DP>();
    uint32_t a0, a1, a2, a3, l0, l1, l2, l3;
    split_half2(c[0][0], c[0][1], a0, l0);
    split_half2(c[0][2], c[0][3], a1, l1);
    split_half2(c[1][0], c[1][1], a2, l2);
    split_half2(c[1][2], c[1][3], a3, l3);
#pragma unroll
    for (int n2 = 0; n2 < DP / 16; ++n2) {
        uint32_t bh[4], bl[4];
        const int mi = lane >> 3, r = lane & 7;
        const int off = ((mi & 1) * 8 + r) * RB + (n2 * 16 + (mi >> 1) * 8) * 2;
        ldmatrix_x4_trans(bh, rh + off);
        ldmatrix_x4_trans(bl, rl + off);
        mma_f16_16816(acc[2 * n2], a0, a1, a2, a3, bh[0], bh[1]);
        mma_f16_16816(acc[2 * n2], a0, a1, a2, a3, bl[0], bl[1]);
        mma_f16_16816(acc[2 * n2], l0, l1, l2, l3, bh[0], bh[1]);
        mma_f16_16816(acc[2 * n2 + 1], a0, a1, a2, a3, bh[2], bh[3]);
        mma_f16_16816(acc[2 * n2 + 1], a0, a1, a2, a3, bl[2], bl[3]);
        mma_f16_16816(acc[2 * n2 + 1], l0, l1, l2, l3, bh[2], bh[3]);
    }
}

// C (16 keys x 16 rows) += K_w (16 x DP, exact fp16) . R^T (R: 16 rows x DP, hi + lo).
template <int DP>
__device__ __forceinline__ void keys_dot_rows(float (&acc)[2][4], const char *keys, const char *rh, const char *rl,
                                              int lane) {
    constexpr int RB = trow<DP>();
#pragma unroll
    for (int ks = 0; ks < DP / 16; ++ks) {
        uint32_t ka[4];
        lda16(ka, keys, RB, ks * 16, lane);
#pragma unroll
        for (int n = 0; n < 2; ++n) {
            uint32_t bh[4], bl[4];
            // x4 over 8 rows: (k 0-7), (k 8-15) of this k-step, twice
            const int off = (n * 8 + (lane & 7)) * RB + (ks * 16 + ((lane >> 3) & 1) * 8) * 2;
            ldmatrix_x4(bh, rh + off);
            ldmatrix_x4(bl, rl + off);
            mma_f16_16816(acc[n], ka[0], ka[1], ka[2], ka[3], bh[0], bh[1]);
            mma_f16_16816(acc[n], ka[0], ka[1], ka[2], ka[3], bl[0], bl[1]);
        }
    }
}

template <int DP>
__global__ void __launch_bounds__(128) train_attn_bwd_kv_kernel(const TrainAttnArgs a) {
    constexpr int RB = trow<DP>(), KV = kTKeys * RB, NO = DP / 8;
    constexpr size_t STAGE = static_cast<size_t>(4) * 16 * RB + 1024 + 128;
    extern __shared__ __align__(16) char sm[];
    char *kt = sm, *vt = sm + KV;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int nctx = a.Lp / kTKeys;
    const int h = blockIdx.y;
    // blocks [0, nctx x kKvSplit): context tile, share of its windows; then one per window's slots
    const bool slot_tile = static_cast<int>(blockIdx.x) >= nctx * kKvSplit;
    const int tile = slot_tile ? nctx + (static_cast<int>(blockIdx.x) - nctx * kKvSplit) : blockIdx.x / kKvSplit;
    const int part = slot_tile ? 0 : blockIdx.x % kKvSplit;
    const int wslot = tile - nctx;
    auto sbase = [&](int st) { return sm + 2 * KV + st * STAGE; };
    // the windows that see this context tile, in window order (the forward's table;
    // without it, or with more windows than the list holds, every window)
    uint16_t *wlist = reinterpret_cast<uint16_t *>(sm + 2 * KV + 2 * STAGE);
    __shared__ int nlive_s;
    const bool listed = !slot_tile && a.live && a.W <= kLiveList;
    if (listed && threadIdx.x < 32) {
        const int ntiles = nctx + 1;
        int count = 0;
        for (int w0 = 0; w0 < a.W; w0 += 32) {
            const int w = w0 + static_cast<int>(threadIdx.x);
            const bool on = w < a.W && a.live[static_cast<int64_t>(w) * ntiles + tile] != 0;
            const unsigned mask = __ballot_sync(0xffffffffu, on);
            if (on) wlist[count + __popc(mask & ((1u << threadIdx.x) - 1u))] = static_cast<uint16_t>(w);
            count += __popc(mask);
        }
        if (threadIdx.x == 0) nlive_s = count;
    }
    __syncthreads();
    const int nwin = listed ? nlive_s : a.W;
    const int w_begin = part * nwin / kKvSplit, w_end = (part + 1) * nwin / kKvSplit;
    const int nq = slot_tile ? a.g : (w_end - w_begin) * a.g;
    // the query tile qt: its rows (hi, lo of q and dO), mask (16 x 64), lse and dr
    auto stage_q = [&](int st, int qt) {
        const int wi = w_begin + qt / a.g;
        const int w = slot_tile ? wslot : (listed ? static_cast<int>(wlist[wi]) : wi);
        const int j = slot_tile ? qt : qt % a.g;
        char *b = sbase(st);
        constexpr int CH = DP * 2 / 16;
        const int64_t row0 = ((static_cast<int64_t>(h) * a.W + w) * a.g + j) * 16;
        for (int i = threadIdx.x; i < 4 * 16 * CH; i += blockDim.x) {
            const int which = i / (16 * CH), r = (i / CH) % 16, c = i % CH;
            const __half *src = which == 0 ? a.qh : which == 1 ? a.ql : which == 2 ? a.doh : a.dol;
            cp_async16(b + (which * 16 + r) * RB + c * 16, src + (row0 + r) * DP + c * 8, 16);
        }
        uint8_t *mk = reinterpret_cast<uint8_t *>(b + 4 * 16 * RB);
        for (int i = threadIdx.x; i < 64; i += blockDim.x) {
            const int s = i >> 2, c = i & 3;
            const uint8_t *src = a.mslot;
            int bytes = 0;
            if (!slot_tile) {
                src = a.mctx + (static_cast<int64_t>(w) * 16 + s) * a.Lp + static_cast<int64_t>(tile) * kTKeys + c * 16;
                bytes = 16;
            } else if (c == 0) {
                src = a.mslot + s * 16;
                bytes = 16;
            }
            cp_async16(mk + s * 64 + c * 16, src, bytes);
        }
        float *sc = reinterpret_cast<float *>(b + 4 * 16 * RB + 1024);
        if (threadIdx.x < 8) {
            const int which = threadIdx.x >> 2, c = threadIdx.x & 3;
            cp_async16(sc + which * 16 + c * 4, (which ? a.dr : a.lse_in) + row0 + c * 4, 16);
        }
    };
    // the key tile (and a dummy mask area: masks come with the query tiles)
    {
        constexpr int CH = DP * 2 / 16;
        for (int i = threadIdx.x; i < kTKeys * CH; i += blockDim.x) {
            const int r = i / CH, c = i % CH;
            const __half *sk = a.ks, *sv = a.vs;
            int bytes = 0;
            if (!slot_tile) {
                const int64_t row = static_cast<int64_t>(h) * a.Lp + static_cast<int64_t>(tile) * kTKeys + r;
                sk = a.kc + row * DP + c * 8;
                sv = a.vc + row * DP + c * 8;
                bytes = 16;
            } else if (r < 16) {
                const int64_t row = (static_cast<int64_t>(h) * a.W + wslot) * 16 + r;
                sk = a.ks + row * DP + c * 8;
                sv = a.vs + row * DP + c * 8;
                bytes = 16;
            }
            cp_async16(kt + r * RB + c * 16, sk, bytes);
            cp_async16(vt + r * RB + c * 16, sv, bytes);
        }
    }
    if (nq > 0) stage_q(0, 0);
    cp_async_commit();

    float dk[NO][4], dv[NO][4];
#pragma unroll
    for (int n = 0; n < NO; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) dk[n][i] = dv[n][i] = 0.0f;
    const bool warp_live = !slot_tile || warp == 0;  // a slot tile has 16 live keys
    for (int qt = 0; qt < nq; ++qt) {
        const int st = qt & 1;
        if (qt + 1 < nq) {
            stage_q(st ^ 1, qt + 1);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        char *b = sbase(st);
        const char *qh = b, *ql = b + 16 * RB, *dh = b + 32 * RB, *dl = b + 48 * RB;
        const uint8_t *mk = reinterpret_cast<const uint8_t *>(b + 4 * 16 * RB);
        const float *lse = reinterpret_cast<const float *>(b + 4 * 16 * RB + 1024), *dr = lse + 16;
        // this warp's 16 keys: mask bytes (row s, key 16 warp + 0..15), 8 per lane
        const uint2 mw = *reinterpret_cast<const uint2 *>(mk + (lane >> 1) * 64 + warp * 16 + (lane & 1) * 8);
        if (warp_live && __any_sync(0xffffffffu, (mw.x | mw.y) != 0u)) {
            const char *kw = kt + warp * 16 * RB, *vw = vt + warp * 16 * RB;
            float sT[2][4] = {}, dpT[2][4] = {};
            keys_dot_rows<DP>(sT, kw, qh, ql, lane);
            keys_dot_rows<DP>(dpT, vw, dh, dl, lane);
#pragma unroll
            for (int n = 0; n < 2; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int key = warp * 16 + g + 8 * (i >> 1), q = n * 8 + 2 * t + (i & 1);
                    const bool ok = mk[q * 64 + key] != 0;
                    const float p = ok ? __expf(sT[n][i] * a.scale - lse[q]) : 0.0f;
                    sT[n][i] = p;
                    dpT[n][i] = p * (dpT[n][i] - dr[q]) * a.scale;
                }
            keys_times_rows<DP>(dv, sT, dh, dl, lane);
            keys_times_rows<DP>(dk, dpT, qh, ql, lane);
        }
        __syncthreads();
    }
    if (!warp_live) return;
    const float un = *a.unscale;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int key = warp * 16 + g + 8 * r;
        float *dkp, *dvp;
        if (!slot_tile) {
            // this share's partial sums (the shares are added in order afterwards)
            const int64_t l = static_cast<int64_t>(tile) * kTKeys + key;
            if (l >= a.L) continue;
            const int64_t stride = static_cast<int64_t>(kKvSplit) * a.L * a.kvh * a.D;
            dkp = a.kv_part + ((static_cast<int64_t>(part) * a.L + l) * a.kvh + h) * a.D;
            dvp = dkp + stride;
        } else {
            if (key >= a.k) continue;
            const int64_t row = (static_cast<int64_t>(wslot) * a.k + key) * a.kvh + h;
            dkp = a.dks + row * a.D;
            dvp = a.dvs + row * a.D;
        }
#pragma unroll
        for (int n = 0; n < NO; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int col = n * 8 + 2 * t + e;
                if (col < a.D) {
                    dkp[col] = dk[n][2 * r + e] * un;
                    dvp[col] = dv[n][2 * r + e] * un;
                }
            }
    }
}

// ------------------------------------------------------------------ backward: dQ

template <int DP>
constexpr size_t q_smem() {
    // [2 stages][2 halves] x (K + V tiles) + masks, then q and dO rows (hi, lo) of four heads, lse, dr
    return static_cast<size_t>(8) * kTKeys * trow<DP>() + 4 * 1024 + static_cast<size_t>(4) * 64 * trow<DP>() +
           2 * 64 * sizeof(float);
}

template <int DP>
__global__ void __launch_bounds__(256, 1) train_attn_bwd_q_kernel(const TrainAttnArgs a) {
    constexpr int RB = trow<DP>(), KV = kTKeys * RB, NO = DP / 8;
    extern __shared__ __align__(16) char sm[];
    uint8_t *mbase = reinterpret_cast<uint8_t *>(sm + 8 * KV);
    char *qs_hi = sm + 8 * KV + 4 * 1024, *qs_lo = qs_hi + 64 * RB, *ds_hi = qs_lo + 64 * RB, *ds_lo = ds_hi + 64 * RB;
    float *lse = reinterpret_cast<float *>(ds_lo + 64 * RB), *dr = lse + 64;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, g = lane >> 2, t = lane & 3;
    const int hw = warp & 3, kh = warp >> 2;
    const int w = blockIdx.x, h = blockIdx.y;
    const bool head_live = hw < a.g;
    const int ntiles = a.Lp / kTKeys + 1;
    const int iters = (ntiles + 1) / 2;
    auto kbuf = [&](int st, int half) { return sm + ((st * 2 + half) * 2) * KV; };
    auto vbuf = [&](int st, int half) { return sm + ((st * 2 + half) * 2 + 1) * KV; };
    auto mbuf = [&](int st, int half) { return mbase + (st * 2 + half) * 1024; };

    stage_rows<DP>(a, a.qh, a.ql, h, w, qs_hi, qs_lo, threadIdx.x, blockDim.x);
    stage_rows<DP>(a, a.doh, a.dol, h, w, ds_hi, ds_lo, threadIdx.x, blockDim.x);
    if (threadIdx.x < 32) {
        const int which = threadIdx.x >> 4, c = threadIdx.x & 15;  // 4 heads x 16 rows = 16 chunks of 4
        const int j = c >> 2;
        const bool live = j < a.g;
        const int64_t row0 = ((static_cast<int64_t>(h) * a.W + w) * a.g + (live ? j : 0)) * 16;
        cp_async16((which ? dr : lse) + c * 4, (which ? a.dr : a.lse_in) + row0 + (c & 3) * 4, live ? 16 : 0);
    }
    for (int half = 0; half < 2; ++half)
        stage_key_tile<DP>(a, h, w, half, kbuf(0, half), vbuf(0, half), mbuf(0, half), threadIdx.x, blockDim.x);
    cp_async_commit();

    float dq[NO][4];
#pragma unroll
    for (int n = 0; n < NO; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) dq[n][i] = 0.0f;
    for (int it = 0; it < iters; ++it) {
        const int st = it & 1;
        if (it + 1 < iters) {
            for (int half = 0; half < 2; ++half)
                stage_key_tile<DP>(a, h, w, 2 * (it + 1) + half, kbuf(st ^ 1, half), vbuf(st ^ 1, half),
                                   mbuf(st ^ 1, half), threadIdx.x, blockDim.x);
            cp_async_commit();
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const int tile = 2 * it + kh;
        const uint8_t *mk = mbuf(st, kh);
        if (head_live && tile < ntiles && tile_any(mk, lane)) {
            float s[8][4], dp[8][4];
#pragma unroll
            for (int n = 0; n < 8; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) s[n][i] = dp[n][i] = 0.0f;
            rows_times_keys<DP>(s, qs_hi + hw * 16 * RB, qs_lo + hw * 16 * RB, kbuf(st, kh), lane);
            rows_times_keys<DP>(dp, ds_hi + hw * 16 * RB, ds_lo + hw * 16 * RB, vbuf(st, kh), lane);
#pragma unroll
            for (int n = 0; n < 8; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int row = g + 8 * (i >> 1), key = n * 8 + 2 * t + (i & 1);
                    const bool ok = mk[row * 64 + key] != 0;
                    const float p = ok ? __expf(s[n][i] * a.scale - lse[hw * 16 + row]) : 0.0f;
                    s[n][i] = p * (dp[n][i] - dr[hw * 16 + row]) * a.scale;  // dS
                }
            // dQ += dS . K: K rows as the (keys x DP) B operand
            probs_times_values<DP>(dq, s, kbuf(st, kh), lane);
        }
        __syncthreads();
    }
    // the two halves' dQ meet in the key-tile area, summed in a fixed order
    constexpr int X = NO * 4;
    float *xch = reinterpret_cast<float *>(sm) + (hw * X) * 32 + lane;
    if (head_live && kh == 1) {
#pragma unroll
        for (int n = 0; n < NO; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) xch[(n * 4 + i) * 32] = dq[n][i];
    }
    __syncthreads();
    if (!head_live || kh == 1) return;
    const float un = *a.unscale;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const int slot = g + 8 * r;
        if (slot >= a.k) continue;
        float *dst = a.dq + ((((static_cast<int64_t>(w) * a.k + slot) * a.kvh + h) * a.g + hw) * a.D);
#pragma unroll
        for (int n = 0; n < NO; ++n)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int col = n * 8 + 2 * t + e;
                if (col < a.D) dst[col] = (dq[n][2 * r + e] + xch[(n * 4 + 2 * r + e) * 32]) * un;
            }
    }
}

// ------------------------------------------------------------------ operand preparation

// fp32 rows [W][k][kvh][g][D] (times *factor when given) -> fp16 hi + lo rows
// [kvh][W][g][16][DP], zero padded; also the forward's lse rows set to +inf.
__global__ void pack_query_kernel(const float *__restrict__ x, int W, int k, int kvh, int g, int D, int DP,
                                  const float *__restrict__ factor, __half *__restrict__ hi, __half *__restrict__ lo,
                                  float *__restrict__ lse_init) {
    const int64_t total = static_cast<int64_t>(kvh) * W * g * 16 * DP;
    const float f = factor ? *factor : 1.0f;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int e = static_cast<int>(i % DP);
        const int64_t row = i / DP;  // (h, w, j, s)
        const int s = static_cast<int>(row % 16);
        const int64_t hwj = row / 16;
        const int j = static_cast<int>(hwj % g);
        const int64_t hw = hwj / g;
        const int w = static_cast<int>(hw % W), h = static_cast<int>(hw / W);
        float v = 0.0f;
        if (s < k && e < D) v = __fmul_rn(x[((((static_cast<int64_t>(w) * k + s) * kvh + h) * g + j) * D) + e], f);
        const __half vh = __float2half_rn(v);
        hi[i] = vh;
        lo[i] = __float2half_rn(__fsub_rn(v, __half2float(vh)));
        if (lse_init && e == 0) lse_init[row] = INFINITY;
    }
}

// fp32 K and V rows -> fp16 rows [kvh][R][DP] (exact: the values are fp16 already).
// Context: source [L][kvh][D], R = Lp, row r = key r.  Slots: source [W][k][kvh][D],
// R = W x 16, row r = (window r / 16, slot r % 16).
__global__ void pack_kv_kernel(const float *__restrict__ ksrc, const float *__restrict__ vsrc, int kvh, int D, int DP,
                               int64_t R, int live_rows, int slots, int k, __half *__restrict__ kdst,
                               __half *__restrict__ vdst) {
    const int64_t total = static_cast<int64_t>(kvh) * R * DP;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int e = static_cast<int>(i % DP);
        const int64_t r = (i / DP) % R;
        const int h = static_cast<int>(i / (DP * R));
        int64_t src = -1;
        if (e < D) {
            if (!slots) {
                if (r < live_rows) src = (r * kvh + h) * D + e;
            } else {
                const int64_t w = r / 16;
                const int s = static_cast<int>(r % 16);
                if (s < k) src = ((w * k + s) * kvh + h) * D + e;
            }
        }
        kdst[i] = __float2half_rn(src >= 0 ? ksrc[src] : 0.0f);
        vdst[i] = __float2half_rn(src >= 0 ? vsrc[src] : 0.0f);
    }
}

// Masks: ctx [W][16][Lp] from allowed (element strides sw, ss, sl; 0 broadcasts),
// slots [16][16] from slot_allowed (strides s0, s1) or all allowed.
__global__ void pack_masks_kernel(const uint8_t *__restrict__ allowed, int64_t sw, int64_t ss, int64_t sl, int W, int k,
                                  int L, int Lp, uint8_t *__restrict__ mctx, const uint8_t *__restrict__ slot_allowed,
                                  int64_t s0, int64_t s1, uint8_t *__restrict__ mslot) {
    const int64_t total = static_cast<int64_t>(W) * 16 * Lp;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total + 256;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        if (i < total) {
            const int l = static_cast<int>(i % Lp);
            const int s = static_cast<int>((i / Lp) % 16);
            const int64_t w = i / (static_cast<int64_t>(Lp) * 16);
            mctx[i] = (s < k && l < L && allowed[w * sw + s * ss + l * sl]) ? 1 : 0;
        } else {
            const int s = static_cast<int>((i - total) / 16), t = static_cast<int>((i - total) % 16);
            mslot[s * 16 + t] = (s < k && t < k && (!slot_allowed || slot_allowed[s * s0 + t * s1])) ? 1 : 0;
        }
    }
}

// Largest |g| as the bits of a non-negative float (ordered like unsigned integers).
__global__ void abs_max_kernel(const float *__restrict__ g, int64_t n, unsigned *__restrict__ out) {
    unsigned m = 0;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        m = max(m, __float_as_uint(fabsf(g[i])));
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, d));
    if ((threadIdx.x & 31) == 0 && m) atomicMax(out, m);
}

// 2^-ceil(log2 m) for the largest magnitude m (1 when m is 0, subnormal or not finite).
__device__ __forceinline__ float pow2_factor(unsigned bits) {
    const unsigned e = (bits >> 23) & 0xffu;
    if (e == 0u || e == 0xffu) return 1.0f;
    int c = static_cast<int>(e) - 127 + ((bits & 0x7fffffu) ? 1 : 0);
    int fe = 127 - c;
    fe = fe < 1 ? 1 : (fe > 254 ? 254 : fe);
    return __uint_as_float(static_cast<unsigned>(fe) << 23);
}

__global__ void grad_factor_kernel(const unsigned *__restrict__ maxbits, float *__restrict__ factor,
                                   float *__restrict__ unscale) {
    const float f = pow2_factor(*maxbits);
    *factor = f;
    *unscale = __frcp_rn(f);  // exact: a power of two
}

// dr[h][w][j][s] = sum_e (dO * factor)[row] * O[row] (0 for padding rows): one warp per row.
__global__ void grad_rowdot_kernel(const float *__restrict__ dout, const float *__restrict__ out,
                                   const float *__restrict__ factor, int W, int k, int kvh, int g, int D,
                                   float *__restrict__ dr) {
    const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row >= static_cast<int64_t>(kvh) * W * g * 16) return;
    const int s = static_cast<int>(row % 16);
    const int64_t hwj = row / 16;
    const int j = static_cast<int>(hwj % g);
    const int w = static_cast<int>((hwj / g) % W), h = static_cast<int>(hwj / g / W);
    float acc = 0.0f;
    if (s < k) {
        const float f = *factor;
        const int64_t base = (((static_cast<int64_t>(w) * k + s) * kvh + h) * g + j) * D;
        for (int e = lane; e < D; e += 32) acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(dout[base + e], f), out[base + e]));
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, d));
    }
    if (lane == 0) dr[row] = acc;
}

// dK, dV of the context: the window shares' partial sums added in share order.
__global__ void kv_share_sum_kernel(const float *__restrict__ part, int64_t n, float *__restrict__ dk,
                                    float *__restrict__ dv) {
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float sk = 0.0f, sv = 0.0f;
#pragma unroll
        for (int p = 0; p < kKvSplit; ++p) {
            sk = __fadd_rn(sk, part[p * n + i]);
            sv = __fadd_rn(sv, part[(kKvSplit + p) * n + i]);
        }
        dk[i] = sk;
        dv[i] = sv;
    }
}

static unsigned pack_grid(int64_t n) {
    const int64_t b = (n + 255) / 256;
    return static_cast<unsigned>(b < 148 * 32 ? (b > 0 ? b : 1) : 148 * 32);
}

template <int DP>
static int launch_train_attn(const TrainAttnArgs &a, bool backward, cudaStream_t stream) {
    if (!backward) {
        const size_t smem = fwd_smem<DP>();
        auto kern = train_attn_fwd_kernel<DP>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
            cudaSuccess)
            return BD_ERR_LAUNCH;
        kern<<<dim3(a.W, a.kvh), 256, smem, stream>>>(a);
        BD_CHECK_LAUNCH();
        return BD_OK;
    }
    {
        const size_t smem = kv_smem<DP>();
        auto kern = train_attn_bwd_kv_kernel<DP>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
            cudaSuccess)
            return BD_ERR_LAUNCH;
        kern<<<dim3(a.Lp / kTKeys * kKvSplit + a.W, a.kvh), 128, smem, stream>>>(a);
        BD_CHECK_LAUNCH();
        if (a.L > 0) {
            const int64_t n = static_cast<int64_t>(a.L) * a.kvh * a.D;
            kv_share_sum_kernel<<<pack_grid(n), 256, 0, stream>>>(a.kv_part, n, a.dkc, a.dvc);
            BD_CHECK_LAUNCH();
        }
    }
    {
        const size_t smem = q_smem<DP>();
        auto kern = train_attn_bwd_q_kernel<DP>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) !=
            cudaSuccess)
            return BD_ERR_LAUNCH;
        kern<<<dim3(a.W, a.kvh), 256, smem, stream>>>(a);
        BD_CHECK_LAUNCH();
    }
    return BD_OK;
}

static int train_attn(TrainAttnArgs a, bool backward, cudaStream_t stream) {
    if (a.W <= 0 || a.W > 65535 || a.k < 1 || a.k > 16 || a.kvh < 1 || a.kvh > 65535 || a.g < 1 || a.g > 4 ||
        a.D < 1 || a.D > 128 || a.L < 0 || a.Lp != (a.L + kTKeys - 1) / kTKeys * kTKeys || !(a.scale > 0.0f))
        return BD_ERR_INVALID;
    const void *need[] = {a.qh, a.ql, a.ks, a.vs, a.mslot};
    for (const void *p : need)
        if (!p) return BD_ERR_INVALID;
    if (a.Lp > 0 && (!a.kc || !a.vc || !a.mctx)) return BD_ERR_INVALID;
    if (!backward && (!a.o || !a.lse)) return BD_ERR_INVALID;
    if (backward && (!a.doh || !a.dol || !a.lse_in || !a.dr || !a.unscale || !a.dq || !a.dks || !a.dvs ||
                     (a.L > 0 && (!a.dkc || !a.dvc || !a.kv_part))))
        return BD_ERR_INVALID;
    const void *aligned[] = {a.qh, a.ql, a.doh, a.dol, a.kc, a.vc, a.ks, a.vs, a.mctx, a.mslot, a.lse_in, a.dr};
    for (const void *p : aligned)
        if (reinterpret_cast<uintptr_t>(p) & 15) return BD_ERR_ALIGNMENT;
    const int dp = a.D <= 16 ? 16 : a.D <= 32 ? 32 : a.D <= 64 ? 64 : 128;
    switch (dp) {
        case 16: return launch_train_attn<16>(a, backward, stream);
        case 32: return launch_train_attn<32>(a, backward, stream);
        case 64: return launch_train_attn<64>(a, backward, stream);
        default: return launch_train_attn<128>(a, backward, stream);
    }
}

}  // namespace bd

using namespace bd;

extern "C" int bd_train_attention_pack(const float *query, const float *ctx_k, const float *ctx_v,
                                       const float *slot_k, const float *slot_v, const uint8_t *ctx_allowed,
                                       int64_t allowed_stride_w, int64_t allowed_stride_s, int64_t allowed_stride_l,
                                       const uint8_t *slot_allowed, int64_t slot_stride_s, int64_t slot_stride_t,
                                       int windows, int slots, int kv_heads, int groups, int head_dim, int keys,
                                       void *q_hi, void *q_lo, void *kc, void *vc, void *ks, void *vs,
                                       uint8_t *ctx_mask, uint8_t *slot_mask, float *lse, bd_stream_t stream) {
    if (windows < 1 || slots < 1 || slots > 16 || kv_heads < 1 || groups < 1 || groups > 4 || head_dim < 1 ||
        head_dim > 128 || keys < 0)
        return BD_ERR_INVALID;
    if (!query || !slot_k || !slot_v || !q_hi || !q_lo || !ks || !vs || !slot_mask || !lse ||
        (keys > 0 && (!ctx_k || !ctx_v || !ctx_allowed || !kc || !vc || !ctx_mask)))
        return BD_ERR_INVALID;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int dp = head_dim <= 16 ? 16 : head_dim <= 32 ? 32 : head_dim <= 64 ? 64 : 128;
    const int lp = (keys + kTKeys - 1) / kTKeys * kTKeys;
    const int64_t nq = static_cast<int64_t>(kv_heads) * windows * groups * 16 * dp;
    pack_query_kernel<<<pack_grid(nq), 256, 0, st>>>(query, windows, slots, kv_heads, groups, head_dim, dp, nullptr,
                                                     static_cast<__half *>(q_hi), static_cast<__half *>(q_lo), lse);
    BD_CHECK_LAUNCH();
    if (lp > 0) {
        pack_kv_kernel<<<pack_grid(static_cast<int64_t>(kv_heads) * lp * dp), 256, 0, st>>>(
            ctx_k, ctx_v, kv_heads, head_dim, dp, lp, keys, 0, slots, static_cast<__half *>(kc),
            static_cast<__half *>(vc));
        BD_CHECK_LAUNCH();
    }
    pack_kv_kernel<<<pack_grid(static_cast<int64_t>(kv_heads) * windows * 16 * dp), 256, 0, st>>>(
        slot_k, slot_v, kv_heads, head_dim, dp, static_cast<int64_t>(windows) * 16, 0, 1, slots,
        static_cast<__half *>(ks), static_cast<__half *>(vs));
    BD_CHECK_LAUNCH();
    pack_masks_kernel<<<pack_grid(static_cast<int64_t>(windows) * 16 * lp + 256), 256, 0, st>>>(
        ctx_allowed ? ctx_allowed : slot_mask, allowed_stride_w, allowed_stride_s, allowed_stride_l, windows, slots,
        keys, lp, ctx_mask ? ctx_mask : slot_mask, slot_allowed, slot_stride_s, slot_stride_t, slot_mask);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_train_attention_pack_grad(const float *dout, const float *out, int windows, int slots,
                                            int kv_heads, int groups, int head_dim, void *d_hi, void *d_lo, float *dr,
                                            float *scalars, bd_stream_t stream) {
    if (windows < 1 || slots < 1 || slots > 16 || kv_heads < 1 || groups < 1 || groups > 4 || head_dim < 1 ||
        head_dim > 128 || !dout || !out || !d_hi || !d_lo || !dr || !scalars)
        return BD_ERR_INVALID;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int dp = head_dim <= 16 ? 16 : head_dim <= 32 ? 32 : head_dim <= 64 ? 64 : 128;
    // scalars: [0] the largest |dout| (bits), [1] the power-of-two factor, [2] its inverse
    unsigned *maxbits = reinterpret_cast<unsigned *>(scalars);
    if (cudaMemsetAsync(maxbits, 0, sizeof(unsigned), st) != cudaSuccess) return BD_ERR_LAUNCH;
    const int64_t n = static_cast<int64_t>(windows) * slots * kv_heads * groups * head_dim;
    abs_max_kernel<<<pack_grid(n), 256, 0, st>>>(dout, n, maxbits);
    BD_CHECK_LAUNCH();
    grad_factor_kernel<<<1, 1, 0, st>>>(maxbits, scalars + 1, scalars + 2);
    BD_CHECK_LAUNCH();
    const int64_t nq = static_cast<int64_t>(kv_heads) * windows * groups * 16 * dp;
    pack_query_kernel<<<pack_grid(nq), 256, 0, st>>>(dout, windows, slots, kv_heads, groups, head_dim, dp,
                                                     scalars + 1, static_cast<__half *>(d_hi),
                                                     static_cast<__half *>(d_lo), nullptr);
    BD_CHECK_LAUNCH();
    const int64_t rows = static_cast<int64_t>(kv_heads) * windows * groups * 16;
    grad_rowdot_kernel<<<static_cast<unsigned>((rows * 32 + 255) / 256), 256, 0, st>>>(
        dout, out, scalars + 1, windows, slots, kv_heads, groups, head_dim, dr);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_train_attention_forward(const void *q_hi, const void *q_lo, const void *ctx_k, const void *ctx_v,
                                          const void *slot_k, const void *slot_v, const uint8_t *ctx_mask,
                                          const uint8_t *slot_mask, int windows, int slots, int kv_heads,
                                          int groups, int head_dim, int keys, float scale, float *out, float *lse,
                                          uint8_t *tile_live, bd_stream_t stream) {
    TrainAttnArgs a = {};
    a.qh = static_cast<const __half *>(q_hi);
    a.ql = static_cast<const __half *>(q_lo);
    a.kc = static_cast<const __half *>(ctx_k);
    a.vc = static_cast<const __half *>(ctx_v);
    a.ks = static_cast<const __half *>(slot_k);
    a.vs = static_cast<const __half *>(slot_v);
    a.mctx = ctx_mask;
    a.mslot = slot_mask;
    a.W = windows;
    a.k = slots;
    a.kvh = kv_heads;
    a.g = groups;
    a.D = head_dim;
    a.L = keys;
    a.Lp = (keys + kTKeys - 1) / kTKeys * kTKeys;
    a.scale = scale;
    a.o = out;
    a.lse = lse;
    a.live = tile_live;
    return train_attn(a, false, static_cast<cudaStream_t>(stream));
}

extern "C" int bd_train_attention_backward(const void *q_hi, const void *q_lo, const void *ctx_k, const void *ctx_v,
                                           const void *slot_k, const void *slot_v, const uint8_t *ctx_mask,
                                           const uint8_t *slot_mask, const void *dout_hi, const void *dout_lo,
                                           const float *lse, const float *dr, const float *unscale,
                                           const uint8_t *tile_live, int windows, int slots, int kv_heads,
                                           int groups, int head_dim, int keys, float scale, float *dq, float *d_ctx_k,
                                           float *d_ctx_v, float *d_slot_k, float *d_slot_v, float *kv_partials,
                                           bd_stream_t stream) {
    TrainAttnArgs a = {};
    a.qh = static_cast<const __half *>(q_hi);
    a.ql = static_cast<const __half *>(q_lo);
    a.kc = static_cast<const __half *>(ctx_k);
    a.vc = static_cast<const __half *>(ctx_v);
    a.ks = static_cast<const __half *>(slot_k);
    a.vs = static_cast<const __half *>(slot_v);
    a.mctx = ctx_mask;
    a.mslot = slot_mask;
    a.doh = static_cast<const __half *>(dout_hi);
    a.dol = static_cast<const __half *>(dout_lo);
    a.lse_in = lse;
    a.dr = dr;
    a.unscale = unscale;
    a.live = const_cast<uint8_t *>(tile_live);
    a.W = windows;
    a.k = slots;
    a.kvh = kv_heads;
    a.g = groups;
    a.D = head_dim;
    a.L = keys;
    a.Lp = (keys + kTKeys - 1) / kTKeys * kTKeys;
    a.scale = scale;
    a.dq = dq;
    a.dkc = d_ctx_k;
    a.dvc = d_ctx_v;
    a.dks = d_slot_k;
    a.dvs = d_slot_v;
    a.kv_part = kv_partials;
    return train_attn(a, true, static_cast<cudaStream_t>(stream));
}
