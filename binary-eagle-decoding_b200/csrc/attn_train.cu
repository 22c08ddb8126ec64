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
//                         over the query tiles that see the tile (every window
//                         for a context tile, its own window for a slot tile),
//                         recomputes P^T from the saved log-sum-exp and
//                         accumulates dV = P^T dO and dK = dS^T Q in registers.
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
    const int tile = blockIdx.x, h = blockIdx.y;
    const bool slot_tile = tile >= nctx;
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
    const int nq = slot_tile ? a.g : (listed ? nlive_s : a.W) * a.g;
    // the query tile qt: its rows (hi, lo of q and dO), mask (16 x 64), lse and dr
    auto stage_q = [&](int st, int qt) {
        const int w = slot_tile ? wslot : (listed ? static_cast<int>(wlist[qt / a.g]) : qt / a.g);
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
            const int64_t l = static_cast<int64_t>(tile) * kTKeys + key;
            if (l >= a.L) continue;
            dkp = a.dkc + (l * a.kvh + h) * a.D;
            dvp = a.dvc + (l * a.kvh + h) * a.D;
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
        kern<<<dim3(a.Lp / kTKeys + a.W, a.kvh), 128, smem, stream>>>(a);
        BD_CHECK_LAUNCH();
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
                     (a.L > 0 && (!a.dkc || !a.dvc))))
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
                                           float *d_ctx_v, float *d_slot_k, float *d_slot_v, bd_stream_t stream) {
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
    return train_attn(a, true, static_cast<cudaStream_t>(stream));
}
