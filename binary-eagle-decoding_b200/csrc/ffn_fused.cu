// HE4 SwiGLU block for decode sizes (tokens <= 16) in two launches:
//   y = residual + down(silu(gate(n)) * up(n)),  n = rms(x, norm) (w1a1_eagle/model.py:220-223),
// every projection an HE4 Projection.forward (model.py:128-150) on packed signs.
//
// Gate/up kernel (clusters of CA CTAs, one CTA per SM):
//   * before griddepcontrol.wait: each CTA bulk-copies its gate/up sign slice
//     (W8 words of its n-tile pairs, all of K) from this GPU's own memory into
//     shared memory;
//   * the cluster quantizes x: CTA r reads columns [r H / CA, (r + 1) H / CA),
//     the per-token sums of squares of the rms are exchanged through
//     distributed shared memory, and every CTA pushes its A4 codes (C16 layout)
//     into every CTA of the cluster;
//   * int8 m16n8k32 MMAs from shared memory (warps take (pair, 512-column
//     group) units and meet in shared-memory integer sums); SwiGLU and the A8
//     quantizer of the down input in the epilogue, which writes the codes to a
//     C16 buffer in global memory and this CTA's per-token code sums.
// Down kernel (PDL: its CTAs stream their D8 down signs into shared memory
// while the gate/up kernel runs; clusters of CB CTAs):
//   * a cluster owns a range of output n-tiles; its CTAs split K (the F rows)
//     in 4-k-step groups, each reads its slice of the codes, multiplies all of
//     the cluster's n-tiles, and the CTAs' exact integer partial dots meet
//     through distributed shared memory; each CTA finishes a share of the
//     n-tiles (HE4 epilogue + residual).
// No atomics leave a CTA, nothing is left in the workspace between calls, and
// every sum is exact or in a fixed order, so results are deterministic.  The
// only waits are the bounded waits of each CTA for its own bulk copies
// (BD_FLAG_TIMEOUT when one runs out) and the cluster barriers.
#include <algorithm>
#include <map>
#include <mutex>
#include <tuple>

#include "kernels.cuh"

namespace bd {

constexpr int kGuWarps = 16;  // gate/up kernel
constexpr int kGuThreads = kGuWarps * 32;
constexpr int kDnWarps = 8;   // down kernel
constexpr int kDnThreads = kDnWarps * 32;
constexpr int kFuTokens = 16;
constexpr int kDnNt = 12;  // output n-tiles per cluster of the down kernel, at most
constexpr uint32_t kFuSpin = 1u << 22;

struct GuArgs {
    int tokens;
    int64_t hidden, inter;
    const uint32_t *gu;   // W8 gate/up words, n-tile pairs interleaved: [np][2][ng][32][4]
    int64_t np, ng;       // n-tile pairs, W8 word groups of K
    const float *x, *norm_w;
    float eps;
    const float *gain_gu, *bound_gu, *gain_dn, *bound_dn;
    const float *scale_g, *mid_g, *scale_u, *mid_u;
    float *hidden_out;
    int8_t *hcodes;       // C16 codes of the down input: [inter / 32][32][16]
    int32_t *hsum;        // [gridDim][16] per-CTA code sums of the down input
    int32_t *flags;
    int pairs_max, cols_max;
};

struct DnArgs {
    int tokens;
    int64_t hidden, inter;
    const uint8_t *dn;    // D8 down bytes: [hidden / 8][g4][32][4]
    int64_t nt, g4;       // output n-tiles, 4-k-step groups of K
    const int8_t *hcodes;
    const int32_t *hsum;
    int gu_ctas;
    const float *bound_dn, *scale_d, *mid_d, *residual;
    float *y;
    int32_t *flags;
    int groups_max;
};

// ---- cluster helpers
__device__ __forceinline__ uint32_t fu_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}
__device__ __forceinline__ void fu_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t fu_remote(const void *local, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(out) : "r"(smem_u32(local)), "r"(rank));
    return out;
}
__device__ __forceinline__ void fu_st_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared::cluster.u32 [%0], %1;\n" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void fu_st_f32(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;\n" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ int fu_ld_s32(uint32_t addr) {
    int v;
    asm volatile("ld.shared::cluster.s32 %0, [%1];\n" : "=r"(v) : "r"(addr) : "memory");
    return v;
}
// D8 nibble -> one B register of an m16n8k32 k-step: bit j -> byte j (0 or 1).
__device__ __forceinline__ uint32_t fu_nibble(uint32_t nib) { return (nib * 0x00204081u) & 0x01010101u; }
__device__ __forceinline__ uint32_t fu_word(const uint4 &v, int q) { return q == 0 ? v.x : q == 1 ? v.y : q == 2 ? v.z : v.w; }
__host__ __device__ __forceinline__ uint32_t fu_al(uint32_t n) { return (n + 127u) & ~127u; }

// ------------------------------------------------------------------ gate/up kernel

// Dynamic shared memory, every piece 128-byte aligned: W8 words of this CTA's
// pairs, C16 codes of x, gate/up integer sums [pairs][2][4][32], the x slice
// [16][cols_max], the gain and norm slices, five per-row epilogue vectors.
struct GuSmem {
    uint32_t gu, xc, red, x, gain, norm, prm, bytes;
};
__host__ __device__ inline GuSmem gu_carve(int pairs_max, int64_t ng, int cols_max) {
    GuSmem s{};
    uint32_t o = 0;
    s.gu = o;
    o += fu_al(static_cast<uint32_t>(pairs_max) * 2u * static_cast<uint32_t>(ng) * 512u);
    s.xc = o;
    o += fu_al(static_cast<uint32_t>(ng) * 16u * 512u);
    s.red = o;
    o += fu_al(static_cast<uint32_t>(pairs_max) * 2u * 4u * 32u * 4u);
    s.x = o;
    o += fu_al(static_cast<uint32_t>(kFuTokens) * static_cast<uint32_t>(cols_max) * 4u);
    s.gain = o;
    o += fu_al(static_cast<uint32_t>(cols_max) * 4u);
    s.norm = o;
    o += fu_al(static_cast<uint32_t>(cols_max) * 4u);
    s.prm = o;
    o += fu_al(5u * static_cast<uint32_t>(pairs_max) * 8u * 4u);
    s.bytes = o;
    return s;
}

template <int C>
__global__ void __launch_bounds__(kGuThreads, 1) ffn_gu_kernel(const GuArgs a) {
    extern __shared__ __align__(128) uint8_t fu_raw[];
    __shared__ __align__(8) uint64_t bar_w, bar_x;
    __shared__ float ssq[C][kFuTokens];
    __shared__ int csx[C][kFuTokens];
    __shared__ int cs_loc[kFuTokens], hs_loc[kFuTokens];
    __shared__ int abort_copy;
    const GuSmem sm = gu_carve(a.pairs_max, a.ng, a.cols_max);
    uint8_t *sgu = fu_raw + sm.gu, *sxc = fu_raw + sm.xc;
    int *red = reinterpret_cast<int *>(fu_raw + sm.red);
    float *sx = reinterpret_cast<float *>(fu_raw + sm.x);
    float *sgain = reinterpret_cast<float *>(fu_raw + sm.gain), *snorm = reinterpret_cast<float *>(fu_raw + sm.norm);
    float *sprm = reinterpret_cast<float *>(fu_raw + sm.prm);  // [5][pairs_max * 8]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int T = a.tokens;
    const int64_t H = a.hidden, F = a.inter;
    const uint32_t r = fu_rank();
    const int64_t p0 = blockIdx.x * a.np / gridDim.x, p1 = (blockIdx.x + 1) * a.np / gridDim.x;
    const int npc = static_cast<int>(p1 - p0);
    const int64_t c0 = r * H / C, c1 = (r + 1) * H / C;
    const int cw = static_cast<int>(c1 - c0);
    const int groups = cw / 4;
    const int pstride = a.pairs_max * 8;

    // ---------------- prologue: weights only (nothing an earlier kernel writes)
    if (tid == 0) {
        mbar_init(&bar_w, 1);
        mbar_init(&bar_x, 1);
        mbar_init_fence();
        abort_copy = 0;
        const uint32_t gu_bytes = static_cast<uint32_t>(npc) * 2u * static_cast<uint32_t>(a.ng) * 512u;
        const uint32_t col_bytes = static_cast<uint32_t>(cw) * 4u, row_bytes = static_cast<uint32_t>(npc) * 32u;
        mbar_expect_tx(&bar_w, gu_bytes + col_bytes * (a.norm_w ? 2u : 1u) + (npc ? 5u * row_bytes : 0u));
        if (gu_bytes) bulk_load(sgu, a.gu + p0 * 2 * a.ng * 128, gu_bytes, &bar_w);
        bulk_load(sgain, a.gain_gu + c0, col_bytes, &bar_w);
        if (a.norm_w) bulk_load(snorm, a.norm_w + c0, col_bytes, &bar_w);
        if (npc) {
            const float *src[5] = {a.scale_g, a.mid_g, a.scale_u, a.mid_u, a.gain_dn};
#pragma unroll
            for (int i = 0; i < 5; ++i) bulk_load(sprm + i * pstride, src[i] + p0 * 8, row_bytes, &bar_w);
        }
    }
    for (int i = tid; i < npc * 2 * 4 * 32; i += kGuThreads) red[i] = 0;
    if (tid < kFuTokens) cs_loc[tid] = hs_loc[tid] = 0;
    // x k-steps beyond H (inside the last 512-column group) read as zero codes
    for (int64_t i = H / 32 * 512 + tid * 16; i < a.ng * 16 * 512; i += kGuThreads * 16)
        *reinterpret_cast<uint4 *>(sxc + i) = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();
    fu_cluster_sync();  // every CTA of the cluster runs before any distributed shared-memory store
    grid_wait();
    grid_launch_dependents();
    if (tid == 0) {  // this CTA's columns of x, one bulk copy per token row
        mbar_expect_tx(&bar_x, static_cast<uint32_t>(T) * static_cast<uint32_t>(cw) * 4u);
        for (int t = 0; t < T; ++t) bulk_load(sx + t * cw, a.x + t * H + c0, static_cast<uint32_t>(cw) * 4u, &bar_x);
    }
    const float b_gu = __ldg(a.bound_gu), b_dn = __ldg(a.bound_dn);
    if ((bad_bound(b_gu) || bad_bound(b_dn)) && blockIdx.x == 0 && tid == 0) set_flag(a.flags, BD_FLAG_BAD_BOUND);
    bool ok = mbar_wait_bounded(&bar_x, 0, kFuSpin) && mbar_wait_bounded(&bar_w, 0, kFuSpin);
    if (!ok) abort_copy = 1;

    // ---------------- x: sums of squares of this CTA's columns, shared with the cluster
    if (a.norm_w && warp < T) {
        const float4 *row = reinterpret_cast<const float4 *>(sx + warp * cw);
        float ss = 0.0f;
        for (int gi = lane; gi < groups; gi += 32) {
            const float4 v = row[gi];
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
        if (lane < C) fu_st_f32(fu_remote(&ssq[r][warp], static_cast<uint32_t>(lane)), ss);
    }
    fu_cluster_sync();

    // ---------------- x: A4 codes of this CTA's columns into every CTA's C16 buffer
    Quant qin;
    qin.init(b_gu, 4);
    bool bad = false;
    float inv[kFuTokens];
#pragma unroll
    for (int t = 0; t < kFuTokens; ++t) {
        float total = 0.0f;
#pragma unroll
        for (int rr = 0; rr < C; ++rr) total += ssq[rr][t];
        inv[t] = a.norm_w ? rsqrtf(total / static_cast<float>(H) + a.eps) : 1.0f;
    }
    for (int e = tid; e < T * groups; e += kGuThreads) {
        const int t = e / groups, gi = e - t * groups;
        const float4 v = reinterpret_cast<const float4 *>(sx + t * cw)[gi];
        const float4 gn = reinterpret_cast<const float4 *>(sgain)[gi];
        float xv[4] = {v.x, v.y, v.z, v.w};
        float scale = 1.0f;
#pragma unroll
        for (int tt = 0; tt < kFuTokens; ++tt)
            if (tt == t) scale = inv[tt];
        if (a.norm_w) {
            const float4 w = reinterpret_cast<const float4 *>(snorm)[gi];
            xv[0] = xv[0] * scale * w.x;
            xv[1] = xv[1] * scale * w.y;
            xv[2] = xv[2] * scale * w.z;
            xv[3] = xv[3] * scale * w.w;
        }
        const float gv[4] = {gn.x, gn.y, gn.z, gn.w};
        uint32_t packed = 0;
        int sum = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float gained = __fmul_rn(xv[j], gv[j]);
            bad |= !isfinite(gained);
            const int c = qin.code(gained);
            sum += c;
            packed |= (static_cast<uint32_t>(c) & 0xFFu) << (8 * j);
        }
        if (sum) atomicAdd(&cs_loc[t], sum);
        const uint8_t *dst = sxc + c16_offset(t, c0 + 4 * gi, 1);
#pragma unroll
        for (int rr = 0; rr < C; ++rr) fu_st_u32(fu_remote(dst, static_cast<uint32_t>(rr)), packed);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) set_flag(a.flags, BD_FLAG_NONFINITE_INPUT);
    __syncthreads();
    if (tid < kFuTokens) {
#pragma unroll
        for (int rr = 0; rr < C; ++rr)
            fu_st_u32(fu_remote(&csx[r][tid], static_cast<uint32_t>(rr)), static_cast<uint32_t>(cs_loc[tid]));
    }
    fu_cluster_sync();  // no distributed shared-memory access after this point

    // ---------------- gate/up: (pair, 512-column group) units over the warps, two
    // independent accumulator chains per matrix (even and odd k-steps)
    const bool aborted = abort_copy != 0;
    if (aborted && tid == 0) set_flag(a.flags, BD_FLAG_TIMEOUT);
    const int units = aborted ? 0 : npc * static_cast<int>(a.ng);
    for (int u = warp; u < units; u += kGuWarps) {
        const int p = u / static_cast<int>(a.ng), j = u - p * static_cast<int>(a.ng);
        const uint4 bg = *reinterpret_cast<const uint4 *>(sgu + ((static_cast<int64_t>(p * 2 + 0) * a.ng + j) * 32 + lane) * 16);
        const uint4 bu = *reinterpret_cast<const uint4 *>(sgu + ((static_cast<int64_t>(p * 2 + 1) * a.ng + j) * 32 + lane) * 16);
        int acc[2][2][4] = {};
#pragma unroll
        for (int s = 0; s < 16; ++s) {
            const uint4 A = *reinterpret_cast<const uint4 *>(sxc + ((static_cast<int64_t>(j) * 16 + s) * 32 + lane) * 16);
            const uint32_t wg = fu_word(bg, s >> 2), wu = fu_word(bu, s >> 2);
            const int sh = 2 * (s & 3);
            mma_s8_16832(acc[0][s & 1], A.x, A.y, A.z, A.w, (wg >> sh) & 0x01010101u, (wg >> (sh + 1)) & 0x01010101u);
            mma_s8_16832(acc[1][s & 1], A.x, A.y, A.z, A.w, (wu >> sh) & 0x01010101u, (wu >> (sh + 1)) & 0x01010101u);
        }
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int i = 0; i < 4; ++i)
                atomicAdd(&red[((p * 2 + m) * 4 + i) * 32 + lane], acc[m][0][i] + acc[m][1][i]);
    }
    __syncthreads();

    // ---------------- epilogue: h = silu(g) * u, A8 codes of h (C16, global) and their sums
    Quant qdn;
    qdn.init(b_dn, 8);
    int csin[2], lsum[2] = {0, 0};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int tok = g + 8 * h;
        int s = 0;
        if (tok < T)
#pragma unroll
            for (int rr = 0; rr < C; ++rr) s += csx[rr][tok];
        csin[h] = s;
    }
    bad = false;
    for (int p = warp; p < npc; p += kGuWarps) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int lo = p * 8 + 2 * t4 + e;  // row within this CTA's slice
            const int64_t o = p0 * 8 + lo;
            if (o >= F) continue;
            const float sg = sprm[0 * pstride + lo], mg = sprm[1 * pstride + lo];
            const float su = sprm[2 * pstride + lo], mu = sprm[3 * pstride + lo];
            const float gd = sprm[4 * pstride + lo];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int tok = g + 8 * h;
                if (tok >= T) continue;
                const int i = 2 * h + e;
                const int Dg = 2 * red[((p * 2 + 0) * 4 + i) * 32 + lane] - csin[h];
                const int Du = 2 * red[((p * 2 + 1) * 4 + i) * 32 + lane] - csin[h];
                const float gv = he4_value(Dg, sg, qin.step, csin[h], mg);
                const float uv = he4_value(Du, su, qin.step, csin[h], mu);
                const float hv = __fmul_rn(silu(gv), uv);
                if (a.hidden_out) a.hidden_out[tok * F + o] = hv;
                const float gained = __fmul_rn(hv, gd);
                bad |= !isfinite(gained);
                const int code = qdn.code(gained);
                lsum[h] += code;
                a.hcodes[c16_offset(tok, o, 1)] = static_cast<int8_t>(code);
            }
        }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) set_flag(a.flags, BD_FLAG_NONFINITE_INPUT);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        int v = lsum[h];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if (t4 == 0 && g + 8 * h < T && v) atomicAdd(&hs_loc[g + 8 * h], v);  // shared, exact
    }
    __syncthreads();
    if (tid < kFuTokens) a.hsum[blockIdx.x * kFuTokens + tid] = hs_loc[tid];
    if (aborted && tid == 0) {  // copies still in flight land before exit
        mbar_wait_bounded(&bar_w, 0, kFuSpin);
        mbar_wait_bounded(&bar_x, 0, kFuSpin);
    }
}

// ------------------------------------------------------------------ down kernel

// Dynamic shared memory, 128-byte aligned pieces: D8 bytes of the cluster's
// n-tiles x this CTA's groups [kDnNt][groups_max][32][4], the codes of this CTA's
// k-steps [4 groups_max][32][16], the integer partial dots [kDnNt][4][32], the
// gate/up CTAs' code sums [gu_ctas][16], and for the n-tiles this CTA finishes
// (at most kDnNt) their scale, midpoint and residual rows [16][kDnNt * 8].
struct DnSmem {
    uint32_t dn, hc, red, hs, scale, mid, res, bytes;
};
__host__ __device__ inline DnSmem dn_carve(int groups_max, int gu_ctas) {
    DnSmem s{};
    uint32_t o = 0;
    s.dn = o;
    o += fu_al(static_cast<uint32_t>(kDnNt) * static_cast<uint32_t>(groups_max) * 128u);
    s.hc = o;
    o += fu_al(static_cast<uint32_t>(groups_max) * 4u * 512u);
    s.red = o;
    o += fu_al(static_cast<uint32_t>(kDnNt) * 4u * 32u * 4u);
    s.hs = o;
    o += fu_al(static_cast<uint32_t>(gu_ctas) * kFuTokens * 4u);
    s.scale = o;
    o += fu_al(kDnNt * 8u * 4u);
    s.mid = o;
    o += fu_al(kDnNt * 8u * 4u);
    s.res = o;
    o += fu_al(static_cast<uint32_t>(kFuTokens) * kDnNt * 8u * 4u);
    s.bytes = o;
    return s;
}

template <int C>
__global__ void __launch_bounds__(kDnThreads, 1) ffn_dn_kernel(const DnArgs a) {
    extern __shared__ __align__(128) uint8_t fu_raw[];
    __shared__ __align__(8) uint64_t bar_w, bar_x;
    __shared__ int hsum[kFuTokens];
    __shared__ int abort_copy;
    const DnSmem sm = dn_carve(a.groups_max, a.gu_ctas);
    const uint32_t *sdn = reinterpret_cast<const uint32_t *>(fu_raw + sm.dn);
    const uint8_t *shc = fu_raw + sm.hc;
    int *red = reinterpret_cast<int *>(fu_raw + sm.red);
    const int *shs = reinterpret_cast<const int *>(fu_raw + sm.hs);
    float *sscale = reinterpret_cast<float *>(fu_raw + sm.scale), *smid = reinterpret_cast<float *>(fu_raw + sm.mid);
    float *sres = reinterpret_cast<float *>(fu_raw + sm.res);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int T = a.tokens;
    const int64_t H = a.hidden;
    const uint32_t r = fu_rank();
    const int64_t Q = gridDim.x / C, cl = blockIdx.x / C;
    const int64_t n0 = cl * a.nt / Q, n1 = (cl + 1) * a.nt / Q;
    const int ntc = static_cast<int>(n1 - n0);
    const int64_t g0 = r * a.g4 / C, g1 = (r + 1) * a.g4 / C;
    const int ngc = static_cast<int>(g1 - g0);
    const int64_t nks = a.inter / 32;
    const int64_t s0 = 4 * g0, s1 = 4 * g1 < nks ? 4 * g1 : nks;
    const int f0 = static_cast<int>(r * ntc / C), f1 = static_cast<int>((r + 1) * ntc / C);
    const uint32_t fin_bytes = static_cast<uint32_t>(f1 - f0) * 32u;  // finished rows x 4 bytes

    // ---------------- prologue: the down signs and epilogue vectors (weights) before the wait
    if (tid == 0) {
        mbar_init(&bar_w, 1);
        mbar_init(&bar_x, 1);
        mbar_init_fence();
        abort_copy = 0;
        const uint32_t row_bytes = static_cast<uint32_t>(ngc) * 128u;
        mbar_expect_tx(&bar_w, row_bytes * static_cast<uint32_t>(ntc) + 2u * fin_bytes);
        if (row_bytes)
            for (int n = 0; n < ntc; ++n)
                bulk_load(fu_raw + sm.dn + n * row_bytes, a.dn + ((n0 + n) * a.g4 + g0) * 128, row_bytes, &bar_w);
        if (fin_bytes) {
            bulk_load(sscale, a.scale_d + (n0 + f0) * 8, fin_bytes, &bar_w);
            bulk_load(smid, a.mid_d + (n0 + f0) * 8, fin_bytes, &bar_w);
        }
    }
    for (int i = tid; i < kDnNt * 4 * 32; i += kDnThreads) red[i] = 0;
    __syncthreads();
    grid_wait();
    grid_launch_dependents();
    if (tid == 0) {  // what the gate/up kernel wrote, and the residual rows this CTA finishes
        const uint32_t hc_bytes = static_cast<uint32_t>(s1 - s0) * 512u;
        const uint32_t hs_bytes = static_cast<uint32_t>(a.gu_ctas) * kFuTokens * 4u;
        const bool res = a.residual && fin_bytes;
        mbar_expect_tx(&bar_x, hc_bytes + hs_bytes + (res ? static_cast<uint32_t>(T) * fin_bytes : 0u));
        if (hc_bytes) bulk_load(fu_raw + sm.hc, a.hcodes + s0 * 512, hc_bytes, &bar_x);
        bulk_load(fu_raw + sm.hs, a.hsum, hs_bytes, &bar_x);
        if (res)
            for (int t = 0; t < T; ++t)
                bulk_load(sres + t * (kDnNt * 8), a.residual + t * H + (n0 + f0) * 8, fin_bytes, &bar_x);
    }
    const bool ok = mbar_wait_bounded(&bar_x, 0, kFuSpin) && mbar_wait_bounded(&bar_w, 0, kFuSpin);
    if (!ok) abort_copy = 1;
    if (tid < 16 * kFuTokens) {  // total code sums: 16 threads per token, then a fixed-order tree
        const int t = tid >> 4, part = tid & 15;
        int sum = 0;
        for (int b = part; b < a.gu_ctas; b += 16) sum += shs[b * kFuTokens + t];
#pragma unroll
        for (int d = 8; d > 0; d >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, d);
        if (part == 0) hsum[t] = sum;
    }
    __syncthreads();
    const bool aborted = abort_copy != 0;
    if (aborted && tid == 0) set_flag(a.flags, BD_FLAG_TIMEOUT);

    // ---------------- partial dots: warps split this CTA's groups, all n-tiles of the cluster
    const int wg0 = warp * ngc / kDnWarps, wg1 = (warp + 1) * ngc / kDnWarps;
    int acc[kDnNt][4] = {};
    if (!aborted) {
        for (int gl = wg0; gl < wg1; ++gl) {
            uint4 A[4];
#pragma unroll
            for (int q = 0; q < 4; ++q)
                A[q] = s0 + 4 * gl + q < s1 ? *reinterpret_cast<const uint4 *>(shc + ((4 * gl + q) * 32 + lane) * 16)
                                            : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int n = 0; n < kDnNt; ++n) {
                if (n < ntc) {
                    const uint32_t bytes = sdn[(n * ngc + gl) * 32 + lane];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint32_t byte = (bytes >> (8 * q)) & 0xFFu;
                        mma_s8_16832(acc[n], A[q].x, A[q].y, A[q].z, A[q].w, fu_nibble(byte & 0xFu), fu_nibble(byte >> 4));
                    }
                }
            }
        }
    }
#pragma unroll
    for (int n = 0; n < kDnNt; ++n)
        if (n < ntc)
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (acc[n][i]) atomicAdd(&red[(n * 4 + i) * 32 + lane], acc[n][i]);
    __syncthreads();
    fu_cluster_sync();  // every CTA's partial dots are complete

    // ---------------- CTA r finishes n-tiles [f0, f1) of the cluster
    Quant qd;
    qd.init(__ldg(a.bound_dn), 8);
    for (int n = f0 + warp; n < f1; n += kDnWarps) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int tok = g + 8 * (i >> 1);
            const int row = (n - f0) * 8 + 2 * t4 + (i & 1);  // within the finished rows
            const int64_t o = (n0 + f0) * 8 + row;
            int d01 = 0;
#pragma unroll
            for (int rr = 0; rr < C; ++rr) d01 += fu_ld_s32(fu_remote(&red[(n * 4 + i) * 32 + lane], static_cast<uint32_t>(rr)));
            if (tok >= T || o >= H) continue;
            const int cs = hsum[tok];
            float yv = he4_value(2 * d01 - cs, sscale[row], qd.step, cs, smid[row]);
            if (a.residual) yv = __fadd_rn(sres[tok * (kDnNt * 8) + row], yv);
            a.y[tok * H + o] = yv;
        }
    }
    fu_cluster_sync();  // no CTA leaves while another still reads its partial dots
    if (aborted && tid == 0) {
        mbar_wait_bounded(&bar_w, 0, kFuSpin);
        mbar_wait_bounded(&bar_x, 0, kFuSpin);
    }
}

// ------------------------------------------------------------------ D8 sign bytes of the down matrix

// Byte ((n * g4 + s / 4) * 32 + lane) * 4 + s % 4, lane = 4 g + t: bit 4 r + j is
// latent[8 n + g, 32 s + 16 r + 4 t + j] >= 0 (0 past the matrix).
__global__ void tile_d8_kernel(const float *__restrict__ latent, int64_t rows, int64_t cols, int64_t nt, int64_t g4,
                               uint32_t *__restrict__ out, int32_t *flags) {
    const int64_t total = nt * g4 * 32;
    bool bad = false;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int lane = static_cast<int>(i & 31);
        const int64_t rest = i >> 5;
        const int64_t gq = rest % g4, n = rest / g4;
        const int g = lane >> 2, t = lane & 3;
        const int64_t row = n * 8 + g;
        uint32_t word = 0;
        if (row < rows) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const int64_t s = gq * 4 + q;
                uint32_t byte = 0;
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int64_t col = 32 * s + 16 * h + 4 * t + j;
                        if (col < cols) {
                            const float v = latent[row * cols + col];
                            bad |= !isfinite(v);
                            if (v >= 0.0f) byte |= 1u << (4 * h + j);
                        }
                    }
                word |= byte << (8 * q);
            }
        }
        out[i] = word;
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_NONFINITE_LATENT);
}

int64_t d8_bytes(int64_t rows, int64_t cols) { return (rows + 7) / 8 * (((cols + 31) / 32 + 3) / 4) * 128; }

// ------------------------------------------------------------------ launch

namespace {
struct FuPlan {
    int ca = 0, cb = 0;      // cluster sizes of the two kernels
    int64_t ga = 0, gb = 0;  // grids (CTAs)
    int pairs_max = 0, cols_max = 0, groups_max = 0;
    size_t smem_a = 0, smem_b = 0;
};

template <typename Kern>
int active_clusters(Kern kern, int c, int threads, size_t smem, int64_t want) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
        return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(want * c));
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(c);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) return 0;
    return n;
}

template <typename Kern, typename Args>
int launch_cluster_pdl(Kern kern, const Args &a, int c, int threads, int64_t grid, size_t smem, cudaStream_t stream) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess)
        return BD_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(c);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? BD_OK : BD_ERR_LAUNCH;
}

constexpr size_t kFuSmemLimit = 200 * 1024;
constexpr int64_t kGuMaxCtas = 1024;

// Launch shapes.  Gate/up: the largest cluster size (8, 4 or 2) unless a smaller
// one has a quarter more co-resident CTAs (at least one n-tile pair each):
// larger clusters quantize less of x per CTA.  Down: clusters of 4 when they
// fit (the smaller shared-memory slice lets its CTAs sit beside the gate/up
// kernel's and stream their signs while it runs), never more than kDnNt n-tiles
// per cluster.  Cached per (device, shape).
int fu_plan(FuPlan &out, int64_t hidden, int64_t inter) {
    static std::mutex mu;
    static std::map<std::tuple<int, int64_t, int64_t>, FuPlan> cache;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return BD_ERR_DEVICE;
    std::lock_guard<std::mutex> lock(mu);
    const auto key = std::make_tuple(dev, hidden, inter);
    const auto it = cache.find(key);
    if (it != cache.end()) {
        out = it->second;
        return BD_OK;
    }
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms < 1) return BD_ERR_DEVICE;
    const int64_t np = inter / 8, ng = (hidden + 511) / 512, nt = hidden / 8, g4 = (inter / 32 + 3) / 4;
    FuPlan best;
    for (int c : {8, 4, 2}) {
        const int64_t grid = std::min<int64_t>(std::min<int64_t>(sms, kGuMaxCtas) / c, np / c) * c;
        if (grid < c) continue;
        const int cols = static_cast<int>(hidden / c);
        const int pm = static_cast<int>((np + grid - 1) / grid);
        const size_t smem = gu_carve(pm, ng, cols).bytes;
        if (smem > kFuSmemLimit) continue;
        const int act = c == 8   ? active_clusters(ffn_gu_kernel<8>, 8, kGuThreads, smem, grid / c)
                        : c == 4 ? active_clusters(ffn_gu_kernel<4>, 4, kGuThreads, smem, grid / c)
                                 : active_clusters(ffn_gu_kernel<2>, 2, kGuThreads, smem, grid / c);
        const int64_t g = std::min<int64_t>(grid, static_cast<int64_t>(act) * c);
        // a larger cluster quantizes less of x per CTA: keep it unless a smaller one has 1/4 more CTAs
        if (g * 4 > best.ga * 5 || (best.ca == 0 && g > 0)) {
            best.ca = c;
            best.ga = g;
            best.cols_max = cols;
            best.pairs_max = static_cast<int>((np + g - 1) / g);
            best.smem_a = gu_carve(best.pairs_max, ng, cols).bytes;
        }
    }
    if (best.ca == 0) return BD_ERR_LAUNCH;
    for (int c : {4, 2}) {
        const int gm = static_cast<int>((g4 + c - 1) / c);
        const size_t smem = dn_carve(gm, static_cast<int>(best.ga)).bytes;
        if (smem > kFuSmemLimit) continue;
        const int64_t qmin = (nt + kDnNt - 1) / kDnNt;
        const int64_t want = std::max<int64_t>(qmin, sms / c);
        const int act = c == 4 ? active_clusters(ffn_dn_kernel<4>, 4, kDnThreads, smem, want)
                               : active_clusters(ffn_dn_kernel<2>, 2, kDnThreads, smem, want);
        if (act < 1) continue;
        const int64_t q = std::min<int64_t>(std::max<int64_t>(act, qmin), nt);
        best.cb = c;
        best.gb = q * c;
        best.groups_max = gm;
        best.smem_b = smem;
        break;
    }
    if (best.cb == 0) return BD_ERR_LAUNCH;
    cache[key] = best;
    out = best;
    return BD_OK;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
}  // namespace

size_t ffn_fused_workspace_bytes(int64_t hidden, int64_t inter) {
    (void)hidden;
    const size_t codes = (static_cast<size_t>(inter / 32) * 512 + 255) / 256 * 256;
    return codes + kGuMaxCtas * kFuTokens * sizeof(int32_t);  // code sums of up to 1024 gate/up CTAs
}

int ffn_fused_he4(const FfnW8 &f, const uint8_t *signs_down_d8, cudaStream_t stream) {
    if (f.tokens < 1 || f.tokens > kFuTokens || f.hidden < 32 || f.inter < 32 || f.hidden % 32 || f.inter % 32)
        return BD_ERR_INVALID;
    // every operand the kernels bulk-copy starts on a 16-byte boundary
    for (const void *p : {static_cast<const void *>(f.x), static_cast<const void *>(f.gain_gate_up),
                          static_cast<const void *>(f.norm_w), static_cast<const void *>(f.signs_gate_up),
                          static_cast<const void *>(signs_down_d8), static_cast<const void *>(f.scale_gate),
                          static_cast<const void *>(f.mid_gate), static_cast<const void *>(f.scale_up),
                          static_cast<const void *>(f.mid_up), static_cast<const void *>(f.gain_down),
                          static_cast<const void *>(f.scale_down), static_cast<const void *>(f.mid_down),
                          static_cast<const void *>(f.residual)})
        if (!aligned16(p)) return BD_ERR_ALIGNMENT;
    if (reinterpret_cast<uintptr_t>(f.workspace) & 255) return BD_ERR_ALIGNMENT;
    if (!f.workspace || f.workspace_bytes < ffn_fused_workspace_bytes(f.hidden, f.inter)) return BD_ERR_WORKSPACE;
    FuPlan pl;
    if (int st = fu_plan(pl, f.hidden, f.inter)) return st;
    char *ws = static_cast<char *>(f.workspace);
    const size_t codes_bytes = (static_cast<size_t>(f.inter / 32) * 512 + 255) / 256 * 256;
    GuArgs a{};
    a.tokens = f.tokens;
    a.hidden = f.hidden;
    a.inter = f.inter;
    a.gu = f.signs_gate_up;
    a.np = f.inter / 8;
    a.ng = (f.hidden + 511) / 512;
    a.x = f.x;
    a.norm_w = f.norm_w;
    a.eps = f.eps;
    a.gain_gu = f.gain_gate_up;
    a.bound_gu = f.bound_gate_up;
    a.gain_dn = f.gain_down;
    a.bound_dn = f.bound_down;
    a.scale_g = f.scale_gate;
    a.mid_g = f.mid_gate;
    a.scale_u = f.scale_up;
    a.mid_u = f.mid_up;
    a.hidden_out = f.hidden_out;
    a.hcodes = reinterpret_cast<int8_t *>(ws);
    a.hsum = reinterpret_cast<int32_t *>(ws + codes_bytes);
    a.flags = f.flags;
    a.pairs_max = pl.pairs_max;
    a.cols_max = pl.cols_max;
    int st = pl.ca == 8   ? launch_cluster_pdl(ffn_gu_kernel<8>, a, 8, kGuThreads, pl.ga, pl.smem_a, stream)
             : pl.ca == 4 ? launch_cluster_pdl(ffn_gu_kernel<4>, a, 4, kGuThreads, pl.ga, pl.smem_a, stream)
                          : launch_cluster_pdl(ffn_gu_kernel<2>, a, 2, kGuThreads, pl.ga, pl.smem_a, stream);
    if (st) return st;
    DnArgs d{};
    d.tokens = f.tokens;
    d.hidden = f.hidden;
    d.inter = f.inter;
    d.dn = signs_down_d8;
    d.nt = f.hidden / 8;
    d.g4 = (f.inter / 32 + 3) / 4;
    d.hcodes = a.hcodes;
    d.hsum = a.hsum;
    d.gu_ctas = static_cast<int>(pl.ga);
    d.bound_dn = f.bound_down;
    d.scale_d = f.scale_down;
    d.mid_d = f.mid_down;
    d.residual = f.residual;
    d.y = f.y;
    d.flags = f.flags;
    d.groups_max = pl.groups_max;
    return pl.cb == 4 ? launch_cluster_pdl(ffn_dn_kernel<4>, d, 4, kDnThreads, pl.gb, pl.smem_b, stream)
                      : launch_cluster_pdl(ffn_dn_kernel<2>, d, 2, kDnThreads, pl.gb, pl.smem_b, stream);
}

int ffn_fused_shape(int64_t hidden, int64_t inter, int *shape) {
    FuPlan pl;
    if (int st = fu_plan(pl, hidden, inter)) return st;
    shape[0] = pl.ca;
    shape[1] = static_cast<int>(pl.ga);
    shape[2] = pl.cb;
    shape[3] = static_cast<int>(pl.gb);
    return BD_OK;
}

}  // namespace bd

using namespace bd;

extern "C" int64_t bd_d8_bytes(int64_t rows, int64_t cols) {
    if (rows < 0 || cols < 0) return -1;
    return d8_bytes(rows, cols);
}

extern "C" int bd_tile_signs_d8(const float *latent, int64_t rows, int64_t cols, uint8_t *tiled, int32_t *flags,
                                bd_stream_t stream) {
    if (rows < 0 || cols < 1) return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    if (!latent || !tiled || (reinterpret_cast<uintptr_t>(tiled) & 3)) return BD_ERR_INVALID;
    const int64_t nt = (rows + 7) / 8, g4 = ((cols + 31) / 32 + 3) / 4;
    const int64_t total = nt * g4 * 32;
    int64_t grid = (total + 255) / 256;
    if (grid > 148 * 32) grid = 148 * 32;
    tile_d8_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(latent, rows, cols, nt, g4,
                                                                    reinterpret_cast<uint32_t *>(tiled), flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" size_t bd_ffn_fused_workspace_bytes(int64_t hidden, int64_t inter) {
    return hidden < 1 || inter < 1 ? 0 : ffn_fused_workspace_bytes(hidden, inter);
}

extern "C" int bd_ffn_fused_shape(int64_t hidden, int64_t inter, int *shape) {
    if (hidden < 32 || inter < 32 || hidden % 32 || inter % 32 || !shape) return BD_ERR_INVALID;
    return ffn_fused_shape(hidden, inter, shape);
}
