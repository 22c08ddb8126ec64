// Decode-size (tokens <= 32) one-bit SwiGLU blocks with the tokens on the M
// side of the int8 m16n8k32 MMA ("swap AB").
//
// Activation codes (C16, c16_offset) are the A fragments: one 16-byte load per
// lane per 32-column k-step, shared by every weight tile of the warp.  Signs
// (W8) are the B fragments: per 8-row n-tile and 128-column word, lane 4 g + t
// holds one uint32 whose bit 8 j + 2 ks + r is row g, column 32 ks + 16 r + 4 t
// + j; the register of k-step ks, half r is (word >> (2 ks + r)) & 0x01010101 --
// two instructions per register, no shuffles.  Words are stored in groups of
// four per lane ([n-tile][group][lane][4 words]) so that one 16-byte load per
// lane streams 512 columns of an n-tile (512 contiguous bytes per warp).  With
// b in {0, 1} (1 for latent >= 0) the +-1 dot is D = 2 D01 - sum(codes), exact
// in int32.
//
// gateup_w8_kernel: CTAs own a few gate/up n-tile pairs; their warps split K
//   in word groups, keep every pair's accumulators in registers and meet once in
//   shared memory; each lane then finishes its own fragment elements (SwiGLU and
//   the down projection's quantizer) and the code sums reduce with shuffles.
// down_w8_kernel: clusters of CS CTAs split K, and the warps of a CTA split its
//   slice again; each warp covers all n-tiles of the cluster, the CTA sums its
//   warps in shared memory and the cluster sums its CTAs through distributed
//   shared memory; every CTA finishes a 1/CS share of the n-tiles.
// Both read their sign words into registers before griddepcontrol.wait, so the
// weight stream of one kernel overlaps the tail of the one before (PDL).
#include "kernels.cuh"

namespace bd {

// ------------------------------------------------------------------ W8 layout

static int64_t w8_groups(int64_t cols) { return ((cols + 127) / 128 + 3) / 4; }

int64_t w8_words(int64_t rows, int64_t cols) { return (rows + 7) / 8 * w8_groups(cols) * 128; }

// One thread per word: (n-tile, group, lane, word-in-group), consecutive threads
// write consecutive words.
__global__ void tile_w8_kernel(const float *__restrict__ latent, int64_t rows, int64_t cols, int64_t ng,
                               uint32_t *__restrict__ out, int stride, int offset, int32_t *flags) {
    const int64_t nt = (rows + 7) / 8;
    const int64_t total = nt * ng * 128;
    bool bad = false;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int q = static_cast<int>(i & 3);
        const int lane = static_cast<int>((i >> 2) & 31);
        const int64_t rest = i >> 7;
        const int64_t n = rest / ng, grp = rest - n * ng;
        const int64_t w = grp * 4 + q;
        const int g = lane >> 2, t = lane & 3;
        const int64_t row = n * 8 + g;
        uint32_t word = 0;
        if (row < rows) {
            const float *src = latent + row * cols;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
#pragma unroll
                for (int r = 0; r < 2; ++r)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int64_t k = w * 128 + 32 * ks + 16 * r + 4 * t + j;
                        if (k < cols) {
                            const float v = src[k];
                            bad |= !isfinite(v);
                            if (v >= 0.0f) word |= 1u << (8 * j + 2 * ks + r);
                        }
                    }
        }
        out[((n * stride + offset) * ng + grp) * 128 + lane * 4 + q] = word;
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_NONFINITE_LATENT);
}

// Sign words are weights (never written by a kernel that can run concurrently):
// a non-volatile streaming load the compiler may schedule anywhere.
__device__ __forceinline__ uint4 ld_bits(const uint32_t *p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
        : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
        : "l"(p));
    return v;
}

// Codes come from the previous kernel: an ordinary read-only load, ordered after grid_wait().
__device__ __forceinline__ uint4 ld_codes(const void *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }

__device__ __forceinline__ uint32_t word_of(const uint4 &v, int q) { return q == 0 ? v.x : q == 1 ? v.y : q == 2 ? v.z : v.w; }

// D(16 tokens x 8 rows) += A(16 x 32 codes) . B(32 x 8 bits)
__device__ __forceinline__ void mma_tok(int (&d)[4], const uint4 &a, uint32_t b0, uint32_t b1) {
    mma_s8_16832(d, a.x, a.y, a.z, a.w, b0, b1);
}

template <int PLANES>
__device__ __forceinline__ int pm_dot8(int d0, int d1, int cs0, int cs1) {
    if (PLANES == 2) return 256 * (2 * d0 - cs0) + (2 * d1 - cs1);
    return 2 * d0 - cs0;
}

// Pairs per CTA at most: accumulators (8 PLANES MT) plus prefetched sign words
// (8 GMAX) per pair within about 80 registers.
__host__ __device__ constexpr int gu_pmax(int mt, int planes, int gmax) {
    return 80 / (8 * planes * mt + 8 * gmax) > 0 ? 80 / (8 * planes * mt + 8 * gmax) : 1;
}

struct GuW8Args {
    const uint32_t *bits;  // W8, gate/up n-tiles interleaved: [np][2][ng][32][4]
    int64_t np, ng, rows;  // n-tile pairs, 512-column word groups, rows (= intermediate size)
    int tokens;
    const int8_t *codes0, *codes1;  // C16 code planes of the input
    const int32_t *csum0, *csum1;   // input code sums: [tokens][cs_parts] partials
    int cs_parts;
    const float *scale0, *mid0, *scale1, *mid1;  // gate, up
    const float *bound;
    int code_bits;
    const float *row_scale;  // W1 / W1A1 per-token input scale
    const float *next_gain, *next_bound;
    int8_t *next_codes;  // HE4: C16 A8 codes of the down projection's input
    int next_mt;
    int32_t *next_part;  // HE4: [8][32] code sums of the down input (zeroed by the quantizer), CTA b adds into copy b % 8
    float *out;          // hidden h [tokens][rows] (optional for HE4)
    int32_t *flags;
    int gpw;  // word groups per warp
};

template <int MT, int PLANES, int EPI, int GMAX>
__global__ void __launch_bounds__(320) gateup_w8_kernel(const GuW8Args a) {
    constexpr int PMAX = gu_pmax(MT, PLANES, GMAX);
    constexpr int ACC = 2 * PLANES * MT * 4;  // accumulator ints per pair per lane
    extern __shared__ __align__(16) int red[];
    __shared__ int csum_part[2][10][32];  // input code sums: [plane][warp][token], summed in the epilogue
    __shared__ int csum_next[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const int64_t p0 = static_cast<int64_t>(blockIdx.x) * a.np / gridDim.x;
    const int npc = static_cast<int>(static_cast<int64_t>(blockIdx.x + 1) * a.np / gridDim.x - p0);
    const int64_t g0 = static_cast<int64_t>(warp) * a.gpw;
    const int64_t left = a.ng - g0;
    const int ngl = left <= 0 ? 0 : (left < a.gpw ? static_cast<int>(left) : a.gpw);

    // sign words of all pairs x my K-slice, before waiting on the producer of the codes
    uint4 bits[PMAX][2][GMAX];
#pragma unroll
    for (int p = 0; p < PMAX; ++p)
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int j = 0; j < GMAX; ++j)
                bits[p][m][j] = (p < npc && j < ngl)
                                    ? ld_bits(a.bits + ((((p0 + p) * 2 + m) * a.ng + g0 + j) * 32 + lane) * 4)
                                    : make_uint4(0u, 0u, 0u, 0u);
    // epilogue parameters of the first pair this warp finishes (pair `warp`), rows
    // 2 t and 2 t + 1 of it: parameters, like weights, are read before the wait
    const int t4 = lane & 3;
    float ep[5][2] = {};  // scale gate, mid gate, scale up, mid up, next gain
    if (warp < npc) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int64_t o = (p0 + warp) * 8 + 2 * t4 + e;
            if (o < a.rows) {
                ep[0][e] = __ldg(a.scale0 + o);
                ep[2][e] = __ldg(a.scale1 + o);
                if (EPI == EPI_HE4) {
                    ep[1][e] = a.mid0 ? __ldg(a.mid0 + o) : 0.0f;
                    ep[3][e] = a.mid1 ? __ldg(a.mid1 + o) : 0.0f;
                    ep[4][e] = __ldg(a.next_gain + o);
                }
            }
        }
    }
    grid_wait();
    grid_launch_dependents();
    // input code sums: warp w requests partials w, w + nwarps, ... of token `lane`
    // now and files them after the MMAs, so no warp waits on them before its MMAs
    int cs_v0 = 0, cs_v1 = 0;
    if (lane < a.tokens)
        for (int i = warp; i < a.cs_parts; i += nwarps) {
            cs_v0 += a.csum0[lane * a.cs_parts + i];
            if (PLANES == 2) cs_v1 += a.csum1[lane * a.cs_parts + i];
        }
    if (threadIdx.x < 32) csum_next[threadIdx.x] = 0;
    int acc[PMAX][2][PLANES][MT][4];
#pragma unroll
    for (int p = 0; p < PMAX; ++p)
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int r = 0; r < 4; ++r) acc[p][m][pl][mt][r] = 0;
#pragma unroll
    for (int j = 0; j < GMAX; ++j) {
        if (j < ngl) {
            // all 16 k-steps of the group's codes in one round trip
            uint4 A[16][PLANES][MT];
#pragma unroll
            for (int s = 0; s < 16; ++s)
#pragma unroll
                for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
                        A[s][pl][mt] = ld_codes((pl ? a.codes1 : a.codes0) +
                                                ((((g0 + j) * 16 + s) * MT + mt) * 32 + lane) * 16);
#pragma unroll
            for (int s = 0; s < 16; ++s)
#pragma unroll
                for (int p = 0; p < PMAX; ++p) {
                    if (p < npc) {
#pragma unroll
                        for (int m = 0; m < 2; ++m) {
                            const uint32_t word = word_of(bits[p][m][j], s >> 2);
                            const uint32_t b0 = (word >> (2 * (s & 3))) & 0x01010101u;
                            const uint32_t b1 = (word >> (2 * (s & 3) + 1)) & 0x01010101u;
#pragma unroll
                            for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
                                for (int mt = 0; mt < MT; ++mt) mma_tok(acc[p][m][pl][mt], A[s][pl][mt], b0, b1);
                        }
                    }
                }
        }
    }
    csum_part[0][warp][lane] = cs_v0;
    csum_part[1][warp][lane] = cs_v1;
#pragma unroll
    for (int p = 0; p < PMAX; ++p) {
        if (p < npc) {
            int *dst = red + (static_cast<size_t>(warp) * PMAX + p) * ACC * 32 + lane;
#pragma unroll
            for (int m = 0; m < 2; ++m)
#pragma unroll
                for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int r = 0; r < 4; ++r)
                            dst[(((m * PLANES + pl) * MT + mt) * 4 + r) * 32] = acc[p][m][pl][mt][r];
        }
    }
    __syncthreads();

    // epilogue: the warp that owns pair p (p = warp, warp + nwarps, ...) sums its
    // lanes' fragment registers over the K-split warps; lane 4 g + t finishes the
    // elements (token 16 mt + g + 8 h, row 2 t + e) of its fragment
    Quant qin, qnext;
    if (EPI == EPI_HE4) {
        qin.init(__ldg(a.bound), a.code_bits);
        const float nb = __ldg(a.next_bound);
        qnext.init(nb, 8);
        if (bad_bound(nb) && blockIdx.x == 0 && threadIdx.x == 0) set_flag(a.flags, BD_FLAG_BAD_BOUND);
    }
    bool bad = false;
    const int g = lane >> 2;
    int lsum[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) lsum[mt][0] = lsum[mt][1] = 0;
    float rs[MT][2];
    int cin0[MT][2], cin1[MT][2];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int tok = mt * 16 + g + 8 * h;
            rs[mt][h] = (EPI != EPI_HE4 && tok < a.tokens) ? __ldg(a.row_scale + tok) : 0.0f;
            int c0 = 0, c1 = 0;
            for (int w = 0; w < nwarps; ++w) {
                c0 += csum_part[0][w][tok];
                c1 += csum_part[1][w][tok];
            }
            cin0[mt][h] = c0;
            cin1[mt][h] = c1;
        }
    for (int p = warp; p < npc; p += nwarps) {
        int d[2][PLANES][MT][4];
        const int *base = red + static_cast<size_t>(p) * ACC * 32 + lane;
#pragma unroll
        for (int m = 0; m < 2; ++m)
#pragma unroll
            for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const int *s = base + (((m * PLANES + pl) * MT + mt) * 4 + r) * 32;
                        int v = 0;
#pragma unroll
                        for (int w = 0; w < 10; ++w)
                            if (w < nwarps) v += s[static_cast<size_t>(w) * PMAX * ACC * 32];
                        d[m][pl][mt][r] = v;
                    }
        // parameters: prefetched for the first owned pair, loaded here for the others
        float pp[5][2];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int64_t o = (p0 + p) * 8 + 2 * t4 + e;
            const bool first = p == warp, live = o < a.rows;
            pp[0][e] = first ? ep[0][e] : (live ? __ldg(a.scale0 + o) : 0.0f);
            pp[2][e] = first ? ep[2][e] : (live ? __ldg(a.scale1 + o) : 0.0f);
            if (EPI == EPI_HE4) {
                pp[1][e] = first ? ep[1][e] : ((live && a.mid0) ? __ldg(a.mid0 + o) : 0.0f);
                pp[3][e] = first ? ep[3][e] : ((live && a.mid1) ? __ldg(a.mid1 + o) : 0.0f);
                pp[4][e] = first ? ep[4][e] : (live ? __ldg(a.next_gain + o) : 0.0f);
            }
        }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int h = r >> 1, e = r & 1;
                const int tok = mt * 16 + g + 8 * h;
                const int64_t o = (p0 + p) * 8 + 2 * t4 + e;
                if (tok >= a.tokens || o >= a.rows) continue;
                const int cs0 = cin0[mt][h], cs1 = cin1[mt][h];
                const int Dg = pm_dot8<PLANES>(d[0][0][mt][r], d[0][PLANES - 1][mt][r], cs0, cs1);
                const int Du = pm_dot8<PLANES>(d[1][0][mt][r], d[1][PLANES - 1][mt][r], cs0, cs1);
                float gv, uv;
                if (EPI == EPI_HE4) {
                    gv = he4_value(Dg, pp[0][e], qin.step, cs0, pp[1][e]);
                    uv = he4_value(Du, pp[2][e], qin.step, cs0, pp[3][e]);
                } else if (EPI == EPI_W1) {
                    gv = __fmul_rn(__fmul_rn(static_cast<float>(Dg), rs[mt][h]), pp[0][e]);
                    uv = __fmul_rn(__fmul_rn(static_cast<float>(Du), rs[mt][h]), pp[2][e]);
                } else {
                    gv = __fmul_rn(__fmul_rn(static_cast<float>(Dg), pp[0][e]), rs[mt][h]);
                    uv = __fmul_rn(__fmul_rn(static_cast<float>(Du), pp[2][e]), rs[mt][h]);
                }
                const float hv = __fmul_rn(silu(gv), uv);
                if (a.out) a.out[static_cast<int64_t>(tok) * a.rows + o] = hv;
                if (EPI == EPI_HE4) {
                    const float gained = __fmul_rn(hv, pp[4][e]);
                    bad |= !isfinite(gained);
                    const int code = qnext.code(gained);
                    a.next_codes[c16_offset(tok, o, a.next_mt)] = static_cast<int8_t>(code);
                    lsum[mt][h] += code;
                }
            }
    }
    if (EPI == EPI_HE4) {
        // lanes of one g share tokens g, g + 8: reduce over t, one shared add per warp and token
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                int v = lsum[mt][h];
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                if (t4 == 0 && v) atomicAdd(&csum_next[mt * 16 + g + 8 * h], v);
            }
        if (__any_sync(0xffffffffu, bad) && lane == 0) set_flag(a.flags, BD_FLAG_NONFINITE_INPUT);
        __syncthreads();
        if (threadIdx.x < 32 && csum_next[threadIdx.x])
            atomicAdd(a.next_part + (blockIdx.x & 7) * 32 + threadIdx.x, csum_next[threadIdx.x]);  // exact, order-free
    }
}

// ------------------------------------------------------------------ down projection (cluster split-K)

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

__device__ __forceinline__ int ld_cluster_i32(const int *local, uint32_t rank) {
    const uint32_t addr = static_cast<uint32_t>(__cvta_generic_to_shared(local));
    uint32_t remote;
    int v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(addr), "r"(rank));
    asm volatile("ld.shared::cluster.u32 %0, [%1];\n" : "=r"(v) : "r"(remote) : "memory");
    return v;
}

constexpr int kDnMaxWarps = 8;  // warps per CTA, each a slice of the CTA's word groups
constexpr int kDnGmax = 2;      // word groups (512 columns) per warp at most

// n-tiles per cluster: every warp keeps all of them (accumulators and sign words) in registers
__host__ __device__ constexpr int dn_ntmax(int mt, int planes) {
    return 72 / (4 * mt * planes + 4 * kDnGmax) > 0 ? 72 / (4 * mt * planes + 4 * kDnGmax) : 1;
}

struct DnW8Args {
    const uint32_t *bits;  // W8 [nt][ng][32][4]
    int64_t nt, ng, rows;  // n-tiles, word groups, rows (= hidden size)
    int tokens;
    const int8_t *codes0, *codes1;  // C16 planes of the input (K = intermediate)
    const int32_t *csum0, *csum1;   // [cs_parts][32] partial code sums (HE4: 8 copies) or full sums [32] (parts 1)
    int cs_parts;
    const float *scale0, *mid0, *bound;
    int code_bits;
    const float *row_scale;
    const float *residual;
    float *out;
    int32_t *raw_dot;
    int cs;    // CTAs per cluster (K split)
    int ntpc;  // n-tiles per cluster
};

template <int MT, int PLANES, int EPI>
__global__ void __launch_bounds__(kDnMaxWarps * 32) down_w8_kernel(const DnW8Args a) {
    constexpr int NTMAX = dn_ntmax(MT, PLANES);
    constexpr int ACCD = PLANES * MT * 4;  // accumulator ints per n-tile per lane
    extern __shared__ __align__(16) int dsm[];  // [warps][NTMAX][ACCD][32] then [NTMAX][ACCD][32]
    __shared__ int csum_part[2][kDnMaxWarps][32];  // input code sums: [plane][warp][token]
    __shared__ int csum_s[2][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    const uint32_t rank = cluster_rank();
    const int64_t cid = blockIdx.x / a.cs;
    const int64_t n0 = cid * a.ntpc;
    const int ncl = static_cast<int>(min(static_cast<int64_t>(a.ntpc), a.nt - n0));
    // word groups of this CTA, then of this warp
    const int64_t c0 = rank * a.ng / a.cs, c1 = (rank + 1) * a.ng / a.cs;
    const int64_t g0 = c0 + warp * (c1 - c0) / nwarps;
    const int ngl = static_cast<int>(c0 + (warp + 1) * (c1 - c0) / nwarps - g0);

    uint4 bits[NTMAX][kDnGmax];
#pragma unroll
    for (int n = 0; n < NTMAX; ++n)
#pragma unroll
        for (int j = 0; j < kDnGmax; ++j)
            bits[n][j] = (n < ncl && j < ngl) ? ld_bits(a.bits + (((n0 + n) * a.ng + g0 + j) * 32 + lane) * 4)
                                              : make_uint4(0u, 0u, 0u, 0u);
    // epilogue parameters of the first n-tile this warp finishes (rows 2 t, 2 t + 1)
    const int t4 = lane & 3;
    const int nb = static_cast<int>(rank * ncl / a.cs), ne = static_cast<int>((rank + 1) * ncl / a.cs);
    float ep[2][2] = {};  // scale, midpoint
    // and its residual: the block's input, written before the block's first kernel, which
    // (like every kernel of the block) let this one launch only after its own dependency
    // wait, so it is complete here; out may alias it (each element is read, then written,
    // by the same thread)
    float res[MT][4] = {};
    if (nb + warp < ne) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
            const int64_t o = (n0 + nb + warp) * 8 + 2 * t4 + e;
            if (o < a.rows) {
                ep[0][e] = __ldg(a.scale0 + o);
                ep[1][e] = (EPI == EPI_HE4 && a.mid0) ? __ldg(a.mid0 + o) : 0.0f;
            }
        }
        if (a.residual) {
            const int g8 = lane >> 2;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int tok = mt * 16 + g8 + 8 * (r >> 1);
                    const int64_t o = (n0 + nb + warp) * 8 + 2 * t4 + (r & 1);
                    if (tok < a.tokens && o < a.rows) res[mt][r] = a.residual[static_cast<int64_t>(tok) * a.rows + o];
                }
        }
    }
    grid_wait();
    grid_launch_dependents();
    // input code sums: warp w requests copies w, w + nwarps, ... of token `lane`
    // now and files them after the MMAs, off the MMA path
    int cs_v0 = 0, cs_v1 = 0;
    if (lane < a.tokens)
        for (int c = warp; c < a.cs_parts; c += nwarps) {
            cs_v0 += a.csum0[c * 32 + lane];
            if (PLANES == 2) cs_v1 += a.csum1[c * 32 + lane];
        }
    int acc[NTMAX][PLANES][MT][4];
#pragma unroll
    for (int n = 0; n < NTMAX; ++n)
#pragma unroll
        for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[n][pl][mt][r] = 0;
#pragma unroll
    for (int j = 0; j < kDnGmax; ++j) {
        if (j < ngl) {
            // all 16 k-steps of the group's codes in one round trip
            uint4 A[16][PLANES][MT];
#pragma unroll
            for (int s = 0; s < 16; ++s)
#pragma unroll
                for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
                        A[s][pl][mt] = ld_codes((pl ? a.codes1 : a.codes0) +
                                                ((((g0 + j) * 16 + s) * MT + mt) * 32 + lane) * 16);
#pragma unroll
            for (int s = 0; s < 16; ++s)
#pragma unroll
                for (int n = 0; n < NTMAX; ++n) {
                    if (n < ncl) {
                        const uint32_t word = word_of(bits[n][j], s >> 2);
                        const uint32_t b0 = (word >> (2 * (s & 3))) & 0x01010101u;
                        const uint32_t b1 = (word >> (2 * (s & 3) + 1)) & 0x01010101u;
#pragma unroll
                        for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt) mma_tok(acc[n][pl][mt], A[s][pl][mt], b0, b1);
                    }
                }
        }
    }
    csum_part[0][warp][lane] = cs_v0;
    csum_part[1][warp][lane] = cs_v1;
    int *wpart = dsm;                                                        // per-warp partials
    int *cpart = dsm + static_cast<size_t>(kDnMaxWarps) * NTMAX * ACCD * 32;  // this CTA's sums
#pragma unroll
    for (int n = 0; n < NTMAX; ++n)
        if (n < ncl) {
#pragma unroll
            for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int r = 0; r < 4; ++r)
                        wpart[((warp * NTMAX + n) * ACCD + (pl * MT + mt) * 4 + r) * 32 + lane] = acc[n][pl][mt][r];
        }
    __syncthreads();
    if (threadIdx.x < 32) {
        int s0 = 0, s1 = 0;
        for (int w = 0; w < nwarps; ++w) {
            s0 += csum_part[0][w][threadIdx.x];
            s1 += csum_part[1][w][threadIdx.x];
        }
        csum_s[0][threadIdx.x] = s0;  // read after the cluster barrier below
        csum_s[1][threadIdx.x] = s1;
    }
    for (int n = warp; n < ncl; n += nwarps)
#pragma unroll
        for (int i = 0; i < ACCD; ++i) {
            int v = 0;
#pragma unroll
            for (int w = 0; w < kDnMaxWarps; ++w)
                if (w < nwarps) v += wpart[((w * NTMAX + n) * ACCD + i) * 32 + lane];
            cpart[(n * ACCD + i) * 32 + lane] = v;
        }
    cluster_sync_all();

    // this CTA finishes n-tiles [rank * ncl / cs, (rank + 1) * ncl / cs) of the cluster
    Quant q;
    if (EPI == EPI_HE4) q.init(__ldg(a.bound), a.code_bits);
    const int g = lane >> 2;
    for (int n = nb + warp; n < ne; n += nwarps) {
        int d[PLANES][MT][4];
#pragma unroll
        for (int pl = 0; pl < PLANES; ++pl)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const int *s = cpart + (n * ACCD + (pl * MT + mt) * 4 + r) * 32 + lane;
                    // every CTA's partial requested at once (cluster of 8 at most)
                    int part[8];
#pragma unroll
                    for (int c = 0; c < 8; ++c) part[c] = c < a.cs ? ld_cluster_i32(s, static_cast<uint32_t>(c)) : 0;
                    int v = 0;
#pragma unroll
                    for (int c = 0; c < 8; ++c) v += part[c];
                    d[pl][mt][r] = v;
                }
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const int tok = mt * 16 + g + 8 * (r >> 1);
                const int64_t o = (n0 + n) * 8 + 2 * t4 + (r & 1);
                if (tok >= a.tokens || o >= a.rows) continue;
                const int cs0 = csum_s[0][tok], cs1 = csum_s[1][tok];
                const int D = pm_dot8<PLANES>(d[0][mt][r], d[PLANES - 1][mt][r], cs0, cs1);
                const int e = r & 1;
                const bool first = n == nb + warp;
                const float sc = first ? ep[0][e] : __ldg(a.scale0 + o);
                float y;
                if (EPI == EPI_HE4) {
                    const float mid = first ? ep[1][e] : (a.mid0 ? __ldg(a.mid0 + o) : 0.0f);
                    y = he4_value(D, sc, q.step, cs0, mid);
                } else if (EPI == EPI_W1) {
                    y = __fmul_rn(__fmul_rn(static_cast<float>(D), __ldg(a.row_scale + tok)), sc);
                } else {
                    y = __fmul_rn(__fmul_rn(static_cast<float>(D), sc), __ldg(a.row_scale + tok));
                }
                const int64_t idx = static_cast<int64_t>(tok) * a.rows + o;
                if (a.residual) y = __fadd_rn(first ? res[mt][r] : a.residual[idx], y);
                a.out[idx] = y;
                if (a.raw_dot) a.raw_dot[idx] = D;
            }
    }
    cluster_sync_all();  // no CTA leaves while another still reads its partials
}

// ------------------------------------------------------------------ launchers

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

// Warps of a gate/up CTA: one per word group up to 10, more groups per warp beyond.
static void gu_shape(int64_t ng, int &nwarps, int &gpw) {
    nwarps = static_cast<int>(std::min<int64_t>(10, std::max<int64_t>(1, ng)));
    gpw = static_cast<int>((ng + nwarps - 1) / nwarps);
}

static int gu_gmax(int gpw) { return gpw <= 1 ? 1 : (gpw <= 2 ? 2 : 0); }

// One resident wave when the pairs allow it: as many CTAs as fit on the GPU at
// once (occupancy of this kernel shape), but never more pairs per CTA than PMAX.
static int64_t gu_grid(int64_t np, int pmax, int resident_per_sm) {
    const int64_t slots = static_cast<int64_t>(std::max(1, resident_per_sm)) * sm_count();
    return std::max<int64_t>(std::min<int64_t>(np, slots), (np + pmax - 1) / pmax);
}

template <int MT, int PLANES, int EPI, int GMAX>
static int launch_gu(GuW8Args a, int nwarps, cudaStream_t stream) {
    constexpr int PMAX = gu_pmax(MT, PLANES, GMAX);
    const size_t smem = static_cast<size_t>(nwarps) * PMAX * 2 * PLANES * MT * 4 * 32 * sizeof(int);
    auto kern = gateup_w8_kernel<MT, PLANES, EPI, GMAX>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
        return BD_ERR_LAUNCH;
    static int resident[11];  // per warp count; the kernel shape is fixed per instantiation
    if (!resident[nwarps] &&
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident[nwarps], kern, 32 * nwarps, smem) != cudaSuccess)
        return BD_ERR_LAUNCH;
    const int64_t grid = gu_grid(a.np, PMAX, resident[nwarps]);
    return launch_pdl(kern, dim3(static_cast<unsigned>(grid)), dim3(32 * nwarps), smem, stream, a);
}

template <int MT, int PLANES, int EPI>
static int launch_gu_w(GuW8Args a, cudaStream_t stream) {
    int nwarps = 0;
    gu_shape(a.ng, nwarps, a.gpw);
    const int gmax = gu_gmax(a.gpw);
    if (gmax == 1) return launch_gu<MT, PLANES, EPI, 1>(a, nwarps, stream);
    if (gmax == 2) return launch_gu<MT, PLANES, EPI, 2>(a, nwarps, stream);
    return BD_ERR_INVALID;  // K above 10 warps x 2 groups x 512 columns
}

template <int MT, int PLANES, int EPI>
static int launch_dn(DnW8Args a, cudaStream_t stream) {
    constexpr int NTMAX = dn_ntmax(MT, PLANES);
    // cluster size: long K is spread over four (or more) CTAs; within a CTA one
    // warp per word group (kDnGmax groups per warp at most)
    int cs = a.ng >= 8 ? 4 : 1;
    while ((a.ng + cs - 1) / cs > static_cast<int64_t>(kDnMaxWarps) * kDnGmax && cs < 8) cs *= 2;
    const int64_t per_cta = (a.ng + cs - 1) / cs;
    if (per_cta > static_cast<int64_t>(kDnMaxWarps) * kDnGmax) return BD_ERR_INVALID;
    const int nwarps = static_cast<int>(std::min<int64_t>(kDnMaxWarps, std::max<int64_t>(1, per_cta)));
    a.cs = cs;
    const int64_t clusters_target = std::max<int64_t>(1, sm_count() / cs);
    a.ntpc = static_cast<int>(std::max<int64_t>(1, (a.nt + clusters_target - 1) / clusters_target));
    if (a.ntpc > NTMAX) a.ntpc = NTMAX;
    const int64_t clusters = (a.nt + a.ntpc - 1) / a.ntpc;
    const size_t smem = static_cast<size_t>(kDnMaxWarps + 1) * NTMAX * PLANES * MT * 4 * 32 * sizeof(int);
    auto kern = down_w8_kernel<MT, PLANES, EPI>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)) != cudaSuccess ||
        cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
        return BD_ERR_LAUNCH;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(clusters * cs));
    cfg.blockDim = dim3(32 * nwarps);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(cs);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, a) == cudaSuccess ? BD_OK : BD_ERR_LAUNCH;
}

// ------------------------------------------------------------------ the block

namespace {
struct W8Pieces {
    int8_t *codes_in, *codes_in_lo, *codes_mid, *codes_mid_lo;
    int32_t *sum_in, *sum_in_lo, *sum_mid, *sum_mid_lo, *gu_part;
    float *scale_in, *scale_mid, *hidden;
    size_t bytes;
};

// C16 buffers hold whole 512-column groups (the kernels read codes group by group)
size_t c16_bytes(int64_t cols) { return static_cast<size_t>(w8_groups(cols)) * 16 * 2 * 512; }

W8Pieces carve_w8(void *ws, int64_t hidden, int64_t inter) {
    char *base = static_cast<char *>(ws);
    size_t off = 0;
    auto take = [&](size_t n) {
        off = (off + 255) & ~static_cast<size_t>(255);
        char *p = base ? base + off : nullptr;
        off += n;
        return p;
    };
    W8Pieces p{};
    p.codes_in = reinterpret_cast<int8_t *>(take(c16_bytes(hidden)));
    p.codes_in_lo = reinterpret_cast<int8_t *>(take(c16_bytes(hidden)));
    p.codes_mid = reinterpret_cast<int8_t *>(take(c16_bytes(inter)));
    p.codes_mid_lo = reinterpret_cast<int8_t *>(take(c16_bytes(inter)));
    p.sum_in = reinterpret_cast<int32_t *>(take(32 * quant_parts(hidden) * sizeof(int32_t)));
    p.sum_in_lo = reinterpret_cast<int32_t *>(take(32 * sizeof(int32_t)));
    p.sum_mid = reinterpret_cast<int32_t *>(take(32 * sizeof(int32_t)));
    p.sum_mid_lo = reinterpret_cast<int32_t *>(take(32 * sizeof(int32_t)));
    p.gu_part = reinterpret_cast<int32_t *>(take(8 * 32 * sizeof(int32_t)));
    p.scale_in = reinterpret_cast<float *>(take(32 * sizeof(float)));
    p.scale_mid = reinterpret_cast<float *>(take(32 * sizeof(float)));
    p.hidden = reinterpret_cast<float *>(take(static_cast<size_t>(32) * inter * sizeof(float)));
    p.bytes = off;
    return p;
}

template <int MT>
int ffn_w8_mt(const FfnW8 &f, int epi, const W8Pieces &w, cudaStream_t stream) {
    const int64_t ld_h = (f.hidden + 255) / 256 * 256, ld_f = (f.inter + 255) / 256 * 256;
    const int T = f.tokens;
    int st;
    GuW8Args g{};
    g.bits = f.signs_gate_up;
    g.np = (f.inter + 7) / 8;
    g.ng = w8_groups(f.hidden);
    g.rows = f.inter;
    g.tokens = T;
    g.codes0 = w.codes_in;
    g.scale0 = f.scale_gate;
    g.mid0 = f.mid_gate;
    g.scale1 = f.scale_up;
    g.mid1 = f.mid_up;
    g.flags = f.flags;
    DnW8Args d{};
    d.bits = f.signs_down;
    d.nt = (f.hidden + 7) / 8;
    d.ng = w8_groups(f.inter);
    d.rows = f.hidden;
    d.tokens = T;
    d.codes0 = w.codes_mid;
    d.scale0 = f.scale_down;
    d.mid0 = f.mid_down;
    d.residual = f.residual;
    d.out = f.y;
    if (epi == EPI_HE4) {
        // the quantizer also zeroes the 8 x 32 code-sum copies that gate/up accumulates for the down input
        st = launch_quantize_codes(f.x, T, f.hidden, ld_h, f.gain_gate_up, f.bound_gate_up, 4, w.codes_in, w.sum_in,
                                   true, f.flags, w.gu_part, 8 * 32, stream, f.norm_w, f.eps, MT);
        if (st) return st;
        g.csum0 = w.sum_in;
        g.cs_parts = quant_parts(f.hidden);
        g.bound = f.bound_gate_up;
        g.code_bits = 4;
        g.next_gain = f.gain_down;
        g.next_bound = f.bound_down;
        g.next_codes = w.codes_mid;
        g.next_mt = MT;
        g.next_part = w.gu_part;
        g.out = f.hidden_out;
        st = launch_gu_w<MT, 1, EPI_HE4>(g, stream);
        if (st) return st;
        d.csum0 = w.gu_part;
        d.cs_parts = 8;
        d.bound = f.bound_down;
        d.code_bits = 8;
        return launch_dn<MT, 1, EPI_HE4>(d, stream);
    }
    float *hidden = f.hidden_out ? f.hidden_out : w.hidden;
    g.out = hidden;
    g.row_scale = w.scale_in;
    g.cs_parts = 1;
    g.csum0 = w.sum_in;
    d.cs_parts = 1;
    d.csum0 = w.sum_mid;
    d.row_scale = w.scale_mid;
    if (epi == EPI_W1) {
        st = launch_quantize_planes(f.x, T, f.hidden, ld_h, w.codes_in, w.codes_in_lo, w.sum_in, w.sum_in_lo,
                                    w.scale_in, f.flags, stream, MT);
        if (st) return st;
        g.codes1 = w.codes_in_lo;
        g.csum1 = w.sum_in_lo;
        st = launch_gu_w<MT, 2, EPI_W1>(g, stream);
        if (st) return st;
        st = launch_quantize_planes(hidden, T, f.inter, ld_f, w.codes_mid, w.codes_mid_lo, w.sum_mid, w.sum_mid_lo,
                                    w.scale_mid, f.flags, stream, MT);
        if (st) return st;
        d.codes1 = w.codes_mid_lo;
        d.csum1 = w.sum_mid_lo;
        return launch_dn<MT, 2, EPI_W1>(d, stream);
    }
    st = launch_binarize(f.x, T, f.hidden, ld_h, w.codes_in, w.sum_in, w.scale_in, nullptr, 0, f.flags, stream, MT);
    if (st) return st;
    st = launch_gu_w<MT, 1, EPI_W1A1>(g, stream);
    if (st) return st;
    st = launch_binarize(hidden, T, f.inter, ld_f, w.codes_mid, w.sum_mid, w.scale_mid, nullptr, 0, f.flags, stream,
                         MT);
    if (st) return st;
    return launch_dn<MT, 1, EPI_W1A1>(d, stream);
}
}  // namespace

size_t ffn_w8_workspace_bytes(int64_t hidden, int64_t inter) { return carve_w8(nullptr, hidden, inter).bytes; }

int ffn_w8(const FfnW8 &f, int epi, cudaStream_t stream) {
    if (f.tokens < 1 || f.tokens > 32 || f.hidden < 1 || f.inter < 1) return BD_ERR_INVALID;
    const W8Pieces w = carve_w8(f.workspace, f.hidden, f.inter);
    if (!f.workspace || w.bytes > f.workspace_bytes) return BD_ERR_WORKSPACE;
    return f.tokens <= 16 ? ffn_w8_mt<1>(f, epi, w, stream) : ffn_w8_mt<2>(f, epi, w, stream);
}

}  // namespace bd

using namespace bd;

extern "C" int64_t bd_w8_words(int64_t rows, int64_t cols) {
    if (rows < 0 || cols < 0) return -1;
    return w8_words(rows, cols);
}

extern "C" int bd_tile_signs_w8(const float *latent, int64_t rows, int64_t cols, uint32_t *tiled, int block_stride,
                                int block_offset, int32_t *flags, bd_stream_t stream) {
    if (rows < 0 || cols < 1 || block_stride < 1 || block_offset < 0 || block_offset >= block_stride)
        return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    if (!latent || !tiled) return BD_ERR_INVALID;
    const int64_t ng = w8_groups(cols);
    const int64_t total = w8_words(rows, cols);
    int64_t grid = (total + 255) / 256;
    if (grid > 148 * 32) grid = 148 * 32;
    tile_w8_kernel<<<static_cast<unsigned>(grid), 256, 0, stream>>>(latent, rows, cols, ng, tiled, block_stride,
                                                                    block_offset, flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}
