// Decode-size (tokens <= 32) packed-sign projections on the integer tensor pipe.
//
// Weights arrive as T16 sign words (see pack.cu); each lane expands its 16-byte
// slice of a 512-byte unit directly into the 0/1 int8 A fragments of
// m16n8k32 MMAs (two instructions per register, no shared memory for weights).
// Activation codes are kept in the B-fragment layout (see frag_offset): each
// lane fetches the B fragments of two k-steps with one 16-byte L1-cached load,
// shared by the gate and up matrices.  With b in {0,1} (b = 1 for latent >= 0)
// the +-1 dot is D = 2 * D01 - sum(codes), exact in int32, so every epilogue
// starts from the exact integer dot.  Kernels use programmatic dependent
// launch: the weight bits (read-only) are requested before grid_wait(), so
// their HBM latency overlaps the previous kernel.
#include "kernels.cuh"

namespace bd {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kSplit = 4;                 // warps sharing one row block (pair) along K
constexpr int kBlocksPerCta = kWarps / kSplit;
constexpr int kBatch = 4;                 // column pairs of weight bits in flight per warp

// Load the B fragments (NT n-tiles) of k-step pair sp for this lane.
template <int NT>
__device__ __forceinline__ void load_b(uint4 (&b)[NT], const int8_t *codes, int64_t nsp, int64_t sp, int lane) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
        b[nt] = __ldg(reinterpret_cast<const uint4 *>(codes + (((nt * nsp + sp) * 32 + lane) << 4)));
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

// One 256-column unit of up to two matrices (M matrices) against PLANES code planes.
template <int NT, int PLANES, int M>
__device__ __forceinline__ void unit_mma(int (&acc)[M][PLANES][NT][4], const uint4 (&w)[M], const int8_t *codes0,
                                         const int8_t *codes1, int64_t nsp, int64_t cp, int lane) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int qp = 0; qp < 2; ++qp) {
            const int64_t sp = cp * 4 + c * 2 + qp;
            uint4 b0[NT], b1[NT];
            load_b<NT>(b0, codes0, nsp, sp, lane);
            if (PLANES == 2) load_b<NT>(b1, codes1, nsp, sp, lane);
#pragma unroll
            for (int qq = 0; qq < 2; ++qq) {
                const int q = 2 * qp + qq;
#pragma unroll
                for (int m = 0; m < M; ++m) {
                    const AFrag a(c ? w[m].z : w[m].x, c ? w[m].w : w[m].y, q);
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        mma_s8_16832(acc[m][0][nt], a.r[0], a.r[1], a.r[2], a.r[3], qq ? b0[nt].z : b0[nt].x,
                                     qq ? b0[nt].w : b0[nt].y);
                        if (PLANES == 2)
                            mma_s8_16832(acc[m][PLANES - 1][nt], a.r[0], a.r[1], a.r[2], a.r[3],
                                         qq ? b1[nt].z : b1[nt].x, qq ? b1[nt].w : b1[nt].y);
                    }
                }
            }
        }
    }
}

// Exact +-1 dot from the 0/1 partial sums of all planes.
template <int PLANES>
__device__ __forceinline__ int pm_dot(const int (&d01)[PLANES], int cs0, int cs1) {
    if (PLANES == 2) return 256 * (2 * d01[0] - cs0) + (2 * d01[PLANES - 1] - cs1);
    return 2 * d01[0] - cs0;
}

template <int M, int PLANES, int NT>
__device__ __forceinline__ void zero_acc(int (&acc)[M][PLANES][NT][4]) {
#pragma unroll
    for (int m = 0; m < M; ++m)
#pragma unroll
        for (int p = 0; p < PLANES; ++p)
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[m][p][n][i] = 0;
}

// Sum the kSplit K-slices of each row block through shared memory; the slice-0
// warp ends with the totals.  All warps of the CTA must call this.
template <int M, int PLANES, int NT>
__device__ __forceinline__ void reduce_split(int (&acc)[M][PLANES][NT][4], int *red, int slot, int ks, int lane) {
    constexpr int VALS = M * PLANES * NT * 4;
    int *buf = red + slot * 32 * VALS + lane;
#pragma unroll
    for (int r = 1; r < kSplit; ++r) {
        if (ks == r) {
            int v = 0;
#pragma unroll
            for (int m = 0; m < M; ++m)
#pragma unroll
                for (int p = 0; p < PLANES; ++p)
#pragma unroll
                    for (int n = 0; n < NT; ++n)
#pragma unroll
                        for (int i = 0; i < 4; ++i) buf[(v++) * 32] = acc[m][p][n][i];
        }
        __syncthreads();
        if (ks == 0) {
            int v = 0;
#pragma unroll
            for (int m = 0; m < M; ++m)
#pragma unroll
                for (int p = 0; p < PLANES; ++p)
#pragma unroll
                    for (int n = 0; n < NT; ++n)
#pragma unroll
                        for (int i = 0; i < 4; ++i) acc[m][p][n][i] += buf[(v++) * 32];
        }
        __syncthreads();
    }
}

// Row sums of the codes: either full sums ([tokens]) or nparts partial sums per token.
__device__ __forceinline__ int code_sum(const int32_t *sums, int nparts, int token) {
    int s = 0;
    for (int i = 0; i < nparts; ++i) s += sums[token * nparts + i];
    return s;
}

// --------------------------------------------------------------------------- gate/up pair kernel
template <int NT, int PLANES, int EPI>
__global__ void __launch_bounds__(kThreads) gateup_kernel(const ProjArgs a) {
    __shared__ int red[kBlocksPerCta * 32 * 2 * PLANES * NT * 4];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int slot = warp / kSplit, ks = warp % kSplit;
    const int64_t npairs = (a.rows + 15) / 16;
    const int64_t pair = static_cast<int64_t>(blockIdx.x) * kBlocksPerCta + slot;
    const int ncp = static_cast<int>(a.ncp);
    const int cp0 = ks * ncp / kSplit, cp1 = (ks + 1) * ncp / kSplit;
    const bool active = pair < npairs && cp0 < cp1;
    const int64_t nsp = a.ld / 64;

    const uint32_t *bits0 = a.bits + (2 * pair) * a.ncp * 128 + lane * 4;
    const uint32_t *bits1 = a.bits + (2 * pair + 1) * a.ncp * 128 + lane * 4;
    uint4 wg[kBatch], wu[kBatch];
    if (active) {
#pragma unroll
        for (int i = 0; i < kBatch; ++i)
            if (cp0 + i < cp1) {
                wg[i] = ld_stream_u4(bits0 + (cp0 + i) * 128);
                wu[i] = ld_stream_u4(bits1 + (cp0 + i) * 128);
            }
    }
    grid_wait();
    grid_launch_dependents();

    int acc[2][PLANES][NT][4];
    zero_acc(acc);
    if (active) {
        for (int base = cp0; base < cp1; base += kBatch) {
            if (base != cp0) {
#pragma unroll
                for (int i = 0; i < kBatch; ++i)
                    if (base + i < cp1) {
                        wg[i] = ld_stream_u4(bits0 + (base + i) * 128);
                        wu[i] = ld_stream_u4(bits1 + (base + i) * 128);
                    }
            }
#pragma unroll
            for (int i = 0; i < kBatch; ++i)
                if (base + i < cp1) {
                    const uint4 w[2] = {wg[i], wu[i]};
                    unit_mma<NT, PLANES, 2>(acc, w, a.codes0, a.codes1, nsp, base + i, lane);
                }
        }
    }
    reduce_split(acc, red, slot, ks, lane);
    if (ks != 0 || pair >= npairs) return;

    Quant qin, qnext;
    if (EPI == EPI_HE4) {
        qin.init(*a.bound, a.code_bits);
        qnext.init(*a.next_bound, 8);
    }
    const int64_t next_nsp = a.next_ld / 64;
    bool bad = false;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        int next_sum[2] = {0, 0};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = g + 8 * (i >> 1);
            const int token = n * 8 + 2 * t + (i & 1);
            const int64_t o = pair * 16 + row;
            if (token >= a.tokens || o >= a.rows) continue;
            int dg[PLANES], du[PLANES];
#pragma unroll
            for (int p = 0; p < PLANES; ++p) {
                dg[p] = acc[0][p][n][i];
                du[p] = acc[1][p][n][i];
            }
            const int cs0 = code_sum(a.csum0, a.nparts, token);
            const int cs1 = PLANES == 2 ? code_sum(a.csum1, a.nparts, token) : 0;
            const int Dg = pm_dot<PLANES>(dg, cs0, cs1);
            const int Du = pm_dot<PLANES>(du, cs0, cs1);
            float gv, uv;
            if (EPI == EPI_HE4) {
                gv = he4_value(Dg, a.scale0[o], qin.step, cs0, a.mid0[o]);
                uv = he4_value(Du, a.scale1[o], qin.step, cs0, a.mid1[o]);
            } else if (EPI == EPI_W1) {
                const float rs = a.row_scale[token];
                gv = __fmul_rn(__fmul_rn(static_cast<float>(Dg), rs), a.scale0[o]);
                uv = __fmul_rn(__fmul_rn(static_cast<float>(Du), rs), a.scale1[o]);
            } else {
                const float rs = a.row_scale[token];
                gv = __fmul_rn(__fmul_rn(static_cast<float>(Dg), a.scale0[o]), rs);
                uv = __fmul_rn(__fmul_rn(static_cast<float>(Du), a.scale1[o]), rs);
            }
            const float h = __fmul_rn(silu(gv), uv);
            if (a.out) a.out[token * a.rows + o] = h;
            if (EPI == EPI_HE4) {
                const float gained = __fmul_rn(h, a.next_gain[o]);
                bad |= !isfinite(gained);
                const int code = qnext.code(gained);
                a.next_codes[frag_offset(token, o, next_nsp)] = static_cast<int8_t>(code);
                next_sum[i & 1] += code;
            }
        }
        if (EPI == EPI_HE4) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                int s = next_sum[j];
                s += __shfl_xor_sync(0xffffffffu, s, 4);
                s += __shfl_xor_sync(0xffffffffu, s, 8);
                s += __shfl_xor_sync(0xffffffffu, s, 16);
                const int token = n * 8 + 2 * t + j;
                if (g == 0 && token < a.tokens && s != 0) atomicAdd(a.next_csum + token, s);
            }
        }
    }
    if (EPI == EPI_HE4 && __any_sync(0xffffffffu, bad) && lane == 0) set_flag(a.flags, BD_FLAG_NONFINITE_INPUT);
}

// --------------------------------------------------------------------------- single-matrix kernel
template <int NT, int PLANES, int EPI>
__global__ void __launch_bounds__(kThreads) proj_kernel(const ProjArgs a) {
    __shared__ int red[kBlocksPerCta * 32 * PLANES * NT * 4];
    constexpr int TP = NT * 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int slot = warp / kSplit, ks = warp % kSplit;
    const int64_t nrb = (a.rows + 15) / 16;
    const int64_t rb = static_cast<int64_t>(blockIdx.x) * kBlocksPerCta + slot;
    const int ncp = static_cast<int>(a.ncp);
    const int kc0 = static_cast<int>(blockIdx.y) * ncp / a.kgroups;
    const int kc1 = static_cast<int>(blockIdx.y + 1) * ncp / a.kgroups;
    const int cp0 = kc0 + ks * (kc1 - kc0) / kSplit;
    const int cp1 = kc0 + (ks + 1) * (kc1 - kc0) / kSplit;
    const bool active = rb < nrb && cp0 < cp1;
    const int64_t nsp = a.ld / 64;

    const uint32_t *bits = a.bits + rb * a.ncp * 128 + lane * 4;
    uint4 wr[kBatch];
    if (active) {
#pragma unroll
        for (int i = 0; i < kBatch; ++i)
            if (cp0 + i < cp1) wr[i] = ld_stream_u4(bits + (cp0 + i) * 128);
    }
    grid_wait();
    grid_launch_dependents();

    int acc[1][PLANES][NT][4];
    zero_acc(acc);
    if (active) {
        for (int base = cp0; base < cp1; base += kBatch) {
            if (base != cp0) {
#pragma unroll
                for (int i = 0; i < kBatch; ++i)
                    if (base + i < cp1) wr[i] = ld_stream_u4(bits + (base + i) * 128);
            }
#pragma unroll
            for (int i = 0; i < kBatch; ++i)
                if (base + i < cp1) {
                    const uint4 w[1] = {wr[i]};
                    unit_mma<NT, PLANES, 1>(acc, w, a.codes0, a.codes1, nsp, base + i, lane);
                }
        }
    }
    reduce_split(acc, red, slot, ks, lane);
    if (ks != 0 || rb >= nrb) return;

    if (a.kgroups > 1) {
        // split-K across CTAs: integer partial sums meet in global accumulators;
        // the last arriving CTA of this row block reads them back (and leaves zeros).
        const int64_t rows_pad = nrb * 16;
#pragma unroll
        for (int p = 0; p < PLANES; ++p)
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int row = g + 8 * (i >> 1);
                    const int token = n * 8 + 2 * t + (i & 1);
                    const int v = acc[0][p][n][i];
                    if (v) atomicAdd(a.acc + (p * rows_pad + rb * 16 + row) * TP + token, v);
                }
        __threadfence();
        __syncwarp();
        int old = 0;
        if (lane == 0) old = atomicAdd(a.counters + rb, 1);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old != a.kgroups - 1) return;
        __threadfence();
#pragma unroll
        for (int p = 0; p < PLANES; ++p)
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int row = g + 8 * (i >> 1);
                    const int token = n * 8 + 2 * t + (i & 1);
                    acc[0][p][n][i] = atomicExch(a.acc + (p * rows_pad + rb * 16 + row) * TP + token, 0);
                }
        if (lane == 0) atomicExch(a.counters + rb, 0);
    }

    Quant qin;
    if (EPI == EPI_HE4) qin.init(*a.bound, a.code_bits);
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = g + 8 * (i >> 1);
            const int token = n * 8 + 2 * t + (i & 1);
            const int64_t o = rb * 16 + row;
            if (token >= a.tokens || o >= a.rows) continue;
            int d[PLANES];
#pragma unroll
            for (int p = 0; p < PLANES; ++p) d[p] = acc[0][p][n][i];
            const int cs0 = code_sum(a.csum0, a.nparts, token);
            const int cs1 = PLANES == 2 ? code_sum(a.csum1, a.nparts, token) : 0;
            const int D = pm_dot<PLANES>(d, cs0, cs1);
            float y;
            if (EPI == EPI_HE4) {
                y = he4_value(D, a.scale0[o], qin.step, cs0, a.mid0[o]);
            } else if (EPI == EPI_W1) {
                y = __fmul_rn(__fmul_rn(static_cast<float>(D), a.row_scale[token]), a.scale0[o]);
            } else {
                y = __fmul_rn(__fmul_rn(static_cast<float>(D), a.scale0[o]), a.row_scale[token]);
            }
            if (a.residual) y = __fadd_rn(a.residual[token * a.rows + o], y);
            a.out[token * a.rows + o] = y;
            if (a.raw_dot) a.raw_dot[token * a.rows + o] = D;
        }
}

// --------------------------------------------------------------------------- launchers

template <int NT, int PLANES, int EPI>
static int launch_gateup_t(const ProjArgs &a, cudaStream_t stream) {
    const int64_t npairs = (a.rows + 15) / 16;
    const unsigned grid = static_cast<unsigned>((npairs + kBlocksPerCta - 1) / kBlocksPerCta);
    return launch_pdl(gateup_kernel<NT, PLANES, EPI>, dim3(grid), dim3(kThreads), 0, stream, a);
}

template <int NT, int PLANES, int EPI>
static int launch_proj_t(const ProjArgs &a, cudaStream_t stream) {
    const int64_t nrb = (a.rows + 15) / 16;
    dim3 grid(static_cast<unsigned>((nrb + kBlocksPerCta - 1) / kBlocksPerCta), static_cast<unsigned>(a.kgroups));
    return launch_pdl(proj_kernel<NT, PLANES, EPI>, grid, dim3(kThreads), 0, stream, a);
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
    if (a.tokens < 1 || a.tokens > 32 || a.kgroups < 1 || a.nparts < 1) return BD_ERR_INVALID;
    if (epi == EPI_HE4) BD_DISPATCH_NT(launch_proj_t, 1, EPI_HE4);
    if (epi == EPI_W1) BD_DISPATCH_NT(launch_proj_t, 2, EPI_W1);
    BD_DISPATCH_NT(launch_proj_t, 1, EPI_W1A1);
}

// K groups (CTAs along K) for the single-matrix kernel: about two waves of
// CTAs, at least kSplit column pairs per group.
int choose_kgroups(int64_t rows, int64_t ncp, int sms) {
    const int64_t ctas = ((rows + 15) / 16 + kBlocksPerCta - 1) / kBlocksPerCta;
    int64_t kg = (2 * sms + ctas - 1) / ctas;
    if (kg > ncp / kSplit) kg = ncp / kSplit;
    if (kg < 1) kg = 1;
    return static_cast<int>(kg);
}

}  // namespace bd
