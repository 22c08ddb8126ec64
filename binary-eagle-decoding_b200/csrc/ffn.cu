// Decode-size (tokens <= 32) packed-sign projections on the integer tensor pipe.
//
// Weights arrive as T16 sign words (see pack.cu); each lane expands its 16-byte
// slice of a 512-byte unit directly into the 0/1 int8 A fragments of
// m16n8k32 MMAs (two instructions per register, no shared memory for weights).
// Activations are int8 codes staged once per CTA in shared memory (B operand).
// With b in {0,1} (b = 1 for latent >= 0) the +-1 dot is D = 2 * D01 - sum(codes),
// exact in int32, so every epilogue starts from the exact integer dot.
#include "kernels.cuh"

namespace bd {

constexpr int kThreads = 256;
constexpr int kPairsPerCta = 4;  // gate/up kernel: 4 row-block pairs x 2 K halves = 8 warps
constexpr int kRbPerCta = 4;     // single-matrix kernel: 4 row blocks x 2 K halves
constexpr int kBatch = 8;        // column pairs held in registers per batch

__device__ __forceinline__ void stage_codes(int8_t *smem, const int8_t *codes, int64_t ld, int64_t k0, int klen,
                                            int tokens, int tpad) {
    const int lds = klen + 16;
    const int vpr = klen / 16;
    for (int i = threadIdx.x; i < tpad * vpr; i += blockDim.x) {
        const int t = i / vpr, v = i - t * vpr;
        uint4 val = make_uint4(0u, 0u, 0u, 0u);
        if (t < tokens) val = *reinterpret_cast<const uint4 *>(codes + t * ld + k0 + v * 16);
        *reinterpret_cast<uint4 *>(smem + t * lds + v * 16) = val;
    }
}

// Multiply one 256-column unit (lane words w) with the staged codes.
template <int NT, int PLANES>
__device__ __forceinline__ void unit_mma(int (&acc)[PLANES][NT][4], const uint4 w, const int8_t *sm0,
                                         const int8_t *sm1, int lds, int kc, int g, int t) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const uint32_t wa = c ? w.z : w.x;  // row g
        const uint32_t wb = c ? w.w : w.y;  // row g + 8
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const uint32_t a0 = (wa >> (2 * q)) & 0x01010101u;
            const uint32_t a1 = (wb >> (2 * q)) & 0x01010101u;
            const uint32_t a2 = (wa >> (2 * q + 1)) & 0x01010101u;
            const uint32_t a3 = (wb >> (2 * q + 1)) & 0x01010101u;
            const int col = kc + 128 * c + 32 * q + 4 * t;
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
                const int off = (nt * 8 + g) * lds + col;
                mma_s8_16832(acc[0][nt], a0, a1, a2, a3, *reinterpret_cast<const uint32_t *>(sm0 + off),
                             *reinterpret_cast<const uint32_t *>(sm0 + off + 16));
                if (PLANES == 2)
                    mma_s8_16832(acc[PLANES - 1][nt], a0, a1, a2, a3,
                                 *reinterpret_cast<const uint32_t *>(sm1 + off),
                                 *reinterpret_cast<const uint32_t *>(sm1 + off + 16));
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

// --------------------------------------------------------------------------- gate/up pair kernel
template <int NT, int PLANES, int EPI>
__global__ void __launch_bounds__(kThreads) gateup_kernel(const ProjArgs a) {
    extern __shared__ __align__(16) int8_t smem[];
    constexpr int TP = NT * 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int64_t npairs = (a.rows + 15) / 16;
    const int64_t pair = static_cast<int64_t>(blockIdx.x) * kPairsPerCta + (warp >> 1);
    const int kh = warp & 1;
    const int half = static_cast<int>((a.ncp + 1) / 2);
    const int cp0 = kh * half;
    const int cp1 = min(static_cast<int>(a.ncp), cp0 + half);
    const bool active = pair < npairs && cp0 < cp1;
    const int lds = static_cast<int>(a.ld) + 16;
    int8_t *sm0 = smem;
    int8_t *sm1 = smem + TP * lds;

    const uint32_t *gate_bits = a.bits + (2 * pair) * a.ncp * 128 + lane * 4;
    const uint32_t *up_bits = a.bits + (2 * pair + 1) * a.ncp * 128 + lane * 4;
    uint4 wg[kBatch], wu[kBatch];
    if (active) {
#pragma unroll
        for (int i = 0; i < kBatch; ++i)
            if (cp0 + i < cp1) {
                wg[i] = ld_stream_u4(gate_bits + (cp0 + i) * 128);
                wu[i] = ld_stream_u4(up_bits + (cp0 + i) * 128);
            }
    }
    stage_codes(sm0, a.codes0, a.ld, 0, static_cast<int>(a.ld), a.tokens, TP);
    if (PLANES == 2) stage_codes(sm1, a.codes1, a.ld, 0, static_cast<int>(a.ld), a.tokens, TP);
    __syncthreads();

    int ag[PLANES][NT][4], au[PLANES][NT][4];
#pragma unroll
    for (int p = 0; p < PLANES; ++p)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) ag[p][n][i] = au[p][n][i] = 0;

    if (active) {
        for (int base = cp0; base < cp1; base += kBatch) {
            if (base != cp0) {
#pragma unroll
                for (int i = 0; i < kBatch; ++i)
                    if (base + i < cp1) {
                        wg[i] = ld_stream_u4(gate_bits + (base + i) * 128);
                        wu[i] = ld_stream_u4(up_bits + (base + i) * 128);
                    }
            }
#pragma unroll
            for (int i = 0; i < kBatch; ++i)
                if (base + i < cp1) {
                    unit_mma<NT, PLANES>(ag, wg[i], sm0, sm1, lds, (base + i) * 256, g, t);
                    unit_mma<NT, PLANES>(au, wu[i], sm0, sm1, lds, (base + i) * 256, g, t);
                }
        }
    }
    // combine the two K halves of each pair through shared memory
    __syncthreads();
    constexpr int VALS = PLANES * NT * 4;
    int *red = reinterpret_cast<int *>(smem) + (warp >> 1) * 32 * 2 * VALS + lane * 2 * VALS;
    if (kh == 1) {
#pragma unroll
        for (int p = 0; p < PLANES; ++p)
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    red[(p * NT + n) * 4 + i] = ag[p][n][i];
                    red[VALS + (p * NT + n) * 4 + i] = au[p][n][i];
                }
    }
    __syncthreads();
    if (kh == 1 || pair >= npairs) return;
#pragma unroll
    for (int p = 0; p < PLANES; ++p)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                ag[p][n][i] += red[(p * NT + n) * 4 + i];
                au[p][n][i] += red[VALS + (p * NT + n) * 4 + i];
            }

    // epilogue
    Quant qin, qnext;
    if (EPI == EPI_HE4) {
        qin.init(*a.bound, a.code_bits);
        qnext.init(*a.next_bound, 8);
    }
    bool bad = false;
#pragma unroll
    for (int n = 0; n < NT; ++n) {
        int code_sum[2] = {0, 0};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int row = g + 8 * (i >> 1);
            const int token = n * 8 + 2 * t + (i & 1);
            const int64_t o = pair * 16 + row;
            if (token >= a.tokens || o >= a.rows) continue;
            int dg[PLANES], du[PLANES];
#pragma unroll
            for (int p = 0; p < PLANES; ++p) {
                dg[p] = ag[p][n][i];
                du[p] = au[p][n][i];
            }
            const int cs0 = a.csum0[token];
            const int cs1 = PLANES == 2 ? a.csum1[token] : 0;
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
                a.next_codes[token * a.next_ld + o] = static_cast<int8_t>(code);
                code_sum[i & 1] += code;
            }
        }
        if (EPI == EPI_HE4) {
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                int s = code_sum[j];
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
    extern __shared__ __align__(16) int8_t smem[];
    constexpr int TP = NT * 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const int64_t nrb = (a.rows + 15) / 16;
    const int64_t rb = static_cast<int64_t>(blockIdx.x) * kRbPerCta + (warp >> 1);
    const int kh = warp & 1;
    const int per = static_cast<int>((a.ncp + a.kgroups - 1) / a.kgroups);
    const int kc0 = blockIdx.y * per;
    const int kc1 = min(static_cast<int>(a.ncp), kc0 + per);
    const int half = (kc1 - kc0 + 1) / 2;
    const int cp0 = kc0 + kh * half;
    const int cp1 = min(kc1, cp0 + half);
    const bool active = rb < nrb && cp0 < cp1;
    const int klen = per * 256;
    const int lds = klen + 16;
    int8_t *sm0 = smem;
    int8_t *sm1 = smem + TP * lds;

    const uint32_t *bits = a.bits + rb * a.ncp * 128 + lane * 4;
    uint4 wr[kBatch];
    if (active) {
#pragma unroll
        for (int i = 0; i < kBatch; ++i)
            if (cp0 + i < cp1) wr[i] = ld_stream_u4(bits + (cp0 + i) * 128);
    }
    const int slice = (kc1 - kc0) * 256;
    if (slice > 0) {
        stage_codes(sm0, a.codes0, a.ld, static_cast<int64_t>(kc0) * 256, slice, a.tokens, TP);
        if (PLANES == 2) stage_codes(sm1, a.codes1, a.ld, static_cast<int64_t>(kc0) * 256, slice, a.tokens, TP);
    }
    __syncthreads();

    int acc[PLANES][NT][4];
#pragma unroll
    for (int p = 0; p < PLANES; ++p)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[p][n][i] = 0;
    if (active) {
        for (int base = cp0; base < cp1; base += kBatch) {
            if (base != cp0) {
#pragma unroll
                for (int i = 0; i < kBatch; ++i)
                    if (base + i < cp1) wr[i] = ld_stream_u4(bits + (base + i) * 128);
            }
#pragma unroll
            for (int i = 0; i < kBatch; ++i)
                if (base + i < cp1) unit_mma<NT, PLANES>(acc, wr[i], sm0, sm1, lds, (base + i - kc0) * 256, g, t);
        }
    }
    __syncthreads();
    constexpr int VALS = PLANES * NT * 4;
    int *red = reinterpret_cast<int *>(smem) + (warp >> 1) * 32 * VALS + lane * VALS;
    if (kh == 1) {
#pragma unroll
        for (int p = 0; p < PLANES; ++p)
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) red[(p * NT + n) * 4 + i] = acc[p][n][i];
    }
    __syncthreads();
    if (kh == 1 || rb >= nrb) return;
#pragma unroll
    for (int p = 0; p < PLANES; ++p)
#pragma unroll
        for (int n = 0; n < NT; ++n)
#pragma unroll
            for (int i = 0; i < 4; ++i) acc[p][n][i] += red[(p * NT + n) * 4 + i];

    if (a.kgroups > 1) {
        // split-K: integer partial sums meet in global accumulators; the last
        // arriving CTA of this row block reads them back (and leaves zeros).
        const int64_t rows_pad = nrb * 16;
#pragma unroll
        for (int p = 0; p < PLANES; ++p)
#pragma unroll
            for (int n = 0; n < NT; ++n)
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const int row = g + 8 * (i >> 1);
                    const int token = n * 8 + 2 * t + (i & 1);
                    const int v = acc[p][n][i];
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
                    acc[p][n][i] = atomicExch(a.acc + (p * rows_pad + rb * 16 + row) * TP + token, 0);
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
            for (int p = 0; p < PLANES; ++p) d[p] = acc[p][n][i];
            const int cs0 = a.csum0[token];
            const int cs1 = PLANES == 2 ? a.csum1[token] : 0;
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
    constexpr int TP = NT * 8;
    const size_t codes = static_cast<size_t>(TP) * (a.ld + 16) * PLANES;
    const size_t red = static_cast<size_t>(kPairsPerCta) * 32 * 2 * PLANES * NT * 4 * sizeof(int);
    const size_t bytes = codes > red ? codes : red;
    if (bytes > 227 * 1024) return BD_ERR_INVALID;
    auto kern = gateup_kernel<NT, PLANES, EPI>;
    if (bytes > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) !=
            cudaSuccess)
        return BD_ERR_LAUNCH;
    const int64_t npairs = (a.rows + 15) / 16;
    const unsigned grid = static_cast<unsigned>((npairs + kPairsPerCta - 1) / kPairsPerCta);
    kern<<<grid, kThreads, bytes, stream>>>(a);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

template <int NT, int PLANES, int EPI>
static int launch_proj_t(const ProjArgs &a, cudaStream_t stream) {
    constexpr int TP = NT * 8;
    const int per = static_cast<int>((a.ncp + a.kgroups - 1) / a.kgroups);
    const size_t codes = static_cast<size_t>(TP) * (per * 256 + 16) * PLANES;
    const size_t red = static_cast<size_t>(kRbPerCta) * 32 * PLANES * NT * 4 * sizeof(int);
    const size_t bytes = codes > red ? codes : red;
    if (bytes > 227 * 1024) return BD_ERR_INVALID;
    auto kern = proj_kernel<NT, PLANES, EPI>;
    if (bytes > 48 * 1024 &&
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes)) !=
            cudaSuccess)
        return BD_ERR_LAUNCH;
    const int64_t nrb = (a.rows + 15) / 16;
    dim3 grid(static_cast<unsigned>((nrb + kRbPerCta - 1) / kRbPerCta), static_cast<unsigned>(a.kgroups));
    kern<<<grid, kThreads, bytes, stream>>>(a);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

#define BD_DISPATCH_NT(fn, planes, epi)                                  \
    do {                                                                 \
        if (a.tokens <= 8) return fn<1, planes, epi>(a, stream);         \
        if (a.tokens <= 16) return fn<2, planes, epi>(a, stream);        \
        return fn<4, planes, epi>(a, stream);                            \
    } while (0)

int launch_gateup(const ProjArgs &a, int epi, cudaStream_t stream) {
    if (a.tokens < 1 || a.tokens > 32) return BD_ERR_INVALID;
    if (epi == EPI_HE4) BD_DISPATCH_NT(launch_gateup_t, 1, EPI_HE4);
    if (epi == EPI_W1) BD_DISPATCH_NT(launch_gateup_t, 2, EPI_W1);
    BD_DISPATCH_NT(launch_gateup_t, 1, EPI_W1A1);
}

int launch_proj(const ProjArgs &a, int epi, cudaStream_t stream) {
    if (a.tokens < 1 || a.tokens > 32 || a.kgroups < 1) return BD_ERR_INVALID;
    if (epi == EPI_HE4) BD_DISPATCH_NT(launch_proj_t, 1, EPI_HE4);
    if (epi == EPI_W1) BD_DISPATCH_NT(launch_proj_t, 2, EPI_W1);
    BD_DISPATCH_NT(launch_proj_t, 1, EPI_W1A1);
}

// K groups for the single-matrix kernel: about one wave of CTAs, at least two
// column pairs per group.
int choose_kgroups(int64_t rows, int64_t ncp, int sms) {
    const int64_t groups = ((rows + 15) / 16 + kRbPerCta - 1) / kRbPerCta;
    int64_t kg = (sms + groups - 1) / groups;
    if (kg > ncp / 2) kg = ncp / 2;
    if (kg < 1) kg = 1;
    return static_cast<int>(kg);
}

}  // namespace bd
