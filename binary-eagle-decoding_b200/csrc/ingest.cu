// Teacher-feature ingestion: tap-major captures [taps][rows][hidden] (fp16 or
// fp32, as the capture files store them) become the drafter's token-major
// features [rows][taps * hidden] (fp16, bf16 or fp32), with the finiteness scan
// of the capture loader (w1a1_eagle/numerical/captures.py:34-40, 124-131).
// One thread moves 8 contiguous values of one tap row: a 16-byte (fp16) or two
// 16-byte (fp32) loads, a bit test of every exponent, and one or two 16-byte
// stores; reads and writes are both fully coalesced.
#include "kernels.cuh"

namespace bd {

constexpr int kIngestThreads = 256;

// Non-finite test on raw bits: fp16 exponent all ones, fp32 exponent all ones.
__device__ __forceinline__ bool bad_f16x2(uint32_t w) {
    return ((w & 0x7C00u) == 0x7C00u) || ((w & 0x7C000000u) == 0x7C000000u);
}
__device__ __forceinline__ bool bad_f32(uint32_t w) { return (w & 0x7F800000u) == 0x7F800000u; }

__device__ __forceinline__ float h2f(uint32_t h) { return __half2float(__ushort_as_half(static_cast<unsigned short>(h))); }

// out element type: 0 fp16, 1 bf16, 2 fp32
template <int IN_F32, int OUT>
__global__ void __launch_bounds__(kIngestThreads) ingest_taps_kernel(const void *__restrict__ src, int taps,
                                                                     int64_t rows, int64_t hidden,
                                                                     void *__restrict__ dst, int32_t *flags) {
    const int64_t vec_per_row = hidden / 8;
    const int64_t total = static_cast<int64_t>(taps) * rows * vec_per_row;
    bool bad = false;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t v = i % vec_per_row, rest = i / vec_per_row;
        const int64_t row = rest % rows, tap = rest / rows;
        float f[8];
        uint32_t h[4];  // fp16 pairs when the input is fp16
        if (IN_F32) {
            const uint4 *p = reinterpret_cast<const uint4 *>(static_cast<const float *>(src) + i * 8);
            const uint4 a = __ldg(p), b = __ldg(p + 1);
            const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                bad |= bad_f32(w[k]);
                f[k] = __uint_as_float(w[k]);
            }
        } else {
            const uint4 a = __ldg(reinterpret_cast<const uint4 *>(static_cast<const uint16_t *>(src) + i * 8));
            h[0] = a.x;
            h[1] = a.y;
            h[2] = a.z;
            h[3] = a.w;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                bad |= bad_f16x2(h[k]);
                f[2 * k] = h2f(h[k] & 0xFFFFu);
                f[2 * k + 1] = h2f(h[k] >> 16);
            }
        }
        const int64_t o = row * taps * hidden + tap * hidden + v * 8;  // element offset in [rows][taps * hidden]
        if (OUT == 2) {
            float4 *q = reinterpret_cast<float4 *>(static_cast<float *>(dst) + o);
            q[0] = make_float4(f[0], f[1], f[2], f[3]);
            q[1] = make_float4(f[4], f[5], f[6], f[7]);
        } else if (OUT == 1) {
            uint32_t w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const __nv_bfloat162 b2 = __floats2bfloat162_rn(f[2 * k], f[2 * k + 1]);
                w[k] = *reinterpret_cast<const uint32_t *>(&b2);
            }
            *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(dst) + o) = make_uint4(w[0], w[1], w[2], w[3]);
        } else {
            uint32_t w[4];
            if (IN_F32) {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const __half2 h2 = __floats2half2_rn(f[2 * k], f[2 * k + 1]);
                    w[k] = *reinterpret_cast<const uint32_t *>(&h2);
                }
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) w[k] = h[k];
            }
            *reinterpret_cast<uint4 *>(static_cast<uint16_t *>(dst) + o) = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) set_flag(flags, BD_FLAG_NONFINITE_FEATURES);
}

}  // namespace bd

using namespace bd;

extern "C" int bd_ingest_taps(const void *taps_src, int in_dtype_bits, int taps, int64_t rows, int64_t hidden,
                              void *features, int out_dtype, int32_t *flags, bd_stream_t stream) {
    if (taps < 1 || rows < 0 || hidden < 8 || hidden % 8 || (in_dtype_bits != 16 && in_dtype_bits != 32) ||
        out_dtype < 0 || out_dtype > 2)
        return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    if (!taps_src || !features) return BD_ERR_INVALID;
    if ((reinterpret_cast<uintptr_t>(taps_src) & 15) || (reinterpret_cast<uintptr_t>(features) & 15))
        return BD_ERR_ALIGNMENT;
    const int64_t total = static_cast<int64_t>(taps) * rows * (hidden / 8);
    int64_t grid = (total + kIngestThreads - 1) / kIngestThreads;
    if (grid > 148 * 16) grid = 148 * 16;
    const dim3 g(static_cast<unsigned>(grid)), b(kIngestThreads);
    const bool f32 = in_dtype_bits == 32;
    auto s = static_cast<cudaStream_t>(stream);
    switch (out_dtype + (f32 ? 3 : 0)) {
        case 0: ingest_taps_kernel<0, 0><<<g, b, 0, s>>>(taps_src, taps, rows, hidden, features, flags); break;
        case 1: ingest_taps_kernel<0, 1><<<g, b, 0, s>>>(taps_src, taps, rows, hidden, features, flags); break;
        case 2: ingest_taps_kernel<0, 2><<<g, b, 0, s>>>(taps_src, taps, rows, hidden, features, flags); break;
        case 3: ingest_taps_kernel<1, 0><<<g, b, 0, s>>>(taps_src, taps, rows, hidden, features, flags); break;
        case 4: ingest_taps_kernel<1, 1><<<g, b, 0, s>>>(taps_src, taps, rows, hidden, features, flags); break;
        default: ingest_taps_kernel<1, 2><<<g, b, 0, s>>>(taps_src, taps, rows, hidden, features, flags); break;
    }
    BD_CHECK_LAUNCH();
    return BD_OK;
}
