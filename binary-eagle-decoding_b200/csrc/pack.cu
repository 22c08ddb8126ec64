// Sign packing: GGUF words (export.packed_signs) and the T16 tiled decode layout.
#include "common.cuh"

namespace bd {

// One warp per GGUF word: lane l looks at column 32 w + l; a ballot is the word.
__global__ void pack_signs_kernel(const float *__restrict__ latent, int64_t rows, int64_t cols,
                                  int32_t *__restrict__ words, int32_t *flags) {
    const int lane = threadIdx.x & 31;
    const int64_t nwords = (cols + 31) / 32;
    const int64_t total = rows * nwords;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    bool bad = false;
    for (int64_t item = warp; item < total; item += nwarps) {
        const int64_t r = item / nwords, w = item - r * nwords;
        const int64_t c = w * 32 + lane;
        bool bit = false;
        if (c < cols) {
            const float v = latent[r * cols + c];
            bad |= !isfinite(v);
            bit = v >= 0.0f;  // -0.0 counts as non-negative
        }
        const unsigned word = __ballot_sync(0xffffffffu, bit);
        if (lane == 0) words[item] = static_cast<int32_t>(word);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) set_flag(flags, BD_FLAG_NONFINITE_LATENT);
}

// Spread the 4 low bits of x to bit 0 of each byte.
__device__ __forceinline__ uint32_t spread4(uint32_t x) { return (x * 0x00204081u) & 0x01010101u; }

// T16 word of (row, chunk c in {0,1}, lane t) from the 8 GGUF words g[0..7] of
// a 256-column pair: bit (8 j + 2 q + h) = bit (16 h + 4 t + j) of g[4 c + q].
__device__ __forceinline__ uint32_t t16_word(const uint32_t *g, int c, int t) {
    uint32_t out = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t word = g[4 * c + q];
        out |= spread4((word >> (4 * t)) & 0xFu) << (2 * q);
        out |= spread4((word >> (16 + 4 * t)) & 0xFu) << (2 * q + 1);
    }
    return out;
}

__device__ __forceinline__ int64_t t16_offset(int64_t row, int64_t cp, int64_t ncp, int c, int t, int stride,
                                              int offset) {
    const int64_t rb = (row >> 4) * stride + offset;
    const int rr = static_cast<int>(row & 15);
    const int lane = (rr & 7) * 4 + t;
    const int w = (rr >> 3) + 2 * c;
    return (rb * ncp + cp) * 128 + lane * 4 + w;
}

// One warp per (row, column pair): eight ballots give the eight GGUF words of
// the pair; lanes 0..7 emit the eight T16 words of this row.
__global__ void tile_t16_kernel(const float *__restrict__ latent, int64_t rows, int64_t cols, int64_t ncp,
                                uint32_t *__restrict__ tiled, int stride, int offset, int32_t *flags) {
    const int lane = threadIdx.x & 31;
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5;
    const int64_t rows_pad = (rows + 15) / 16 * 16;
    bool bad = false;
    for (int64_t item = warp; item < rows_pad * ncp; item += nwarps) {
        const int64_t row = item / ncp, cp = item - row * ncp;
        uint32_t g[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int64_t c = cp * 256 + i * 32 + lane;
            bool bit = false;
            if (row < rows && c < cols) {
                const float v = latent[row * cols + c];
                bad |= !isfinite(v);
                bit = v >= 0.0f;
            }
            g[i] = __ballot_sync(0xffffffffu, bit);
        }
        if (lane < 8) {
            const int c = lane >> 2, t = lane & 3;
            tiled[t16_offset(row, cp, ncp, c, t, stride, offset)] = t16_word(g, c, t);
        }
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) set_flag(flags, BD_FLAG_NONFINITE_LATENT);
}

// One thread per T16 word, reading four GGUF words of its row.
__global__ void tile_gguf_kernel(const int32_t *__restrict__ words, int64_t rows, int64_t cols, int64_t ncp,
                                 uint32_t *__restrict__ tiled, int stride, int offset) {
    const int64_t nwords = (cols + 31) / 32;
    const int64_t rows_pad = (rows + 15) / 16 * 16;
    const int64_t total = rows_pad * ncp * 8;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int ct = static_cast<int>(i & 7);
        const int64_t rest = i >> 3;
        const int64_t row = rest / ncp, cp = rest - row * ncp;
        const int c = ct >> 2, t = ct & 3;
        uint32_t g[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int64_t w = cp * 8 + k;
            g[k] = (row < rows && w < nwords) ? static_cast<uint32_t>(words[row * nwords + w]) : 0u;
        }
        tiled[t16_offset(row, cp, ncp, c, t, stride, offset)] = t16_word(g, c, t);
    }
}

}  // namespace bd

using namespace bd;

static int grid_for(int64_t items, int per_block) {
    int64_t g = (items + per_block - 1) / per_block;
    if (g < 1) g = 1;
    if (g > 148 * 16) g = 148 * 16;
    return static_cast<int>(g);
}

extern "C" int bd_pack_signs(const float *latent, int64_t rows, int64_t cols, int32_t *words, int32_t *flags,
                             bd_stream_t stream) {
    if (rows < 0 || cols < 0 || (rows * cols > 0 && (!latent || !words))) return BD_ERR_INVALID;
    const int64_t total = rows * ((cols + 31) / 32);
    if (total == 0) return BD_OK;
    pack_signs_kernel<<<grid_for(total, 8), 256, 0, stream>>>(latent, rows, cols, words, flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int64_t bd_t16_words(int64_t rows, int64_t cols) {
    if (rows < 0 || cols < 0) return -1;
    return ((rows + 15) / 16) * ((cols + 255) / 256) * 128;
}

extern "C" int bd_tile_signs_t16(const float *latent, int64_t rows, int64_t cols, uint32_t *tiled,
                                 int block_stride, int block_offset, int32_t *flags, bd_stream_t stream) {
    if (rows < 0 || cols < 0 || block_stride < 1 || block_offset < 0 || block_offset >= block_stride)
        return BD_ERR_INVALID;
    if (rows == 0 || cols == 0) return BD_OK;
    if (!latent || !tiled) return BD_ERR_INVALID;
    const int64_t ncp = (cols + 255) / 256;
    const int64_t items = (rows + 15) / 16 * 16 * ncp;
    tile_t16_kernel<<<grid_for(items, 8), 256, 0, stream>>>(latent, rows, cols, ncp, tiled, block_stride,
                                                           block_offset, flags);
    BD_CHECK_LAUNCH();
    return BD_OK;
}

extern "C" int bd_tile_gguf_t16(const int32_t *words, int64_t rows, int64_t cols, uint32_t *tiled, int block_stride,
                                int block_offset, bd_stream_t stream) {
    if (rows < 0 || cols < 0 || block_stride < 1 || block_offset < 0 || block_offset >= block_stride)
        return BD_ERR_INVALID;
    if (rows == 0 || cols == 0) return BD_OK;
    if (!words || !tiled) return BD_ERR_INVALID;
    const int64_t ncp = (cols + 255) / 256;
    const int64_t total = (rows + 15) / 16 * 16 * ncp * 8;
    tile_gguf_kernel<<<grid_for(total, 256), 256, 0, stream>>>(words, rows, cols, ncp, tiled, block_stride,
                                                              block_offset);
    BD_CHECK_LAUNCH();
    return BD_OK;
}
