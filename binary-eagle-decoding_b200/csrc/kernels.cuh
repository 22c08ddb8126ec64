// Internal launch helpers shared between the library's translation units.
#pragma once

#include <utility>

#include "common.cuh"

namespace bd {

// Launch with programmatic stream serialization (the kernel calls grid_wait()
// before touching anything an earlier kernel writes).
template <typename... KArgs, typename... Args>
int launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    // a stream created with a priority passes it to its launches explicitly, so that
    // a CUDA graph captured from it keeps the priority on its kernel nodes
    int priority = 0;
    if (cudaStreamGetPriority(stream, &priority) == cudaSuccess && priority != 0) {
        attr[1].id = cudaLaunchAttributePriority;
        attr[1].val.priority = priority;
        cfg.numAttrs = 2;
    }
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) == cudaSuccess ? BD_OK : BD_ERR_LAUNCH;
}

// Column slices (of 1024) of the HE4 quantizer grid = partial code sums per row.
inline int quant_parts(int64_t cols) { return static_cast<int>((cols + 1023) / 1024); }

int launch_quantize_codes(const float *x, int64_t rows, int64_t cols, int64_t ld, const float *gain,
                          const float *bound, int bits, int8_t *codes, int32_t *sums, bool partial, int32_t *flags,
                          int32_t *zero_sums, int zero_count, cudaStream_t stream, const float *norm_w = nullptr,
                          float eps = 0.0f, int c16_mt = 0);
int launch_quantize_planes(const float *x, int64_t rows, int64_t cols, int64_t ld, int8_t *hi, int8_t *lo,
                           int32_t *sums_hi, int32_t *sums_lo, float *row_scale, int32_t *flags,
                           cudaStream_t stream, int c16_mt = 0);
int launch_binarize(const float *x, int64_t rows, int64_t cols, int64_t ld, int8_t *codes, int32_t *sums,
                    float *mean_abs, uint32_t *words, int64_t words_ld, int32_t *flags, cudaStream_t stream,
                    int c16_mt = 0);

// ---- W8 / C16 decode feed-forward (ffn8.cu): tokens are the MMA's M side
int64_t w8_words(int64_t rows, int64_t cols);  // uint32 words of one W8 matrix
struct FfnW8 {
    int tokens;
    int64_t hidden, inter;
    const uint32_t *signs_gate_up, *signs_down;  // W8; gate/up n-tiles interleaved
    const float *scale_gate, *mid_gate, *scale_up, *mid_up, *scale_down, *mid_down;
    const float *gain_gate_up, *bound_gate_up, *gain_down, *bound_down;
    const float *x, *residual, *norm_w;
    float eps;
    float *y, *hidden_out;
    int32_t *flags;
    void *workspace;
    size_t workspace_bytes;
};
size_t ffn_w8_workspace_bytes(int64_t hidden, int64_t inter);
int ffn_w8(const FfnW8 &f, int epi, cudaStream_t stream);

// ---- two-launch HE4 block for tokens <= 16 (ffn_fused.cu): W8 gate/up words, D8 down bytes
int64_t d8_bytes(int64_t rows, int64_t cols);
size_t ffn_fused_workspace_bytes(int64_t hidden, int64_t inter);
int ffn_fused_he4(const FfnW8 &f, const uint8_t *signs_down_d8, cudaStream_t stream);
int ffn_fused_shape(int64_t hidden, int64_t inter, int *shape);

// Epilogue selectors of the T16 integer-MMA projection kernels.
enum Epilogue : int {
    EPI_HE4 = 0,   // HE4 projection value (+ residual)
    EPI_W1 = 1,    // (D * row_scale[t]) * scale[o]   (two int8 planes)
    EPI_W1A1 = 2,  // (D * scale[o]) * mean_abs[t]
};

// Arguments of one T16 projection (single matrix or gate/up pair).
struct ProjArgs {
    const uint32_t *bits;     // T16 words (rb-major units; pairs: virtual rb 2p+m)
    int64_t rows;             // output features (per matrix)
    int64_t cols;             // input features
    int64_t ncp;              // column pairs
    const int8_t *codes0;     // F8 fragment layout (frag_offset), plane 0
    const int8_t *codes1;     // plane 1 (W1) or null
    const int32_t *csum0;     // [tokens][nparts] partial code sums
    const int32_t *csum1;
    int nparts;               // partial sums per token (1: full sums)
    int64_t ld;               // codes row stride (multiple of 256)
    int tokens;
    int kgroups;              // CTAs along K (single-matrix kernel)
    int blocks_per_cta;       // row blocks per CTA (single-matrix kernel)
    // epilogue operands (matrix 0 = gate or the single matrix, 1 = up)
    const float *scale0, *mid0, *scale1, *mid1;
    const float *bound;       // HE4 bound of this projection's codes
    int code_bits;            // HE4 code bits of this projection's input
    const float *row_scale;   // W1 per-token scale, W1A1 per-token mean|x|
    const float *residual;    // [tokens][rows] or null
    float *out;               // [tokens][rows] (single matrix) or hidden [tokens][rows] (pair)
    int32_t *raw_dot;         // optional [tokens][rows] exact +-1 dot (single matrix)
    // gate/up -> down hand-off (HE4): next projection's codes
    const float *next_gain, *next_bound;
    int8_t *next_codes;       // [tokens][next_ld]
    int32_t *next_csum;       // [tokens] (accumulated with atomics; zeroed by the caller)
    int64_t next_ld;
    // split-K accumulators (single matrix, kgroups > 1)
    int32_t *acc;             // [planes][rows_pad][tpad] zero on entry, left zero
    int32_t *counters;        // [nrb] zero on entry, left zero
    int32_t *flags;
};

int launch_gateup(const ProjArgs &a, int epi, cudaStream_t stream);
int launch_proj(const ProjArgs &a, int epi, cudaStream_t stream);
// Choose kgroups / blocks_per_cta of a single-matrix projection (one CTA wave).
void plan_proj(ProjArgs &a, int planes);

}  // namespace bd
