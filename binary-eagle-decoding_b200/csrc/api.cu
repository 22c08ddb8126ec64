// C-ABI entry points: validation, workspace carving and launch sequencing.
#include <mutex>

#include "kernels.cuh"

namespace bd {

constexpr int kMaxTokens = 32;

// Bump allocator over a caller-provided workspace (256-byte aligned pieces).
struct Carver {
    char *base;
    size_t off = 0;
    template <typename T>
    T *take(size_t count) {
        off = (off + 255) & ~static_cast<size_t>(255);
        T *p = base ? reinterpret_cast<T *>(base + off) : nullptr;
        off += count * sizeof(T);
        return p;
    }
};

static int sm_count_cached() {
    static int cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (!cached[dev]) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev] = n;
    }
    return cached[dev];
}


}  // namespace bd

using namespace bd;

extern "C" int bd_abi_version(void) { return 1; }

extern "C" const char *bd_status_string(int status) {
    switch (status) {
        case BD_OK: return "ok";
        case BD_ERR_INVALID: return "invalid argument or unsupported size";
        case BD_ERR_ALIGNMENT: return "misaligned pointer";
        case BD_ERR_LAUNCH: return "CUDA launch or runtime error";
        case BD_ERR_WORKSPACE: return "workspace too small";
        case BD_ERR_DEVICE: return "no usable sm_100 device";
        case BD_ERR_TOO_LARGE: return "size exceeds the fixed scratch capacity of this entry point";
        default: return "unknown status";
    }
}

extern "C" int bd_device_info(int *sm_count, int *major, int *minor) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return BD_ERR_DEVICE;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) return BD_ERR_DEVICE;
    if (sm_count) *sm_count = prop.multiProcessorCount;
    if (major) *major = prop.major;
    if (minor) *minor = prop.minor;
    return BD_OK;
}

extern "C" size_t bd_projection_workspace_bytes(int tokens, int64_t out_features) {
    (void)tokens;
    Carver c{nullptr};
    c.take<int32_t>(2 * ((out_features + 15) / 16 * 16) * kMaxTokens);
    c.take<int32_t>((out_features + 15) / 16);
    return c.off;
}

extern "C" int bd_projection_he4(const int8_t *codes, const int32_t *code_sums, int tokens, int64_t in_features,
                                 int64_t out_features, const uint32_t *signs_t16, const float *scale,
                                 const float *midpoint, const float *bound, int bits, const float *residual, float *y,
                                 int32_t *raw_dot, void *workspace, size_t workspace_bytes, bd_stream_t stream) {
    if (tokens < 1 || tokens > kMaxTokens || in_features < 1 || out_features < 1 || (bits != 4 && bits != 8))
        return BD_ERR_INVALID;
    if (!codes || !code_sums || !signs_t16 || !scale || !midpoint || !bound || !y) return BD_ERR_INVALID;
    ProjArgs a{};
    a.bits = signs_t16;
    a.rows = out_features;
    a.cols = in_features;
    a.ncp = (in_features + 255) / 256;
    a.codes0 = codes;
    a.csum0 = code_sums;
    a.nparts = 1;
    a.ld = a.ncp * 256;
    a.tokens = tokens;
    plan_proj(a, 1);
    a.scale0 = scale;
    a.mid0 = midpoint;
    a.bound = bound;
    a.code_bits = bits;
    a.residual = residual;
    a.out = y;
    a.raw_dot = raw_dot;
    if (workspace) {  // split-K accumulators; without them the launcher does not split K
        Carver c{static_cast<char *>(workspace)};
        a.acc = c.take<int32_t>(2 * ((out_features + 15) / 16 * 16) * kMaxTokens);
        a.counters = c.take<int32_t>((out_features + 15) / 16);
        if (c.off > workspace_bytes) return BD_ERR_WORKSPACE;
    }
    return launch_proj(a, EPI_HE4, stream);
}

extern "C" size_t bd_ffn_workspace_bytes(int tokens, int64_t hidden, int64_t inter) {
    (void)tokens;
    return ffn_w8_workspace_bytes(hidden, inter);
}

static bool ffn_shapes_ok(int tokens, int64_t hidden, int64_t inter) {
    return tokens >= 1 && tokens <= kMaxTokens && hidden >= 1 && inter >= 1;
}

static bool he4_args_ok(const bd_ffn_he4_args *p) {
    return p && ffn_shapes_ok(p->tokens, p->hidden, p->inter) && p->x && p->y && p->signs_gate_up && p->scale_gate &&
           p->midpoint_gate && p->scale_up && p->midpoint_up && p->scale_down && p->midpoint_down &&
           p->gain_gate_up && p->bound_gate_up && p->gain_down && p->bound_down;
}

static FfnW8 he4_block(const bd_ffn_he4_args *p) {
    FfnW8 f{};
    f.tokens = p->tokens;
    f.hidden = p->hidden;
    f.inter = p->inter;
    f.signs_gate_up = p->signs_gate_up;
    f.signs_down = p->signs_down;
    f.scale_gate = p->scale_gate;
    f.mid_gate = p->midpoint_gate;
    f.scale_up = p->scale_up;
    f.mid_up = p->midpoint_up;
    f.scale_down = p->scale_down;
    f.mid_down = p->midpoint_down;
    f.gain_gate_up = p->gain_gate_up;
    f.bound_gate_up = p->bound_gate_up;
    f.gain_down = p->gain_down;
    f.bound_down = p->bound_down;
    f.x = p->x;
    f.residual = p->residual;
    f.norm_w = p->norm_weight;
    f.eps = p->epsilon;
    f.y = p->y;
    f.hidden_out = p->hidden_out;
    f.flags = p->flags;
    f.workspace = p->workspace;
    f.workspace_bytes = p->workspace_bytes;
    return f;
}

extern "C" int bd_ffn_he4(const bd_ffn_he4_args *p, bd_stream_t stream) {
    if (!he4_args_ok(p) || !p->signs_down) return BD_ERR_INVALID;
    return ffn_w8(he4_block(p), EPI_HE4, stream);
}

extern "C" int bd_ffn_he4_fused(const bd_ffn_he4_args *p, const uint8_t *signs_down_d8, bd_stream_t stream) {
    if (!he4_args_ok(p) || !signs_down_d8) return BD_ERR_INVALID;
    return ffn_fused_he4(he4_block(p), signs_down_d8, stream);
}

static FfnW8 w1_block(const bd_ffn_w1_args *p, bd_stream_t stream) {
    (void)stream;
    FfnW8 f{};
    f.tokens = p->tokens;
    f.hidden = p->hidden;
    f.inter = p->inter;
    f.signs_gate_up = p->signs_gate_up;
    f.signs_down = p->signs_down;
    f.scale_gate = p->scale_gate;
    f.scale_up = p->scale_up;
    f.scale_down = p->scale_down;
    f.x = p->x;
    f.y = p->y;
    f.hidden_out = p->hidden_out;
    f.flags = p->flags;
    f.workspace = p->workspace;
    f.workspace_bytes = p->workspace_bytes;
    return f;
}

extern "C" int bd_ffn_w1(const bd_ffn_w1_args *p, bd_stream_t stream) {
    if (!p || !ffn_shapes_ok(p->tokens, p->hidden, p->inter)) return BD_ERR_INVALID;
    if (!p->x || !p->y || !p->signs_gate_up || !p->signs_down || !p->scale_gate || !p->scale_up ||
        !p->scale_down)
        return BD_ERR_INVALID;
    return ffn_w8(w1_block(p, stream), EPI_W1, stream);
}

// ------------------------------------------------------------------------------------ W1A1
// Sign-binarised activations (x >= 0 -> +1, per-token scale mean|x| in a fixed
// summation order) against one-bit weights; the +-1 dot K - 2 popc(x ^ w) is
// computed exactly as 2 * (codes . b01) - sum(codes) on the integer MMA pipe.
// Token counts above 32 run in 32-token chunks on the same stream.

extern "C" int bd_binarize_rows(const float *x, int64_t rows, int64_t cols, uint32_t *words, float *mean_abs,
                                int32_t *flags, bd_stream_t stream) {
    if (rows < 0 || cols < 1 || rows > 0x7fffffff) return BD_ERR_INVALID;
    if (rows == 0) return BD_OK;
    if (!x || !words || !mean_abs) return BD_ERR_INVALID;
    return launch_binarize(x, rows, cols, bd_codes_ld(cols), nullptr, nullptr, mean_abs, words, (cols + 31) / 32,
                           flags, stream);
}

struct W1a1Pieces {
    int8_t *codes;
    int32_t *sums;
    float *mean;
    int32_t *acc, *counters;
};

static W1a1Pieces carve_w1a1(void *ws, int64_t in, int64_t out, size_t *bytes) {
    Carver c{static_cast<char *>(ws)};
    W1a1Pieces p{};
    p.codes = c.take<int8_t>(kMaxTokens * bd_codes_ld(in));
    p.sums = c.take<int32_t>(kMaxTokens);
    p.mean = c.take<float>(kMaxTokens);
    p.acc = c.take<int32_t>(2 * ((out + 15) / 16 * 16) * kMaxTokens);
    p.counters = c.take<int32_t>((out + 15) / 16);
    *bytes = c.off;
    return p;
}

extern "C" size_t bd_projection_w1a1_workspace_bytes(int64_t in_features, int64_t out_features) {
    size_t bytes = 0;
    carve_w1a1(nullptr, in_features, out_features, &bytes);
    return bytes;
}

static ProjArgs w1a1_args(const uint32_t *signs, int64_t in, int64_t out, const W1a1Pieces &w, int tokens) {
    ProjArgs a{};
    a.bits = signs;
    a.rows = out;
    a.cols = in;
    a.ncp = (in + 255) / 256;
    a.codes0 = w.codes;
    a.csum0 = w.sums;
    a.nparts = 1;
    a.ld = a.ncp * 256;
    a.tokens = tokens;
    a.kgroups = 1;
    a.row_scale = w.mean;
    return a;
}

extern "C" int bd_projection_w1a1(const float *x, int tokens, int64_t in_features, int64_t out_features,
                                  const uint32_t *signs_t16, const float *scale, float *y, int32_t *raw_dot,
                                  void *workspace, size_t workspace_bytes, int32_t *flags, bd_stream_t stream) {
    if (tokens < 0 || in_features < 1 || out_features < 1) return BD_ERR_INVALID;
    if (tokens == 0) return BD_OK;
    if (!x || !signs_t16 || !scale || !y) return BD_ERR_INVALID;
    size_t need = 0;
    const W1a1Pieces w = carve_w1a1(workspace, in_features, out_features, &need);
    if (!workspace || need > workspace_bytes) return BD_ERR_WORKSPACE;
    for (int t0 = 0; t0 < tokens; t0 += kMaxTokens) {
        const int n = tokens - t0 < kMaxTokens ? tokens - t0 : kMaxTokens;
        int st = launch_binarize(x + t0 * in_features, n, in_features, bd_codes_ld(in_features), w.codes, w.sums,
                                 w.mean, nullptr, 0, flags, stream);
        if (st) return st;
        ProjArgs a = w1a1_args(signs_t16, in_features, out_features, w, n);
        a.scale0 = scale;
        a.out = y + t0 * out_features;
        a.raw_dot = raw_dot ? raw_dot + t0 * out_features : nullptr;
        a.acc = w.acc;
        a.counters = w.counters;
        a.flags = flags;
        st = launch_proj(a, EPI_W1A1, stream);
        if (st) return st;
    }
    return BD_OK;
}

extern "C" int bd_ffn_w1a1(const bd_ffn_w1_args *p, bd_stream_t stream) {
    if (!p || p->tokens < 0 || p->hidden < 1 || p->inter < 1) return BD_ERR_INVALID;
    if (p->tokens == 0) return BD_OK;
    if (!p->x || !p->y || !p->signs_gate_up || !p->signs_down || !p->scale_gate || !p->scale_up || !p->scale_down)
        return BD_ERR_INVALID;
    for (int t0 = 0; t0 < p->tokens; t0 += kMaxTokens) {
        FfnW8 f = w1_block(p, stream);
        f.tokens = p->tokens - t0 < kMaxTokens ? p->tokens - t0 : kMaxTokens;
        f.x = p->x + t0 * p->hidden;
        f.y = p->y + t0 * p->hidden;
        f.hidden_out = p->hidden_out ? p->hidden_out + t0 * p->inter : nullptr;
        const int st = ffn_w8(f, EPI_W1A1, stream);
        if (st) return st;
    }
    return BD_OK;
}
