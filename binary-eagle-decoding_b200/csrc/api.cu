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

struct FfnPieces {
    int8_t *codes_in, *codes_in_lo, *codes_mid, *codes_mid_lo;
    int32_t *sum_in, *sum_in_lo, *sum_mid, *sum_mid_lo;
    float *scale_in, *scale_mid, *hidden;
    int32_t *acc, *counters;
};

static FfnPieces carve_ffn(void *ws, int64_t hidden, int64_t inter, bool planes, size_t *bytes) {
    Carver c{static_cast<char *>(ws)};
    const int64_t ld_h = (hidden + 255) / 256 * 256, ld_f = (inter + 255) / 256 * 256;
    const int64_t rows_pad_h = (hidden + 15) / 16 * 16;
    FfnPieces p{};
    p.codes_in = c.take<int8_t>(kMaxTokens * ld_h);
    p.codes_mid = c.take<int8_t>(kMaxTokens * ld_f);
    p.sum_in = c.take<int32_t>(kMaxTokens * quant_parts(hidden));
    p.sum_mid = c.take<int32_t>(kMaxTokens);
    if (planes) {
        p.codes_in_lo = c.take<int8_t>(kMaxTokens * ld_h);
        p.codes_mid_lo = c.take<int8_t>(kMaxTokens * ld_f);
        p.sum_in_lo = c.take<int32_t>(kMaxTokens);
        p.sum_mid_lo = c.take<int32_t>(kMaxTokens);
        p.scale_in = c.take<float>(kMaxTokens);
        p.scale_mid = c.take<float>(kMaxTokens);
        p.hidden = c.take<float>(kMaxTokens * inter);
    }
    p.acc = c.take<int32_t>(2 * rows_pad_h * kMaxTokens);
    p.counters = c.take<int32_t>((hidden + 15) / 16);
    *bytes = c.off;
    return p;
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
    size_t bytes = 0;
    carve_ffn(nullptr, hidden, inter, true, &bytes);
    return bytes;
}

static bool ffn_shapes_ok(int tokens, int64_t hidden, int64_t inter) {
    return tokens >= 1 && tokens <= kMaxTokens && hidden >= 1 && inter >= 1;
}

extern "C" int bd_ffn_he4(const bd_ffn_he4_args *p, bd_stream_t stream) {
    if (!p || !ffn_shapes_ok(p->tokens, p->hidden, p->inter)) return BD_ERR_INVALID;
    if (!p->x || !p->y || !p->signs_gate_up || !p->signs_down || !p->scale_gate || !p->midpoint_gate ||
        !p->scale_up || !p->midpoint_up || !p->scale_down || !p->midpoint_down || !p->gain_gate_up ||
        !p->bound_gate_up || !p->gain_down || !p->bound_down)
        return BD_ERR_INVALID;
    size_t need = 0;
    FfnPieces w = carve_ffn(p->workspace, p->hidden, p->inter, false, &need);
    if (!p->workspace || need > p->workspace_bytes) return BD_ERR_WORKSPACE;
    const int64_t ld_h = (p->hidden + 255) / 256 * 256, ld_f = (p->inter + 255) / 256 * 256;
    // The quantizer writes per-slice partial code sums of the gate/up input and
    // zeroes the down projection's code sums, which gate/up accumulate.
    int st = launch_quantize_codes(p->x, p->tokens, p->hidden, ld_h, p->gain_gate_up, p->bound_gate_up, 4,
                                   w.codes_in, w.sum_in, true, p->flags, w.sum_mid, kMaxTokens, stream,
                                   p->norm_weight, p->epsilon);
    if (st) return st;

    ProjArgs gu{};
    gu.bits = p->signs_gate_up;
    gu.rows = p->inter;
    gu.cols = p->hidden;
    gu.ncp = ld_h / 256;
    gu.codes0 = w.codes_in;
    gu.csum0 = w.sum_in;
    gu.nparts = quant_parts(p->hidden);
    gu.ld = ld_h;
    gu.tokens = p->tokens;
    gu.kgroups = 1;
    gu.scale0 = p->scale_gate;
    gu.mid0 = p->midpoint_gate;
    gu.scale1 = p->scale_up;
    gu.mid1 = p->midpoint_up;
    gu.bound = p->bound_gate_up;
    gu.code_bits = 4;
    gu.out = p->hidden_out;
    gu.next_gain = p->gain_down;
    gu.next_bound = p->bound_down;
    gu.next_codes = w.codes_mid;
    gu.next_csum = w.sum_mid;
    gu.next_ld = ld_f;
    gu.flags = p->flags;
    st = launch_gateup(gu, EPI_HE4, stream);
    if (st) return st;

    ProjArgs dn{};
    dn.bits = p->signs_down;
    dn.rows = p->hidden;
    dn.cols = p->inter;
    dn.ncp = ld_f / 256;
    dn.codes0 = w.codes_mid;
    dn.csum0 = w.sum_mid;
    dn.nparts = 1;
    dn.ld = ld_f;
    dn.tokens = p->tokens;
    plan_proj(dn, 1);
    dn.scale0 = p->scale_down;
    dn.mid0 = p->midpoint_down;
    dn.bound = p->bound_down;
    dn.code_bits = 8;
    dn.residual = p->residual;
    dn.out = p->y;
    dn.acc = w.acc;
    dn.counters = w.counters;
    dn.flags = p->flags;
    return launch_proj(dn, EPI_HE4, stream);
}

extern "C" int bd_ffn_w1(const bd_ffn_w1_args *p, bd_stream_t stream) {
    if (!p || !ffn_shapes_ok(p->tokens, p->hidden, p->inter)) return BD_ERR_INVALID;
    if (!p->x || !p->y || !p->signs_gate_up || !p->signs_down || !p->scale_gate || !p->scale_up ||
        !p->scale_down)
        return BD_ERR_INVALID;
    size_t need = 0;
    FfnPieces w = carve_ffn(p->workspace, p->hidden, p->inter, true, &need);
    if (!p->workspace || need > p->workspace_bytes) return BD_ERR_WORKSPACE;
    const int64_t ld_h = (p->hidden + 255) / 256 * 256, ld_f = (p->inter + 255) / 256 * 256;
    int st = launch_quantize_planes(p->x, p->tokens, p->hidden, ld_h, w.codes_in, w.codes_in_lo, w.sum_in,
                                    w.sum_in_lo, w.scale_in, p->flags, stream);
    if (st) return st;
    float *hidden = p->hidden_out ? p->hidden_out : w.hidden;

    ProjArgs gu{};
    gu.bits = p->signs_gate_up;
    gu.rows = p->inter;
    gu.cols = p->hidden;
    gu.ncp = ld_h / 256;
    gu.codes0 = w.codes_in;
    gu.codes1 = w.codes_in_lo;
    gu.csum0 = w.sum_in;
    gu.csum1 = w.sum_in_lo;
    gu.nparts = 1;
    gu.ld = ld_h;
    gu.tokens = p->tokens;
    gu.kgroups = 1;
    gu.scale0 = p->scale_gate;
    gu.scale1 = p->scale_up;
    gu.row_scale = w.scale_in;
    gu.out = hidden;
    gu.flags = p->flags;
    st = launch_gateup(gu, EPI_W1, stream);
    if (st) return st;
    st = launch_quantize_planes(hidden, p->tokens, p->inter, ld_f, w.codes_mid, w.codes_mid_lo, w.sum_mid,
                                w.sum_mid_lo, w.scale_mid, p->flags, stream);
    if (st) return st;

    ProjArgs dn{};
    dn.bits = p->signs_down;
    dn.rows = p->hidden;
    dn.cols = p->inter;
    dn.ncp = ld_f / 256;
    dn.codes0 = w.codes_mid;
    dn.codes1 = w.codes_mid_lo;
    dn.csum0 = w.sum_mid;
    dn.csum1 = w.sum_mid_lo;
    dn.nparts = 1;
    dn.ld = ld_f;
    dn.tokens = p->tokens;
    plan_proj(dn, 2);
    dn.scale0 = p->scale_down;
    dn.row_scale = w.scale_mid;
    dn.out = p->y;
    dn.acc = w.acc;
    dn.counters = w.counters;
    dn.flags = p->flags;
    return launch_proj(dn, EPI_W1, stream);
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
    size_t need = 0;
    FfnPieces w = carve_ffn(p->workspace, p->hidden, p->inter, true, &need);
    if (!p->workspace || need > p->workspace_bytes) return BD_ERR_WORKSPACE;
    const int64_t ld_h = bd_codes_ld(p->hidden), ld_f = bd_codes_ld(p->inter);
    for (int t0 = 0; t0 < p->tokens; t0 += kMaxTokens) {
        const int n = p->tokens - t0 < kMaxTokens ? p->tokens - t0 : kMaxTokens;
        float *hidden = p->hidden_out ? p->hidden_out + t0 * p->inter : w.hidden;
        int st = launch_binarize(p->x + t0 * p->hidden, n, p->hidden, ld_h, w.codes_in, w.sum_in, w.scale_in,
                                 nullptr, 0, p->flags, stream);
        if (st) return st;
        W1a1Pieces in{w.codes_in, w.sum_in, w.scale_in, nullptr, nullptr};
        ProjArgs gu = w1a1_args(p->signs_gate_up, p->hidden, p->inter, in, n);
        gu.scale0 = p->scale_gate;
        gu.scale1 = p->scale_up;
        gu.out = hidden;
        gu.flags = p->flags;
        st = launch_gateup(gu, EPI_W1A1, stream);
        if (st) return st;
        st = launch_binarize(hidden, n, p->inter, ld_f, w.codes_mid, w.sum_mid, w.scale_mid, nullptr, 0, p->flags,
                             stream);
        if (st) return st;
        W1a1Pieces mid{w.codes_mid, w.sum_mid, w.scale_mid, w.acc, w.counters};
        ProjArgs dn = w1a1_args(p->signs_down, p->inter, p->hidden, mid, n);
        dn.scale0 = p->scale_down;
        dn.out = p->y + t0 * p->hidden;
        dn.acc = w.acc;
        dn.counters = w.counters;
        dn.flags = p->flags;
        st = launch_proj(dn, EPI_W1A1, stream);
        if (st) return st;
    }
    return BD_OK;
}
