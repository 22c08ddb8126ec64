// Shared device helpers of the bitdraft sm_100a library.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "bitdraft.h"

#define BD_CHECK_LAUNCH()                                   \
    do {                                                    \
        cudaError_t e_ = cudaGetLastError();                \
        if (e_ != cudaSuccess) return BD_ERR_LAUNCH;        \
    } while (0)

namespace bd {

__device__ __forceinline__ void set_flag(int32_t *flags, uint32_t bit) {
    if (flags) atomicOr(reinterpret_cast<unsigned int *>(flags), bit);
}

__device__ __forceinline__ bool finite(float v) { return isfinite(v); }

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) {
    return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

// Integer MMA m16n8k32: D(int32) += A(16x32 s8, row) * B(32x8 s8, col).
// The MMA and weight-load helpers are not volatile: they touch only registers (or
// read-only weights), so the compiler may interleave them freely; data written by
// an earlier kernel is read with ordinary loads, which stay after grid_wait().
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// bf16 MMA m16n8k16: D(f32) += A(16x16 bf16, row) * B(16x8 bf16, col).
__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- fp16 tensor-core fragments: ldmatrix from shared memory and m16n8k16
__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void *p) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void *p) {
    const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(a));
}
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// fp16 hi + lo halves of a pair: x ~= float(hi) + float(lo) to ~22 bits.
__device__ __forceinline__ void split_half2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(x0, x1);
    const __half2 l = __floats2half2_rn(x0 - __low2float(h), x1 - __high2float(h));
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

// Streaming 16-byte global load that does not allocate in L1 (weights are read once).
__device__ __forceinline__ uint4 ld_stream_u4(const void *p) {
    uint4 v;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// 16-byte asynchronous global->shared copy; src_bytes 0 writes zeros.
__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, int src_bytes) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;\n" ::: "memory");
}

// Programmatic dependent launch: a kernel launched with the PDL attribute may
// start while its predecessor finishes; before grid_wait() it may only read
// data no earlier kernel writes (weights), and it must not write anything.
__device__ __forceinline__ void grid_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n"); }

// ---- mbarriers and 1-D bulk copies (global memory -> this CTA's own shared memory)
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
// Makes initialised mbarriers visible to the async proxy (bulk copies).
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
                 : "=r"(ok)
                 : "r"(smem_u32(b)), "r"(parity)
                 : "memory");
    return ok != 0;
}
// Bounded wait for phase `parity` of an mbarrier: false after `polls` failed polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *b, uint32_t parity, uint32_t polls) {
    for (uint32_t i = 0; i < polls; ++i)
        if (mbar_try_wait(b, parity)) return true;
    return false;
}
// Orders this thread's earlier generic-proxy shared-memory accesses before later bulk copies.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// `bytes` (a multiple of 16) from 16-byte aligned global `src` into 16-byte aligned
// shared `dst`; completion is signalled on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// B-fragment layout of int8 activation codes ("F8"): blocks of 8 tokens by 64
// columns (a pair of 32-column k-steps), 512 bytes each, nt-major; inside a
// block, lane l = 4 g + t (token 8 nt + g) holds 16 bytes: for k-step s of the
// pair, bytes 8 (s & 1) + 4 h + j are the codes of column 32 s + 16 h + 4 t + j.
// nsp = row stride in column pairs (ld / 64).
__device__ __forceinline__ int64_t frag_offset(int token, int64_t k, int64_t nsp) {
    const int64_t nt = token >> 3;
    const int g = token & 7;
    const int64_t s = k >> 5;
    const int kk = static_cast<int>(k & 31);
    const int half = kk >> 4, t = (kk & 15) >> 2, j = kk & 3;
    return (((nt * nsp + (s >> 1)) * 32 + g * 4 + t) << 4) + ((s & 1) << 3) + (half << 2) + j;
}

// A-fragment layout of int8 activation codes ("C16"), tokens as the M side of
// m16n8k32: [k-step s = k / 32][m-tile][lane][16 bytes]; lane 4 (r % 8) + (kk % 16) / 4
// of m-tile token block holds register (r / 8) + 2 (kk / 16), byte kk % 4, for
// token 16 m + r and column 32 s + kk.  One 16-byte load per lane per k-step is
// the whole A fragment.
__device__ __forceinline__ int64_t c16_offset(int token, int64_t k, int mtiles) {
    const int64_t s = k >> 5;
    const int kk = static_cast<int>(k & 31);
    const int r = token & 15, m = token >> 4;
    const int lane = ((r & 7) << 2) + ((kk & 15) >> 2);
    const int reg = (r >> 3) + ((kk >> 4) << 1);
    return (((s * mtiles + m) * 32 + lane) << 4) + (reg << 2) + (kk & 3);
}

// Byte offset of code (token, k): C16 when c16_mt > 0, row-major int8 with row
// stride ld when c16_mt < 0 (the tensor-core path), else F8 with row stride ld.
__device__ __forceinline__ int64_t code_offset(int token, int64_t k, int64_t ld, int c16_mt) {
    if (c16_mt < 0) return static_cast<int64_t>(token) * ld + k;
    return c16_mt > 0 ? c16_offset(token, k, c16_mt) : frag_offset(token, k, ld / 64);
}

// The quantizer of Projection.forward for one element (see bd_quantize_codes).
struct Quant {
    float bound, ratio, step, maximum;
    __device__ __forceinline__ void init(float b, int bits) {
        maximum = static_cast<float>((1 << (bits - 1)) - 1);
        bound = b;
        ratio = __fmul_rn(__frcp_rn(b), maximum);
        step = __fdiv_rn(b, maximum);
    }
    __device__ __forceinline__ int code(float gained) const {
        float clipped = fmaxf(fminf(gained, bound), -bound);
        float normalized = __fmul_rn(clipped, ratio);
        float r = rintf(normalized);
        r = fminf(fmaxf(r, -maximum), maximum);
        return static_cast<int>(r);
    }
};

__device__ __forceinline__ bool bad_bound(float b) { return !(isfinite(b) && b > 0.0f); }

// HE4 projection epilogue: (D * max(scale,0)) * step + (sum * step) * midpoint, op by op.
__device__ __forceinline__ float he4_value(int dot, float scale, float step, int code_sum, float midpoint) {
    float s = scale < 0.0f ? 0.0f : scale;  // clamp_min(scale, 0), NaN propagates
    float a = __fmul_rn(__fmul_rn(static_cast<float>(dot), s), step);
    float b = __fmul_rn(__fmul_rn(static_cast<float>(code_sum), step), midpoint);
    return __fadd_rn(a, b);
}

// x * sigmoid(x) through the fast exponential and a reciprocal (a few ulp from the exact value)
__device__ __forceinline__ float silu(float x) { return __fmul_rn(x, __frcp_rn(__fadd_rn(1.0f, __expf(-x)))); }

}  // namespace bd
