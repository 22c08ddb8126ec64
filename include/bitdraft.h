/*
 * bitdraft.h -- C ABI of the B200 (sm_100a) binary-drafter hot path.
 *
 * Plain pointers and sizes only; every pointer argument is DEVICE memory unless
 * its comment says host.  Every entry point is stream-ordered on the given
 * cudaStream_t (pass 0 for the legacy default stream), returns an int status
 * (BD_OK = 0) for host-side validation and launch errors, and reports
 * data-dependent errors (non-finite inputs, invalid learned bounds) by OR-ing
 * BD_FLAG_* bits into a device int32 `flags` word that the caller reads after
 * the stream has reached the call.  The reference raises ValueError for the
 * same conditions at the same points; the Python host layer turns flags into
 * ValueError with the reference's messages.
 *
 * Each entry point cites the reference (philippesic/binary-eagle-decoding)
 * interface it replaces.
 */
#ifndef BITDRAFT_H
#define BITDRAFT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *bd_stream_t; /* == cudaStream_t */

/* ---- status codes (host return values) ---- */
#define BD_OK 0
#define BD_ERR_INVALID 1   /* bad shape, null pointer or unsupported size */
#define BD_ERR_ALIGNMENT 2 /* pointer not aligned as documented */
#define BD_ERR_LAUNCH 3    /* CUDA launch or runtime error */
#define BD_ERR_WORKSPACE 4 /* workspace too small */
#define BD_ERR_DEVICE 5    /* no usable sm_100 device */
#define BD_ERR_TOO_LARGE 6 /* size beyond a fixed scratch capacity */

/* ---- device-reported flags (OR-ed into *flags) ---- */
#define BD_FLAG_NONFINITE_LATENT 1u   /* export.py:80-81 "finite F32 sign matrix required" */
#define BD_FLAG_NONFINITE_INPUT 2u    /* model.py:130-131 "nonfinite quantizer input" */
#define BD_FLAG_BAD_BOUND 4u          /* model.py:133-134 "invalid learned clipping bound" */
#define BD_FLAG_NONFINITE_LOGITS 8u   /* verifier-trace.hpp:30 "nonfinite verifier logits" */
#define BD_FLAG_BAD_TOKEN 16u         /* a draft token outside [0, vocab) */
#define BD_FLAG_NONFINITE_STATE 32u   /* non-finite values in a forward / update */
#define BD_FLAG_CACHE_OVERFLOW 64u    /* model.py:100-101 "F16 cache storage overflow" */
#define BD_FLAG_SIGN_CHANGE 128u      /* model.py:162-163 "bounded latent scale changed a sign" */
#define BD_FLAG_TIMEOUT 256u          /* a bounded device wait ran out (the kernel returned early) */
#define BD_FLAG_NONFINITE_FEATURES 512u /* captures.py:129-130 "nonfinite teacher features" */
#define BD_FLAG_NONFINITE_LOSS 1024u    /* worker.py:360-361 "nonfinite loss" */

int bd_abi_version(void);
const char *bd_status_string(int status);
/* Number of SMs of the current device and whether it is sm_100 (host query). */
int bd_device_info(int *sm_count, int *major, int *minor);

/* ====================================================================== signs
 * bd_pack_signs replaces export.packed_signs (w1a1_eagle/numerical/export.py:79-86):
 * words[r * ceil(cols/32) + w] bit j = latent[r, 32 w + j] >= 0 (padding bits 0).
 * Sets BD_FLAG_NONFINITE_LATENT if any latent is not finite (words still written).
 */
int bd_pack_signs(const float *latent, int64_t rows, int64_t cols, int32_t *words,
                  int32_t *flags, bd_stream_t stream);

/* T16 tiled sign layout used by the decode kernels (512-byte units of 16 rows by
 * 256 columns, each lane's 16 bytes its m16n8k32 A-fragment bits).  Words:
 * bd_t16_words(rows, cols) uint32.  `block_stride`/`block_offset` interleave
 * several matrices' 16-row blocks into one buffer (stride 2, offset 0/1 puts
 * gate and up row blocks side by side); pass 1/0 for a plain matrix.  Replaces
 * the sign materialisation of hard_sign (w1a1_eagle/model.py:92-95) for the
 * forward: the packed bits ARE the signs. */
int64_t bd_t16_words(int64_t rows, int64_t cols);
int bd_tile_signs_t16(const float *latent, int64_t rows, int64_t cols, uint32_t *tiled,
                      int block_stride, int block_offset, int32_t *flags, bd_stream_t stream);
/* Same tiling from GGUF words (as written by bd_pack_signs / export_he4). */
int bd_tile_gguf_t16(const int32_t *words, int64_t rows, int64_t cols, uint32_t *tiled,
                     int block_stride, int block_offset, bd_stream_t stream);

/* W8 sign layout read by the decode feed-forward blocks (bd_ffn_*), the B
 * fragments of int8 m16n8k32 with the tokens on the M side: n-tiles of 8 rows,
 * words of 128 columns, [n-tile][word][lane] uint32 (bd_w8_words(rows, cols));
 * lane 4 g + t, bit 8 j + 2 ks + r = sign of row 8 n + g, column 128 w + 32 ks +
 * 16 r + 4 t + j (0 past the last column).  block_stride/offset interleave
 * n-tiles of several matrices (2/0 and 2/1 for gate and up). */
int64_t bd_w8_words(int64_t rows, int64_t cols);
int bd_tile_signs_w8(const float *latent, int64_t rows, int64_t cols, uint32_t *tiled,
                     int block_stride, int block_offset, int32_t *flags, bd_stream_t stream);

/* =================================================================== quantizer
 * bd_quantize_codes replaces the activation quantizer of Projection.forward
 * (w1a1_eagle/model.py:128-140): code(t, k) = clamp(rint(clip(x*gain, +-bound)
 * * (1/bound * max)), +-max) as int8, max = 2^(bits-1) - 1, stored in the F8
 * B-fragment layout: blocks of 8 rows by 64 columns, 512 bytes each, row-block
 * major; inside a block the 16 bytes of lane l = 4 (t % 8) + q hold, for the
 * two 32-column k-steps s of the block, the codes of columns 32 s + 16 h + 4 q
 * + j at byte 8 (s & 1) + 4 h + j.  ld = bd_codes_ld(cols) (a multiple of 256),
 * buffer size bd_codes_bytes(rows, cols); columns >= cols are not written.
 * code_sums[t] = exact sum of row t's codes.  gain [cols] and bound [1] are the
 * exponentiated parameters (device). */
int64_t bd_codes_bytes(int64_t rows, int64_t cols);
int bd_quantize_codes(const float *x, int64_t rows, int64_t cols, int64_t ld, const float *gain,
                      const float *bound, int bits, int8_t *codes, int32_t *code_sums,
                      int32_t *flags, bd_stream_t stream);

/* ================================================================ projections
 * One HE4 projection (w1a1_eagle/model.py:141-150, forward value):
 * y[t, o] = (D[t,o] * max(scale[o],0)) * step + (code_sums[t] * step) * midpoint[o]
 *           (+ residual[t, o] if residual != NULL), D = exact codes . signs.
 * signs: T16 [out, in]; codes from bd_quantize_codes with ld = bd_codes_ld(in).
 * tokens <= 32.  raw_dot (optional) receives the exact integer D.  The
 * workspace (bd_projection_workspace_bytes) holds split-K accumulators; zero it
 * once before first use (the kernels leave it zeroed). */
int64_t bd_codes_ld(int64_t cols);
size_t bd_projection_workspace_bytes(int tokens, int64_t out_features);
int bd_projection_he4(const int8_t *codes, const int32_t *code_sums, int tokens, int64_t in_features,
                      int64_t out_features, const uint32_t *signs_t16, const float *scale,
                      const float *midpoint, const float *bound, int bits, const float *residual,
                      float *y, int32_t *raw_dot, void *workspace, size_t workspace_bytes,
                      bd_stream_t stream);

/* ============================================================ feed-forward blocks
 * HE4 SwiGLU block, the FFN of Layer.forward / Layer.group
 * (w1a1_eagle/model.py:220-223, 271-274):
 *   y = residual + down(silu(gate(n)) * up(n)),
 * gate/up: 4-bit codes with the shared gain/bound (model.py:184-187),
 * down: 8-bit codes with its own gain/bound (model.py:188-193).
 * signs_gate_up: W8 of gate and up with n-tiles interleaved (block_stride 2,
 * offsets 0/1); signs_down: W8 [hidden, inter].  tokens <= 32.  Three kernels:
 * the quantizer (with the optional rms), gate/up + SwiGLU + the down
 * projection's quantizer, and the down projection split over K by a 4-CTA
 * cluster.  Workspace: bd_ffn_workspace_bytes. */
typedef struct {
    const float *x;          /* [tokens, hidden] normalised input n            */
    const float *residual;   /* [tokens, hidden] or NULL                        */
    float *y;                /* [tokens, hidden]                                */
    int tokens;
    int64_t hidden, inter;
    const uint32_t *signs_gate_up;
    const float *scale_gate, *midpoint_gate, *scale_up, *midpoint_up;
    const float *gain_gate_up; /* [hidden] */
    const float *bound_gate_up; /* [1] */
    const uint32_t *signs_down;
    const float *scale_down, *midpoint_down;
    const float *gain_down;  /* [inter] */
    const float *bound_down; /* [1] */
    float *hidden_out;       /* optional [tokens, inter] silu(gate)*up, or NULL */
    void *workspace;
    size_t workspace_bytes;
    int32_t *flags;
    const float *norm_weight; /* optional: x is the raw residual stream and n = rms(x, norm_weight,
                                 epsilon) is computed in the quantizer (model.py:220) */
    float epsilon;
} bd_ffn_he4_args;
size_t bd_ffn_workspace_bytes(int tokens, int64_t hidden, int64_t inter);
int bd_ffn_he4(const bd_ffn_he4_args *args, bd_stream_t stream);

/* The same HE4 block (w1a1_eagle/model.py:128-150, 220-223) in two launches
 * for tokens <= 16, hidden and inter multiples of 32.  Gate/up: clusters of
 * CTAs quantize x together (rms shared through distributed shared memory),
 * each CTA streams its gate/up W8 words into shared memory before the
 * dependency wait and writes the A8 codes of the down input.  Down (launched
 * with programmatic dependent launch, so its CTAs stream their signs from
 * signs_down_d8 while gate/up runs): clusters own output rows, their CTAs
 * split K and meet through distributed shared memory.  args->signs_down is not
 * read.  Workspace: bd_ffn_fused_workspace_bytes(hidden, inter) (no zeroing
 * needed; calls sharing one must not overlap on the GPU).
 * bd_tile_signs_d8: down signs [rows = hidden][cols = inter] as D8 bytes
 *   ((n * g4 + s / 4) * 32 + lane) * 4 + s % 4 (n = 8-row tile, s = 32-column
 *   k-step, g4 = ceil(k-steps / 4), lane = 4 g + t): bit 4 r + j is
 *   latent[8 n + g][32 s + 16 r + 4 t + j] >= 0.
 * bd_ffn_fused_shape: the launch shape chosen for these sizes on the current
 *   device, shape[4] = {gate/up cluster size, gate/up CTAs, down cluster size,
 *   down CTAs} (a diagnostic; it has no counterpart in the reference). */
int64_t bd_d8_bytes(int64_t rows, int64_t cols);
int bd_tile_signs_d8(const float *latent, int64_t rows, int64_t cols, uint8_t *tiled, int32_t *flags,
                     bd_stream_t stream);
size_t bd_ffn_fused_workspace_bytes(int64_t hidden, int64_t inter);
int bd_ffn_fused_shape(int64_t hidden, int64_t inter, int *shape);
int bd_ffn_he4_fused(const bd_ffn_he4_args *args, const uint8_t *signs_down_d8, bd_stream_t stream);

/* Pure one-bit-weight SwiGLU (fp32 activations; no reference module -- built
 * from hard_sign (model.py:92-95) and the mean|W| row scale (model.py:123)):
 *   y = sd * sign(Wd) . (silu(sg * sign(Wg) x) * (su * sign(Wu) x)).
 * Activations are carried as per-token 16-bit fixed point (two int8 planes,
 * exact integer accumulation).  tokens <= 32. */
typedef struct {
    const float *x; float *y; int tokens; int64_t hidden, inter;
    const uint32_t *signs_gate_up; const float *scale_gate, *scale_up;
    const uint32_t *signs_down; const float *scale_down;
    float *hidden_out; void *workspace; size_t workspace_bytes; int32_t *flags;
} bd_ffn_w1_args;
int bd_ffn_w1(const bd_ffn_w1_args *args, bd_stream_t stream);

/* ====================================================================== W1A1
 * Sign-binarised activations against one-bit weights.  The reference has no
 * W1A1 module; its export rule string
 * "signed_pm_bound_threshold0_nonnegative_positive_zero_row_scale0"
 * (w1a1_eagle/numerical/export.py:145) fixes the sign rule x >= 0 -> +1 and a
 * per-token scale mean|x|, summed in a fixed order (lane l of 256 adds
 * |x[l + 256 i]| sequentially, then a balanced tree of adjacent pairs).
 *
 * bd_binarize_rows: GGUF-style sign words of x (bit j of word w of row r =
 * x[r, 32w+j] >= 0, padding 0; export.py:79-86 layout) and mean|x| per row. */
int bd_binarize_rows(const float *x, int64_t rows, int64_t cols, uint32_t *words, float *mean_abs,
                     int32_t *flags, bd_stream_t stream);
/* One W1A1 projection y[t,o] = (D[t,o] * scale[o]) * mean|x_t|, with the exact
 * +-1 dot D = K - 2 popc(sign_bits(x_t) ^ sign_bits(W_o)) (raw_dot optional).
 * signs: T16 [out, in].  Any token count (32-token chunks). */
size_t bd_projection_w1a1_workspace_bytes(int64_t in_features, int64_t out_features);
int bd_projection_w1a1(const float *x, int tokens, int64_t in_features, int64_t out_features,
                       const uint32_t *signs_t16, const float *scale, float *y, int32_t *raw_dot,
                       void *workspace, size_t workspace_bytes, int32_t *flags, bd_stream_t stream);
/* W1A1 SwiGLU: every projection input is re-binarised with its own mean|x|:
 *   y = W1A1_down(silu(W1A1_gate(x)) * W1A1_up(x)).
 * Same argument block as bd_ffn_w1; workspace bd_ffn_workspace_bytes. */
int bd_ffn_w1a1(const bd_ffn_w1_args *args, bd_stream_t stream);

/* ============================================================ large-M (tensor cores)
 * Token counts in the hundreds and more run on tcgen05 (int8 operands, s32 TMEM
 * accumulators): activation codes [tokens, K] row-major int8 and an "I8" copy of
 * the signs, +-1 int8 [rows, ld] with ld = bd_i8_ld(K) (a multiple of 16 bytes)
 * and rows padded to 128 (bd_i8_bytes).  bd_tile_signs_i8 writes it from a latent
 * matrix; block_stride/offset interleave 128-row blocks of several matrices (2/0
 * and 2/1: gate and up rows of the same outputs side by side).  The dots are the
 * exact +-1 dots (no rounding anywhere).
 * bd_gemm_i8: dots[t, o] = sum_k codes[t, k] * signs[o, k] (int32).
 * bd_ffn_w1a1_large: the W1A1 SwiGLU block of bd_ffn_w1a1 at any token count
 * (x re-binarised per token, gate/up fused with silu(gate) * up, the hidden
 * re-binarised, down). */
int64_t bd_i8_ld(int64_t cols);
int64_t bd_i8_bytes(int64_t rows, int64_t cols);
int bd_tile_signs_i8(const float *latent, int64_t rows, int64_t cols, int8_t *out, int block_stride,
                     int block_offset, int32_t *flags, bd_stream_t stream);
/* Plain bf16 GEMM on the tensor cores (tcgen05 kind::f16, fp32 accumulators in
 * TMEM): c[m][n] = sum_k a[m][k] b[n][k], a and b row-major bf16 with row strides
 * lda, ldb (elements, multiples of 8, 16-byte aligned bases), c fp32 with row
 * stride ldc.  Used for the context fusion and the context K/V projections of a
 * long prefill (model.py:349-351, 382-386).  workspace: as for
 * bd_gemm_bf16_split (bd_gemm_split_workspace_bytes(m, n, k, 1); NULL runs the
 * product unsplit). */
int bd_gemm_bf16(const uint16_t *a, int64_t m, int64_t k, int64_t lda, const uint16_t *b, int64_t n, int64_t ldb,
                 float *c, int64_t ldc, void *workspace, size_t workspace_bytes, bd_stream_t stream);

int bd_gemm_i8(const int8_t *codes, int64_t tokens, int64_t k, const int8_t *signs_i8, int64_t outs,
               int32_t *dots, bd_stream_t stream);
typedef struct {
    const float *x; float *y; int64_t tokens, hidden, inter;
    const int8_t *signs_gate_up_i8;  /* gate and up interleaved by 128-row blocks */
    const float *scale_gate, *scale_up;
    const int8_t *signs_down_i8; const float *scale_down;
    float *hidden_out; void *workspace; size_t workspace_bytes; int32_t *flags;
} bd_ffn_large_args;
size_t bd_ffn_large_workspace_bytes(int64_t tokens, int64_t hidden, int64_t inter);
int bd_ffn_w1a1_large(const bd_ffn_large_args *args, bd_stream_t stream);

/* ================================================================== acceptance
 * Greedy block acceptance (benchmarks/verifier.py:92-137 core loop 107-113,
 * argmax rule w1a1_eagle/contracts.py:130-137 and native/verifier-trace.hpp:28-34):
 * logits bf16 [requests, drafts+1, vocab] (row-major, raw uint16 bits),
 * drafts int32 [requests, drafts]; eog int32 [n_eog] (sorted or not).
 * Outputs accepted[requests], next_token[requests], targets[requests*(drafts+1)]
 * (targets may be NULL).  emitted = drafts[:accepted] + [next_token].
 * The workspace (bd_accept_workspace_bytes) must be zeroed once before its
 * first use: the kernel needs its counters and argmax keys at zero on entry
 * and every call leaves them zero again. */
size_t bd_accept_workspace_bytes(int requests, int drafts);
int bd_accept_greedy(const uint16_t *logits, int requests, int drafts, int64_t vocab,
                     const int32_t *draft_tokens, const int32_t *eog, int n_eog,
                     int32_t *accepted, int32_t *next_token, int32_t *targets,
                     void *workspace, size_t workspace_bytes, int32_t *flags, bd_stream_t stream);

/* bd_accept_greedy without any device allocation.  This entry point has no
 * counterpart in the reference.  It is for callers that cannot allocate device
 * memory (e.g. a verifier embedded in a serving runtime that only hands out a
 * stream and tensor pointers and forbids cudaMalloc on its decode thread): the
 * per-request counters, the argmax keys and the target rows live in a fixed
 * file-scope device array of the library: 102,400 bytes (100 KiB) per GPU,
 * laid out as counters int32 [256], argmax keys u64 [256 x 33], target rows
 * int32 [256 x 33], held until the process exits.  Limits: requests <= 256 and
 * drafts + 1 <= 33, else BD_ERR_TOO_LARGE.  The first call on a device looks up
 * the array's device address and caches it (make that call before any stream
 * capture; do not keep using the library on a device across cudaDeviceReset,
 * which would leave the cached address stale); every call clears the counters
 * and keys it uses; all calls share the array, so calls that overlap on the GPU
 * race with each other. */
int bd_accept_greedy_noalloc(const uint16_t *logits, int requests, int drafts, int64_t vocab,
                             const int32_t *draft_tokens, const int32_t *eog, int n_eog, int32_t *accepted,
                             int32_t *next_token, int32_t *targets, int32_t *flags, bd_stream_t stream);

/* Temperature-1 speculative rejection sampling (the reference's runtime uses
 * llama.cpp's common_sampler_sample_and_accept_n_rejection, un-vendored; its
 * in-tree pins are native/verifier-test.cpp:43-80 and the EOG break of
 * benchmarks/native.py:19-38).  Deterministic contract: Philox4x32-10 uniforms
 * (key = seed, counter = (request, position, purpose, offset)); e(x) by an
 * exp2 range reduction with a degree-5 polynomial in fused multiply-adds;
 * softmax statistics per 16384-entry chunk (max, fixed-order sum) combined per
 * row; accept d_i iff u q(d_i) < p(d_i); on rejection at i sample from
 * max(0, p_i - q_i) (p_i when that is zero), after n acceptances sample the
 * bonus from p_n, by a fixed inverse-CDF search; an accepted EOG that is not
 * the last draft ends the round.  target_logits bf16 [requests][drafts+1][vocab],
 * draft_logits bf16 [requests][drafts][vocab]; vocab <= 524288; returns
 * BD_ERR_TOO_LARGE when (drafts + 1) * 40 + (2 drafts + 1) * ceil(vocab / 16384)
 * * 8 bytes exceed 160 KiB of shared memory.  Two kernels; the workspace holds
 * per-chunk statistics and partial sums and needs no clearing.  Outputs as
 * bd_accept_greedy. */
size_t bd_rejection_workspace_bytes(int requests, int drafts, int64_t vocab);
int bd_accept_rejection(const uint16_t *target_logits, const uint16_t *draft_logits, int requests, int drafts,
                        int64_t vocab, const int32_t *draft_tokens, const int32_t *eog, int n_eog,
                        unsigned long long seed, uint32_t offset, int32_t *accepted, int32_t *next_token,
                        void *workspace, size_t workspace_bytes, int32_t *flags, bd_stream_t stream);

/* Row argmax of bf16 or fp32 rows (lowest index on ties), used for drafting. */
int bd_argmax_rows_bf16(const uint16_t *logits, int64_t rows, int64_t vocab, int32_t *out,
                        int32_t *flags, bd_stream_t stream);

/* ============================================================ drafter forward
 * The dense bf16 matrices of HE4.forward (w1a1_eagle/model.py:369-396): the
 * attention projections FrozenLinear q/k/v/o (model.py:105-113, 207-219),
 * the context fusion fc (model.py:382-386) and the tied vocabulary head
 * (model.py:396), as y = W x for tokens <= 32.
 * W16: weights re-tiled once (bd_tile_w16 from fp32 or bf16 row-major).
 * X16: activations as bf16 hi/lo fragment planes (bd_pack_x16, optionally
 * rms-normalised with weight, model.py:50-51; `normed` optionally receives the
 * fp32 normalised rows).  bd_gemv_bf16 stores out[t * ld_out + o] (+ residual)
 * and/or folds each row into argmax_keys[t] (largest value, lowest row index on
 * ties; zero the keys before first use, bd_argmax_finish decodes them into token
 * ids and re-zeroes them). */
int64_t bd_w16_bytes(int64_t rows, int64_t cols);
int bd_tile_w16(const void *w, int dtype_bits, int64_t rows, int64_t cols, void *out, bd_stream_t stream);
int64_t bd_x16_bytes(int tokens, int64_t cols);
int bd_pack_x16(const float *x, int tokens, int64_t cols, int64_t ldx, const float *rms_weight, float epsilon,
                void *out, float *normed, int64_t ld_normed, int32_t *flags, bd_stream_t stream);
/* bd_pack_x16 of bf16 rows (the target model's feature rows as they arrive): the
 * same X16 bits as packing their fp32 values, without a conversion pass. */
int bd_pack_x16_bf16(const void *x, int tokens, int64_t cols, int64_t ldx, const float *rms_weight, float epsilon,
                     void *out, float *normed, int64_t ld_normed, int32_t *flags, bd_stream_t stream);
/* The optional workspace (bd_gemv_workspace_bytes) lets long-row matrices
 * split K over CTAs; partial sums are added in a fixed order, so results do not
 * depend on scheduling.  Zero it once: its first 16 KB hold per-row-group
 * counters that every call leaves zeroed, the rest is scratch, so one workspace
 * (sized for the largest need) serves calls of every shape in stream order. */
size_t bd_gemv_workspace_bytes(int tokens, int64_t rows, int64_t cols);
int bd_gemv_bf16(const void *w16, int64_t rows, int64_t cols, const void *x16, int tokens, float *out,
                 int64_t ld_out, const float *residual, unsigned long long *argmax_keys, int32_t *flags,
                 void *workspace, size_t workspace_bytes, bd_stream_t stream);
int bd_argmax_finish(unsigned long long *keys, int n, int32_t *out, bd_stream_t stream);

/* Embedding rows (HE4.forward's functional.embedding, model.py:380-381) from a
 * bf16 [vocab, hidden] table; ids outside the vocabulary set BD_FLAG_BAD_TOKEN. */
/* Teacher-feature ingestion (w1a1_eagle/numerical/captures.py:124-137): tap-major
 * captures [taps][rows][hidden] of fp16 (in_dtype_bits 16) or fp32 (32) become
 * token-major features [rows][taps * hidden] in fp16 (out_dtype 0), bf16 (1) or
 * fp32 (2); a non-finite value sets BD_FLAG_NONFINITE_FEATURES (the loader's
 * "nonfinite teacher features").  hidden % 8 == 0; both pointers 16-byte aligned. */
int bd_ingest_taps(const void *taps_src, int in_dtype_bits, int taps, int64_t rows, int64_t hidden, void *features,
                   int out_dtype, int32_t *flags, bd_stream_t stream);

/* One served draft round from host buffers: copy row_bytes of pinned host rows
 * to dev_rows and the anchor token to dev_first, launch the captured round
 * (a cudaGraphExec_t), copy `drafted` token ids back to pinned host memory and
 * wait for the stream.  row_bytes 0, a NULL host_first and drafted 0 skip the
 * copies (DraftRound.__call__ launches a graph that holds its own copies, the
 * rows' copy beside the draft's first kernels). */
int bd_round_submit(void *graph_exec, const void *host_rows, void *dev_rows, size_t row_bytes,
                    const int32_t *host_first, int32_t *dev_first, const int32_t *dev_drafted, int32_t *host_drafted,
                    int drafted, bd_stream_t stream);

int bd_embed_rows(const uint16_t *table, int64_t vocab, int64_t hidden, const int32_t *ids, int n,
                  float *out, int32_t *flags, bd_stream_t stream);
/* rms(x, weight, eps) rows (model.py:50-51). */
int bd_rms_rows(const float *x, int n, int64_t cols, int64_t ldx, const float *weight, float epsilon,
                float *out, int64_t ldo, bd_stream_t stream);
/* Per-head post-processing of projected q/k/v rows: optional rms over each head
 * with norm_weight (Layer.context / Layer.forward, model.py:197-211), optional
 * rotary embedding at positions pos0 + row (model.py:54-63), fp16 storage with
 * the cache_storage overflow check (model.py:98-102, BD_FLAG_CACHE_OVERFLOW). */
int bd_heads_post(const float *src, int n, int64_t ld_src, int64_t col0, int heads, int head_dim,
                  const float *norm_weight, float epsilon, int rope, float theta, int64_t pos0,
                  uint16_t *dst_f16, int64_t dst_ld, int32_t *flags, bd_stream_t stream);
/* The same for a whole q|k|v row block in one launch (Layer.forward,
 * model.py:207-213): q heads -> fp32 q_out [n][q_ld] (normalised and rotated,
 * not rounded: the reference attends with fp32 queries), k heads -> K cache
 * rows pos0.., v heads -> V cache rows pos0.. (fp16, row stride kv_ld elements). */
int bd_qkv_post(const float *src, int n, int64_t ld_src, int heads, int kv_heads, int head_dim,
                const float *q_norm, const float *k_norm, float epsilon, float theta, int64_t pos0,
                float *q_out, int64_t q_ld, uint16_t *k_cache_f16, uint16_t *v_cache_f16, int64_t kv_ld,
                int32_t *flags, bd_stream_t stream);

/* Context k|v rows of `layers` layers in one launch (Layer.context,
 * model.py:195-200, for every layer of an ingest step): layer l's k|v block
 * (k heads then v heads) starts at column l * layer_cols of src, its k norm
 * weights at k_norms + l * head_dim, and its cache rows pos0.. at
 * k_cache/v_cache + l * cache_layer_stride elements (row stride kv_ld). */
int bd_context_kv_post(const float *src, int n, int64_t ld_src, int layers, int64_t layer_cols, int kv_heads,
                       int head_dim, const float *k_norms, float epsilon, float theta, int64_t pos0,
                       uint16_t *k_cache_f16, uint16_t *v_cache_f16, int64_t kv_ld, int64_t cache_layer_stride,
                       int32_t *flags, bd_stream_t stream);

/* Block-draft attention of Layer.forward (w1a1_eagle/model.py:212-218) over the
 * fp16 K/V cache: out[t][h * d + j] = softmax_k(q_t,h . k_k / sqrt(d)) v_k,j
 * with q head h reading kv head h / (heads / kv_heads), keys 0 .. keys-1 at
 * positions equal to their index, query row t at position anchor + t, and, if
 * `windowed`, only keys with |anchor + t - k| < window (all but the last layer,
 * model.py:390-392).  q fp32 [tokens][heads][d], caches fp16
 * [positions][kv_heads][d]; tokens <= 16, head_dim 64 or 128, heads/kv_heads <= 4.
 * The products keep fp32 precision: q and the probabilities enter the fp16
 * tensor-core MMAs as hi + lo halves.
 * stable_keys: the caller's promise that cache rows [0, stable_keys) were not
 * written by the kernel launched immediately before this call on the stream
 * (they are then read before the launch waits for it; pass 0 when unsure). */
size_t bd_attention_workspace_bytes(int heads, int head_dim, int keys);
/* The same attention writing its output rows straight into the X16 activation
 * layout of bd_pack_x16 (unnormalised, tokens rows of heads * head_dim columns)
 * for the output-projection GEMV, instead of fp32 rows; a non-finite output sets
 * BD_FLAG_NONFINITE_STATE in flags (may be NULL). */
int bd_attention_decode_x16(const float *q, const uint16_t *k_cache, const uint16_t *v_cache, int tokens, int heads,
                            int kv_heads, int head_dim, int keys, int windowed, int64_t anchor, int64_t window,
                            int64_t stable_keys, void *x16, int32_t *flags, void *workspace, size_t workspace_bytes,
                            bd_stream_t stream);
int bd_attention_decode(const float *q, const uint16_t *k_cache, const uint16_t *v_cache, int tokens, int heads,
                        int kv_heads, int head_dim, int keys, int windowed, int64_t anchor, int64_t window,
                        int64_t stable_keys, float *out, void *workspace, size_t workspace_bytes,
                        bd_stream_t stream);

/* ================================================================ row-wise chains (training)
 * bd_rms_forward: out = x * rsqrt(mean(x^2) + eps) * w over rows of cols
 *   (w1a1_eagle/model.py:50-51, torch's rms expression in one kernel), inv[r]
 *   the row's rsqrt factor for the backward.
 * bd_rms_backward: dx and dw; dw_partials is scratch of bd_rms_partials(rows,
 *   cols) floats (per-row sums, and partial rows of dw added in a fixed order).
 * bd_head_post: per (row, head) of head_dim values of x [rows][ld_x] (heads side
 *   by side): the head rms with weight (NULL: none), the rotate-half rotary at
 *   positions[row] with frequencies[head_dim / 2] (NULL: none; model.py:54-63),
 *   and with fp16 != 0 the fp16 storage rounding of cache_storage
 *   (model.py:98-102; BD_FLAG_CACHE_OVERFLOW on overflow) -> out
 *   [rows][heads][head_dim]; inv [rows][heads] the rms factors.  Products and
 *   sums round as the reference's separate tensor operations do.
 * bd_head_post_backward: dx [rows][ld_x] (the fp16 rounding passes the gradient
 *   straight through) and dw (bd_head_post_partials(rows, heads) x head_dim
 *   partials).  No reference C counterpart: the reference is torch autograd. */
int bd_rms_forward(const float *x, int64_t rows, int64_t cols, const float *weight, float eps, float *out, float *inv,
                bd_stream_t stream);
int64_t bd_rms_partials(int64_t rows, int64_t cols);
int bd_rms_backward(const float *x, int64_t rows, int64_t cols, const float *weight, const float *inv,
                         const float *dy, float *dx, float *dw_partials, float *dw, bd_stream_t stream);
int bd_head_post(const float *x, int64_t ld_x, int64_t rows, int heads, int head_dim, const float *weight, float eps,
                 const int64_t *positions, const float *frequencies, int fp16, float *out, float *inv,
                 int32_t *flags, bd_stream_t stream);
int64_t bd_head_post_partials(int64_t rows, int heads);
int bd_head_post_backward(const float *x, int64_t ld_x, int64_t rows, int heads, int head_dim, const float *weight,
                          const float *inv, const int64_t *positions, const float *frequencies, const float *dy,
                          float *dx, float *dw_partials, float *dw, bd_stream_t stream);

/* ================================================================ training attention
 * Layer.group's block attention at training sizes (w1a1_eagle/model.py:225-270,
 * the reference's torch einsum / masked_fill / softmax over [W, heads, k, L + k]
 * scores): W windows of k <= 16 slots; groups = heads / kv_heads <= 4 query heads
 * per kv head; head_dim <= 128; keys = L shared context keys.  Each slot attends
 * to the context keys its ctx_mask row allows and to the slots its slot_mask row
 * allows, one softmax over both.
 * Operands are fp16 rows of DP = head_dim rounded up to 16, 32, 64 or 128 (zero
 * padded), 16-byte aligned:
 *   q_hi, q_lo       [kv_heads][W][groups][16][DP]  fp32 query = hi + lo (rows >= k zero)
 *   ctx_k, ctx_v     [kv_heads][Lp][DP]             Lp = keys rounded up to 64 (fp16 values)
 *   slot_k, slot_v   [kv_heads][W][16][DP]
 *   ctx_mask         [W][16][Lp] uint8 (0 = masked; padding 0), slot_mask [16][16] uint8
 * scale = 1 / sqrt(head_dim).  Forward: out fp32 [W][k][kv_heads][groups][head_dim],
 * lse fp32 [kv_heads][W][groups][16] (the rows' log-sum-exp, +inf for a row with no
 * allowed key).  Backward: dout_hi/lo = the output gradient times a power of two
 * (1 / *unscale) in the q layout; dr [kv_heads][W][groups][16] = rowsum(scaled dout
 * x out); writes dq (out's layout), d_ctx_k/v fp32 [keys][kv_heads][head_dim] and
 * d_slot_k/v fp32 [W][k][kv_heads][head_dim].  tile_live [W][Lp / 64 + 1] (may be
 * NULL): the forward records which key tiles each window sees at all, and the
 * backward then skips the unseen (window, key tile) pairs of the context before
 * staging them.  kv_partials: 8 x keys x kv_heads x head_dim floats of workspace
 * (the context dK, dV of each of the 4 window shares of a key tile, added in
 * order).  fp16 tensor-core products with
 * fp32 accumulation; the fp32 operands enter as hi + lo halves.  Deterministic
 * (no atomics).  No reference C counterpart: the reference is torch autograd. */
/* The operands of the two entries above made on the device from the model's
 * tensors: query fp32 [W][k][kv_heads][groups][head_dim], ctx_k/v fp32
 * [keys][kv_heads][head_dim], slot_k/v fp32 [W][k][kv_heads][head_dim] (fp16
 * values), ctx_allowed bytes addressed with element strides (w, s, l: 0
 * broadcasts) and slot_allowed likewise (NULL: all allowed) -> q_hi/q_lo,
 * kc/vc, ks/vs, ctx_mask, slot_mask in the layouts above (zero padded) and lse
 * set to +inf.  bd_train_attention_pack_grad: dout (out's layout) times the
 * power of two 2^-ceil(log2 max|dout|) as hi + lo rows, dr = rowsum(scaled
 * dout x out); scalars[4] (fp32 workspace): [1] the factor, [2] its inverse
 * (the backward's unscale). */
int bd_train_attention_pack(const float *query, const float *ctx_k, const float *ctx_v, const float *slot_k,
                            const float *slot_v, const uint8_t *ctx_allowed, int64_t allowed_stride_w,
                            int64_t allowed_stride_s, int64_t allowed_stride_l, const uint8_t *slot_allowed,
                            int64_t slot_stride_s, int64_t slot_stride_t, int windows, int slots, int kv_heads,
                            int groups, int head_dim, int keys, void *q_hi, void *q_lo, void *kc, void *vc, void *ks,
                            void *vs, uint8_t *ctx_mask, uint8_t *slot_mask, float *lse, bd_stream_t stream);
int bd_train_attention_pack_grad(const float *dout, const float *out, int windows, int slots, int kv_heads, int groups,
                                 int head_dim, void *d_hi, void *d_lo, float *dr, float *scalars, bd_stream_t stream);
int bd_train_attention_forward(const void *q_hi, const void *q_lo, const void *ctx_k, const void *ctx_v,
                               const void *slot_k, const void *slot_v, const uint8_t *ctx_mask,
                               const uint8_t *slot_mask, int windows, int slots, int kv_heads, int groups,
                               int head_dim, int keys, float scale, float *out, float *lse, uint8_t *tile_live,
                               bd_stream_t stream);
int bd_train_attention_backward(const void *q_hi, const void *q_lo, const void *ctx_k, const void *ctx_v,
                                const void *slot_k, const void *slot_v, const uint8_t *ctx_mask,
                                const uint8_t *slot_mask, const void *dout_hi, const void *dout_lo, const float *lse,
                                const float *dr, const float *unscale, const uint8_t *tile_live, int windows,
                                int slots, int kv_heads, int groups, int head_dim, int keys, float scale, float *dq,
                                float *d_ctx_k, float *d_ctx_v, float *d_slot_k, float *d_slot_v, float *kv_partials,
                                bd_stream_t stream);

/* ================================================================ QAT (training sizes)
 * Projection.forward at any token count (w1a1_eagle/model.py:128-150): codes and
 * +-1 signs are exact in bf16, so D = codes . signs^T is an exact bf16
 * tensor-core GEMM with fp32 output (issued by the caller's GEMM, e.g. cuBLAS);
 * these kernels produce its operands and apply the epilogue.
 * bd_quantize_rows_bf16: codes bf16 [rows, cols] row-major and exact row sums
 *   (model.py:128-139; gain and bound already exponentiated).
 * bd_sign_rows: hard_sign (model.py:66-68, 92-95) of n latents as bf16 and/or
 *   fp32 +-1 (x >= 0 -> +1).
 * bd_he4_epilogue: y = (D * max(scale,0)) * step + (sums * step) * midpoint
 *   (+ residual), D fp32 [tokens, out] holding exact integers. */
int bd_quantize_rows_bf16(const float *x, int64_t rows, int64_t cols, const float *gain, const float *bound,
                          int bits, uint16_t *codes, int32_t *code_sums, int32_t *flags, bd_stream_t stream);
int bd_sign_rows(const float *latent, int64_t n, uint16_t *signs_bf16, float *signs_f32, int32_t *flags,
                 bd_stream_t stream);
int bd_he4_epilogue(const float *dot, int64_t tokens, int64_t out_features, const float *scale,
                    const float *midpoint, const float *bound, int bits, const int32_t *code_sums,
                    const float *residual, float *y, bd_stream_t stream);

/* Straight-through backward of one projection (autograd of model.py:128-150
 * with SIGN's backward, model.py:71-73).  With G = dLoss/dy [tokens, out]:
 * bd_ste_grad_prep: dL = G * max(scale,0) split into bf16 hi + lo [tokens, out];
 *   d_scale[o] = sum_t G (D step) * (scale >= 0); d_midpoint[o] = sum_t G (sums step);
 *   gm[t] = sum_o G midpoint[o].  The caller then forms d_values = dL . signs
 *   (hi and lo GEMMs, fp32) and d_signs = dL^T . codes.
 * bd_ste_input_backward: the quantizer's backward (clip ties split 0.5/0.5):
 *   dx [tokens, in], d_log_gain[in] and d_log_clip (scalar; both added to the
 *   existing values when accumulate != 0, as for gate and up sharing them).
 * bd_ste_sign_backward: out = ((grad + grad2) * step) * 1[|latent| <= window]
 *   (step = bound / max when bound != NULL, else 1), with per-block sums of
 *   squares (bd_ste_sumsq_count(n) of them) for the gradient-norm clip.
 * Workspace: bd_ste_workspace_bytes(tokens, out, in).  Reductions are in a fixed
 * order, so results are deterministic. */
size_t bd_ste_workspace_bytes(int64_t tokens, int64_t out_features, int64_t in_features);
int bd_ste_grad_prep(const float *grad, const float *dot, int64_t tokens, int64_t out_features, const float *scale,
                     const float *midpoint, const float *bound, int bits, const int32_t *code_sums,
                     uint16_t *dl_hi, uint16_t *dl_lo, int64_t ld_dl, uint16_t *dl_t_hi, uint16_t *dl_t_lo,
                     int64_t ld_t, float *d_scale, float *d_midpoint, float *gm,
                     void *workspace, size_t workspace_bytes, bd_stream_t stream);
int bd_ste_input_backward(const float *d_values, const float *d_values2, const float *gm, const float *x,
                          int64_t tokens, int64_t in_features, const float *gain, const float *bound, int bits,
                          float *dx, float *d_log_gain, float *d_log_clip, int accumulate, void *workspace,
                          size_t workspace_bytes, bd_stream_t stream);
int bd_ste_sumsq_count(int64_t n);
int bd_ste_sign_backward(const float *grad, const float *grad2, const float *latent, int64_t n, float window,
                         const float *bound, int bits, float *out, float *sumsq_partials, bd_stream_t stream);

/* The same projection and backward with every product on the 5th-generation
 * tensor cores (tcgen05, TMEM accumulators, TMA-loaded operands), replacing
 * the dense fp32 GEMMs autograd runs for Projection.forward
 * (w1a1_eagle/model.py:141-150) and its backward with SIGN (model.py:71-73):
 * bd_quantize_rows_i8: int8 codes [rows][ld] (ld >= cols, a multiple of 16)
 *   and exact row sums (model.py:128-139).
 * bd_projection_he4_tc: y = HE4 epilogue of D = codes . signs^T (kind::i8, exact
 *   s32), signs as bd_tile_signs_i8; optionally D itself (fp32, exact) in dot.
 * bd_sign_cols_bf16 / bd_codes_transpose_bf16: the +-1 signs [in][ld_t] and the
 *   codes [in][ld_t] (ld_t >= rows, a multiple of 8) as K-major bf16 operands.
 * bd_gemm_bf16_split: c = (a_hi + a_lo) . b^T in fp32 (kind::f16; the two
 *   halves of a are one reduction of twice the length): d_values = dL . signs.
 * bd_ste_weight_grad: d_latent[o][i] = ((dL^T . codes)[o][i] * step) *
 *   1[|latent[o][i]| <= window] (window = *window when window != NULL, else
 *   window_value), dL^T given as bf16 halves [out][ld_t] (bd_ste_grad_prep's
 *   transposed outputs), codes^T as bf16 [in][ld_t].  The clip mask, the step
 *   scale and two sums (of d_latent^2, and of the unmasked gradient times
 *   sign(latent) where |latent| > window: the gradient of a learned window)
 *   are in the GEMM's epilogue; the sums come per (tile, epilogue warp) in
 *   partials [bd_ste_weight_grad_partials(out, in)] as (sum, sum) pairs. */
int bd_quantize_rows_i8(const float *x, int64_t rows, int64_t cols, const float *gain, const float *bound,
                        int bits, int8_t *codes, int64_t ld, int32_t *code_sums, int32_t *flags,
                        bd_stream_t stream);
int bd_projection_he4_tc(const int8_t *codes, int64_t ld_codes, const int32_t *code_sums, int64_t tokens,
                         int64_t in_features, const int8_t *signs_i8, int64_t out_features, const float *scale,
                         const float *midpoint, const float *bound, int bits, const float *residual, float *y,
                         float *dot, int32_t *flags, bd_stream_t stream);
int bd_sign_cols_bf16(const float *latent, int64_t rows, int64_t cols, uint16_t *out, int64_t ld_t, int32_t *flags,
                      bd_stream_t stream);
int bd_codes_transpose_bf16(const int8_t *codes, int64_t rows, int64_t cols, int64_t ld, uint16_t *out,
                            int64_t ld_t, bd_stream_t stream);
int bd_gemm_bf16_split(const uint16_t *a_hi, const uint16_t *a_lo, int64_t m, int64_t k, int64_t lda,
                       const uint16_t *b, int64_t n, int64_t ldb, float *c, int64_t ldc, void *workspace,
                       size_t workspace_bytes, bd_stream_t stream);
/* Split-K workspace of bd_gemm_bf16 / bd_gemm_bf16_split / bd_gemm_bf16_split3
 * (parts = 1, 2 or 3 operand pairs) for an m x n x k product: when the 128 x 256
 * output tiles are fewer than the SMs, the K reduction is cut into slices on
 * more CTAs (slice count from the waves of (tile, slice) units, at most 8), each
 * slice writing an fp32 partial tile, and the last slice of a tile to finish
 * adds them in slice order (deterministic).  0 = no split for this shape.  The workspace (256-byte aligned) must be zero when first used; the
 * calls leave its counters zero.  Calls sharing one workspace must be ordered
 * (one stream); a NULL or smaller workspace runs the product unsplit. */
size_t bd_gemm_split_workspace_bytes(int64_t m, int64_t n, int64_t k, int parts);

/* fp32-accurate products of frozen fp32 operands on the bf16 tensor cores, for
 * FrozenLinear (w1a1_eagle/model.py:105-113) and the tied vocabulary head
 * forward and input gradient: each fp32 operand is split into bf16 halves
 * hi + lo (bd_split_bf16, optionally transposed to K-major), and
 * bd_gemm_bf16_split3 computes c = a_hi b_hi^T + a_lo b_hi^T + a_hi b_lo^T in
 * fp32 (lo x lo is left out: about 2^-16 relative per product; b_lo NULL for a
 * bf16-exact b) as one tcgen05 reduction of two or three times K. */
int bd_split_bf16(const float *x, int64_t rows, int64_t cols, int64_t ldx, int transpose, uint16_t *hi, uint16_t *lo,
                  int64_t ld, bd_stream_t stream);

/* The loss head of TensorWorker.group_loss (w1a1_eagle/numerical/worker.py:315-363):
 * loss = sum_r w[r] * (logsumexp_v(h[r] . vocab[v]) - h[r] . vocab[labels[r]]),
 * with h and the frozen vocabulary as bf16 halves (hi, lo; v_lo NULL for a
 * bf16-exact vocabulary), the products on tcgen05 at fp32 accuracy, and the
 * logits never written to memory:
 * bd_loss_head_forward: per-row softmax statistics in the GEMM's epilogue
 *   (stats: bd_loss_head_stats_count(rows, vocab) floats), then lse[r],
 *   loss_rows[r] = w[r] (lse - target logit) and their fixed-order sum *loss;
 *   BD_FLAG_NONFINITE_LOSS for a non-finite row loss ("nonfinite loss").
 * bd_loss_head_grad: the logits recomputed into dLoss/dlogits = w (softmax -
 *   onehot) in place, as bf16 halves [rows][ld_dl]; dLoss/dh is then
 *   bd_gemm_bf16_split3 of those halves with the transposed vocabulary halves. */
int64_t bd_loss_head_stats_count(int64_t rows, int64_t vocab);
int bd_loss_head_forward(const uint16_t *h_hi, const uint16_t *h_lo, int64_t rows, int64_t hidden, int64_t ld_h,
                         const uint16_t *v_hi, const uint16_t *v_lo, int64_t vocab, const int32_t *labels,
                         const float *weights, float *stats, float *target, float *lse, float *loss_rows, float *loss,
                         int32_t *flags, bd_stream_t stream);
int bd_loss_head_grad(const uint16_t *h_hi, const uint16_t *h_lo, int64_t rows, int64_t hidden, int64_t ld_h,
                      const uint16_t *v_hi, const uint16_t *v_lo, int64_t vocab, const int32_t *labels,
                      const float *weights, const float *lse, uint16_t *dl_hi, uint16_t *dl_lo, int64_t ld_dl,
                      bd_stream_t stream);
int bd_gemm_bf16_split3(const uint16_t *a_hi, const uint16_t *a_lo, int64_t m, int64_t k, int64_t lda,
                        const uint16_t *b_hi, const uint16_t *b_lo, int64_t n, int64_t ldb, float *c, int64_t ldc,
                        void *workspace, size_t workspace_bytes, bd_stream_t stream);
int64_t bd_ste_weight_grad_partials(int64_t out_features, int64_t in_features);
int bd_ste_weight_grad(const uint16_t *grad_t_hi, const uint16_t *grad_t_lo, int64_t out_features, int64_t tokens,
                       int64_t ld_t, const uint16_t *codes_t, int64_t in_features, const float *latent,
                       const float *window, float window_value, const float *bound, int bits, float *d_latent,
                       float *partials, int32_t *flags, bd_stream_t stream);

/* The update (w1a1_eagle/numerical/worker.py:365-392): clip_grad_norm_(1.0),
 * AdamW(weight_decay=0, fused=True) per parameter group, scale.clamp_(min=0),
 * optional clamp_latents (model.py:167-169).
 * bd_sum_squares / bd_grad_norm: fixed-order sum of squares partials, then
 *   total = sqrt(sum), clip_coef = min(1, max_norm / (total + 1e-6)).
 * bd_adamw_latent: AdamW of a latent matrix [rows, cols] fused with the clamp and
 *   the re-pack of its signs into W8 words (block_stride/offset as
 *   bd_tile_signs_w8; signs_w8 may be NULL).  bd_adamw: element AdamW with a
 *   lower clamp (-INFINITY for none).  clip_coef (device scalar) may be NULL.
 * bd_bound_latents: out = clamp(latent / (multiple mean|row|), -1, 1)
 *   (model.py:153-164); BD_FLAG_SIGN_CHANGE if a sign would change.
 * bd_clamp: x = min(max(x, lo), hi). */
int bd_sum_squares_count(int64_t n);
int bd_sum_squares(const float *x, int64_t n, float *partials, bd_stream_t stream);
int bd_grad_norm(const float *partials, int64_t count, float max_norm, float *total_norm, float *clip_coef,
                 int32_t *flags, bd_stream_t stream);
int bd_adamw_latent(float *param, const float *grad, float *exp_avg, float *exp_avg_sq, int64_t rows, int64_t cols,
                    double lr, double beta1, double beta2, double eps, long long step, const float *clip_coef,
                    int clamp_latents, uint32_t *signs_w8, int block_stride, int block_offset, int32_t *flags,
                    bd_stream_t stream);
int bd_adamw(float *param, const float *grad, float *exp_avg, float *exp_avg_sq, int64_t n, double lr, double beta1,
             double beta2, double eps, long long step, const float *clip_coef, float lower, int32_t *flags,
             bd_stream_t stream);
int bd_bound_latents(const float *latent, int64_t rows, int64_t cols, float multiple, float *out, int32_t *flags,
                     bd_stream_t stream);
int bd_clamp(float *x, int64_t n, float lo, float hi, bd_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* BITDRAFT_H */
