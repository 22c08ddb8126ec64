"""ctypes binding of ``libbitdraft.so`` (the C ABI declared in ``include/bitdraft.h``).

The library is the product: there is no CPU fallback.  If it is missing the
first call raises ``RuntimeError`` naming the build step.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "libbitdraft.so"
HEADER = HERE.parent / "include" / "bitdraft.h"

c_int, c_int64, c_size_t, c_void_p = ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p
P = c_void_p  # every device pointer travels as a plain address

BD_OK = 0
FLAG_NONFINITE_LATENT = 1
FLAG_NONFINITE_INPUT = 2
FLAG_BAD_BOUND = 4
FLAG_NONFINITE_LOGITS = 8
FLAG_BAD_TOKEN = 16
FLAG_NONFINITE_STATE = 32
FLAG_CACHE_OVERFLOW = 64
FLAG_SIGN_CHANGE = 128
FLAG_TIMEOUT = 256
FLAG_NONFINITE_FEATURES = 512
FLAG_NONFINITE_LOSS = 1024

# Messages of the reference's ValueErrors for the same conditions.
FLAG_MESSAGES = (
    (FLAG_NONFINITE_LATENT, "finite F32 sign matrix required"),
    (FLAG_NONFINITE_INPUT, "nonfinite quantizer input"),
    (FLAG_BAD_BOUND, "invalid learned clipping bound"),
    (FLAG_NONFINITE_LOGITS, "nonfinite verifier logits"),
    (FLAG_BAD_TOKEN, "draft token outside the vocabulary"),
    (FLAG_NONFINITE_STATE, "nonfinite drafter state"),
    (FLAG_CACHE_OVERFLOW, "F16 cache storage overflow"),
    (FLAG_SIGN_CHANGE, "bounded latent scale changed a sign"),
    (FLAG_NONFINITE_FEATURES, "nonfinite teacher features"),
    (FLAG_NONFINITE_LOSS, "nonfinite loss"),
)
# Device-side failures that are not the reference's ValueErrors.
FLAG_ERRORS = ((FLAG_TIMEOUT, "a bounded device wait timed out"),)


class FfnHe4Args(ctypes.Structure):
    _fields_ = [
        ("x", P), ("residual", P), ("y", P), ("tokens", c_int), ("hidden", c_int64), ("inter", c_int64),
        ("signs_gate_up", P), ("scale_gate", P), ("midpoint_gate", P), ("scale_up", P), ("midpoint_up", P),
        ("gain_gate_up", P), ("bound_gate_up", P), ("signs_down", P), ("scale_down", P), ("midpoint_down", P),
        ("gain_down", P), ("bound_down", P), ("hidden_out", P), ("workspace", P), ("workspace_bytes", c_size_t),
        ("flags", P), ("norm_weight", P), ("epsilon", ctypes.c_float),
    ]


class FfnW1Args(ctypes.Structure):
    _fields_ = [
        ("x", P), ("y", P), ("tokens", c_int), ("hidden", c_int64), ("inter", c_int64),
        ("signs_gate_up", P), ("scale_gate", P), ("scale_up", P), ("signs_down", P), ("scale_down", P),
        ("hidden_out", P), ("workspace", P), ("workspace_bytes", c_size_t), ("flags", P),
    ]


class FfnLargeArgs(ctypes.Structure):
    _fields_ = [
        ("x", P), ("y", P), ("tokens", c_int64), ("hidden", c_int64), ("inter", c_int64),
        ("signs_gate_up_i8", P), ("scale_gate", P), ("scale_up", P), ("signs_down_i8", P), ("scale_down", P),
        ("hidden_out", P), ("workspace", P), ("workspace_bytes", c_size_t), ("flags", P),
    ]


SIGNATURES = {
    "bd_abi_version": (c_int, []),
    "bd_status_string": (ctypes.c_char_p, [c_int]),
    "bd_device_info": (c_int, [P, P, P]),
    "bd_pack_signs": (c_int, [P, c_int64, c_int64, P, P, P]),
    "bd_t16_words": (c_int64, [c_int64, c_int64]),
    "bd_tile_signs_t16": (c_int, [P, c_int64, c_int64, P, c_int, c_int, P, P]),
    "bd_tile_gguf_t16": (c_int, [P, c_int64, c_int64, P, c_int, c_int, P]),
    "bd_w8_words": (c_int64, [c_int64, c_int64]),
    "bd_tile_signs_w8": (c_int, [P, c_int64, c_int64, P, c_int, c_int, P, P]),
    "bd_quantize_codes": (c_int, [P, c_int64, c_int64, c_int64, P, P, c_int, P, P, P, P]),
    "bd_codes_ld": (c_int64, [c_int64]),
    "bd_codes_bytes": (c_int64, [c_int64, c_int64]),
    "bd_projection_workspace_bytes": (c_size_t, [c_int, c_int64]),
    "bd_projection_he4": (c_int, [P, P, c_int, c_int64, c_int64, P, P, P, P, c_int, P, P, P, P, c_size_t, P]),
    "bd_ffn_workspace_bytes": (c_size_t, [c_int, c_int64, c_int64]),
    "bd_ffn_he4": (c_int, [ctypes.POINTER(FfnHe4Args), P]),
    "bd_d8_bytes": (c_int64, [c_int64, c_int64]),
    "bd_tile_signs_d8": (c_int, [P, c_int64, c_int64, P, P, P]),
    "bd_ffn_fused_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "bd_ffn_fused_shape": (c_int, [c_int64, c_int64, P]),
    "bd_ffn_he4_fused": (c_int, [ctypes.POINTER(FfnHe4Args), P, P]),
    "bd_ffn_w1": (c_int, [ctypes.POINTER(FfnW1Args), P]),
    "bd_binarize_rows": (c_int, [P, c_int64, c_int64, P, P, P, P]),
    "bd_projection_w1a1_workspace_bytes": (c_size_t, [c_int64, c_int64]),
    "bd_projection_w1a1": (c_int, [P, c_int, c_int64, c_int64, P, P, P, P, P, c_size_t, P, P]),
    "bd_ffn_w1a1": (c_int, [ctypes.POINTER(FfnW1Args), P]),
    "bd_i8_ld": (c_int64, [c_int64]),
    "bd_i8_bytes": (c_int64, [c_int64, c_int64]),
    "bd_tile_signs_i8": (c_int, [P, c_int64, c_int64, P, c_int, c_int, P, P]),
    "bd_gemm_i8": (c_int, [P, c_int64, c_int64, P, c_int64, P, P]),
    "bd_ffn_large_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
    "bd_ffn_w1a1_large": (c_int, [ctypes.POINTER(FfnLargeArgs), P]),
    "bd_quantize_rows_bf16": (c_int, [P, c_int64, c_int64, P, P, c_int, P, P, P, P]),
    "bd_sign_rows": (c_int, [P, c_int64, P, P, P, P]),
    "bd_he4_epilogue": (c_int, [P, c_int64, c_int64, P, P, P, c_int, P, P, P, P]),
    "bd_ste_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64]),
    "bd_ste_grad_prep": (c_int, [P, P, c_int64, c_int64, P, P, P, c_int, P, P, P, c_int64, P, P, c_int64, P, P, P,
                                 P, c_size_t, P]),
    "bd_quantize_rows_i8": (c_int, [P, c_int64, c_int64, P, P, c_int, P, c_int64, P, P, P]),
    "bd_projection_he4_tc": (c_int, [P, c_int64, P, c_int64, c_int64, P, c_int64, P, P, P, c_int, P, P, P, P, P]),
    "bd_sign_cols_bf16": (c_int, [P, c_int64, c_int64, P, c_int64, P, P]),
    "bd_codes_transpose_bf16": (c_int, [P, c_int64, c_int64, c_int64, P, c_int64, P]),
    "bd_gemm_bf16_split": (c_int, [P, P, c_int64, c_int64, c_int64, P, c_int64, c_int64, P, c_int64, P, c_size_t,
                                   P]),
    "bd_gemm_split_workspace_bytes": (c_size_t, [c_int64, c_int64, c_int64, c_int]),
    "bd_split_bf16": (c_int, [P, c_int64, c_int64, c_int64, c_int, P, P, c_int64, P]),
    "bd_gemm_bf16_split3": (c_int, [P, P, c_int64, c_int64, c_int64, P, P, c_int64, c_int64, P, c_int64, P,
                                    c_size_t, P]),
    "bd_loss_head_stats_count": (c_int64, [c_int64, c_int64]),
    "bd_loss_head_forward": (c_int, [P, P, c_int64, c_int64, c_int64, P, P, c_int64, P, P, P, P, P, P, P, P, P]),
    "bd_loss_head_grad": (c_int, [P, P, c_int64, c_int64, c_int64, P, P, c_int64, P, P, P, P, P, c_int64, P]),
    "bd_rms_forward": (c_int, [P, c_int64, c_int64, P, ctypes.c_float, P, P, P]),
    "bd_rms_partials": (c_int64, [c_int64, c_int64]),
    "bd_rms_backward": (c_int, [P, c_int64, c_int64, P, P, P, P, P, P, P]),
    "bd_head_post": (c_int, [P, c_int64, c_int64, c_int, c_int, P, ctypes.c_float, P, P, c_int, P, P, P, P]),
    "bd_head_post_partials": (c_int64, [c_int64, c_int]),
    "bd_head_post_backward": (c_int, [P, c_int64, c_int64, c_int, c_int, P, P, P, P, P, P, P, P, P]),
    "bd_train_attention_pack": (c_int, [P, P, P, P, P, P, c_int64, c_int64, c_int64, P, c_int64, c_int64, c_int,
                                        c_int, c_int, c_int, c_int, c_int, P, P, P, P, P, P, P, P, P, P]),
    "bd_train_attention_pack_grad": (c_int, [P, P, c_int, c_int, c_int, c_int, c_int, P, P, P, P, P]),
    "bd_train_attention_forward": (c_int, [P, P, P, P, P, P, P, P, c_int, c_int, c_int, c_int, c_int, c_int,
                                           ctypes.c_float, P, P, P, P]),
    "bd_train_attention_backward": (c_int, [P, P, P, P, P, P, P, P, P, P, P, P, P, P, c_int, c_int, c_int, c_int,
                                            c_int, c_int, ctypes.c_float, P, P, P, P, P, P, P]),
    "bd_ste_weight_grad_partials": (c_int64, [c_int64, c_int64]),
    "bd_ste_weight_grad": (c_int, [P, P, c_int64, c_int64, c_int64, P, c_int64, P, P, ctypes.c_float, P, c_int, P, P,
                                   P, P]),
    "bd_ste_input_backward": (c_int, [P, P, P, P, c_int64, c_int64, P, P, c_int, P, P, P, c_int, P, c_size_t,
                                      P]),
    "bd_ste_sumsq_count": (c_int, [c_int64]),
    "bd_ste_sign_backward": (c_int, [P, P, P, c_int64, ctypes.c_float, P, c_int, P, P, P]),
    "bd_sum_squares_count": (c_int, [c_int64]),
    "bd_sum_squares": (c_int, [P, c_int64, P, P]),
    "bd_grad_norm": (c_int, [P, c_int64, ctypes.c_float, P, P, P, P]),
    "bd_adamw_latent": (c_int, [P, P, P, P, c_int64, c_int64, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                                ctypes.c_double, ctypes.c_longlong, P, c_int, P, c_int, c_int, P, P]),
    "bd_adamw": (c_int, [P, P, P, P, c_int64, ctypes.c_double, ctypes.c_double, ctypes.c_double, ctypes.c_double,
                         ctypes.c_longlong, P, ctypes.c_float, P, P]),
    "bd_bound_latents": (c_int, [P, c_int64, c_int64, ctypes.c_float, P, P, P]),
    "bd_clamp": (c_int, [P, c_int64, ctypes.c_float, ctypes.c_float, P]),
    "bd_accept_workspace_bytes": (c_size_t, [c_int, c_int]),
    "bd_accept_greedy": (c_int, [P, c_int, c_int, c_int64, P, P, c_int, P, P, P, P, c_size_t, P, P]),
    "bd_accept_greedy_noalloc": (c_int, [P, c_int, c_int, c_int64, P, P, c_int, P, P, P, P, P]),
    "bd_rejection_workspace_bytes": (c_size_t, [c_int, c_int, c_int64]),
    "bd_ingest_taps": (c_int, [P, c_int, c_int, c_int64, c_int64, P, c_int, P, P]),
    "bd_gemm_bf16": (c_int, [P, c_int64, c_int64, c_int64, P, c_int64, c_int64, P, c_int64, P, c_size_t, P]),
    "bd_accept_rejection": (c_int, [P, P, c_int, c_int, c_int64, P, P, c_int, ctypes.c_ulonglong, ctypes.c_uint32,
                                    P, P, P, c_size_t, P, P]),
    "bd_argmax_rows_bf16": (c_int, [P, c_int64, c_int64, P, P, P]),
    "bd_w16_bytes": (c_int64, [c_int64, c_int64]),
    "bd_tile_w16": (c_int, [P, c_int, c_int64, c_int64, P, P]),
    "bd_x16_bytes": (c_int64, [c_int, c_int64]),
    "bd_pack_x16": (c_int, [P, c_int, c_int64, c_int64, P, ctypes.c_float, P, P, c_int64, P, P]),
    "bd_pack_x16_bf16": (c_int, [P, c_int, c_int64, c_int64, P, ctypes.c_float, P, P, c_int64, P, P]),
    "bd_gemv_workspace_bytes": (c_size_t, [c_int, c_int64, c_int64]),
    "bd_gemv_bf16": (c_int, [P, c_int64, c_int64, P, c_int, P, c_int64, P, P, P, P, c_size_t, P]),
    "bd_argmax_finish": (c_int, [P, c_int, P, P]),
    "bd_embed_rows": (c_int, [P, c_int64, c_int64, P, c_int, P, P, P]),
    "bd_round_submit": (c_int, [P, P, P, c_size_t, P, P, P, P, c_int, P]),
    "bd_rms_rows": (c_int, [P, c_int, c_int64, c_int64, P, ctypes.c_float, P, c_int64, P]),
    "bd_heads_post": (c_int, [P, c_int, c_int64, c_int64, c_int, c_int, P, ctypes.c_float, c_int,
                              ctypes.c_float, c_int64, P, c_int64, P, P]),
    "bd_qkv_post": (c_int, [P, c_int, c_int64, c_int, c_int, c_int, P, P, ctypes.c_float, ctypes.c_float, c_int64,
                            P, c_int64, P, P, c_int64, P, P]),
    "bd_context_kv_post": (c_int, [P, c_int, c_int64, c_int, c_int64, c_int, c_int, P, ctypes.c_float, ctypes.c_float,
                                   c_int64, P, P, c_int64, c_int64, P, P]),
    "bd_attention_workspace_bytes": (c_size_t, [c_int, c_int, c_int]),
    "bd_attention_decode": (c_int, [P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int64, c_int64, c_int64, P,
                                    P, c_size_t, P]),
    "bd_attention_decode_x16": (c_int, [P, P, P, c_int, c_int, c_int, c_int, c_int, c_int, c_int64, c_int64,
                                        c_int64, P, P, P, c_size_t, P]),
}

_lib = None


def header_symbols() -> list[str]:
    """Names of the functions declared in ``include/bitdraft.h``."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(bd_[a-z0-9_]+)\s*\(", text)))


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not LIBRARY.exists():
        raise RuntimeError(
            f"{LIBRARY.name} is not built: run `python __graft_entry__.py build` "
            "(nvcc for sm_100a); there is no CPU fallback"
        )
    lib = ctypes.CDLL(str(LIBRARY))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


# Kernel launches issued by each entry point (for launch accounting).
KERNELS_PER_CALL = {"bd_ffn_he4": 3, "bd_ffn_he4_fused": 2, "bd_loss_head_forward": 3, "bd_ffn_w1": 4, "bd_attention_decode": 2, "bd_attention_decode_x16": 2,
                    "bd_accept_rejection": 2,
                    "bd_ste_grad_prep": 2, "bd_ste_input_backward": 2, "bd_train_attention_backward": 3}
launches = 0


_SIZES: dict[tuple, int] = {}


def size(name: str, *args) -> int:
    """A size query of the library (``bd_*_bytes``, ``*_partials``, ``*_ld``, ...), memoised:
    each is a pure function of its integer arguments within a process."""
    key = (name,) + args
    hit = _SIZES.get(key)
    if hit is None:
        hit = _SIZES[key] = int(getattr(load(), name)(*args))
    return hit


def call(name: str, *args, kernels: int | None = None) -> None:
    """Call an int-status entry point; raise on a non-zero status.  ``kernels``
    overrides the launch count of entry points whose count depends on sizes."""
    global launches
    launches += KERNELS_PER_CALL.get(name, 1) if kernels is None else kernels
    status = getattr(load(), name)(*args)
    if status != BD_OK:
        message = load().bd_status_string(status).decode()
        if status == 1:
            raise ValueError(f"{name}: {message}")
        raise RuntimeError(f"{name}: {message} (status {status})")


def raise_flags(value: int) -> None:
    """Turn device-reported flag bits into the reference's ValueError (RuntimeError
    for device failures such as a timed-out wait)."""
    for bit, message in FLAG_ERRORS:
        if value & bit:
            raise RuntimeError(message)
    for bit, message in FLAG_MESSAGES:
        if value & bit:
            raise ValueError(message)
