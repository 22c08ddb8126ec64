"""Torch-facing wrappers of the C ABI: device memory, streams and error flags.

PyTorch supplies device buffers and the current stream; every computation is a
``libbitdraft.so`` kernel.  Data-dependent errors come back as device flags and
are raised as the reference's ``ValueError`` messages when the wrapper (or the
caller, for deferred checks) reads them.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from . import _lib

MAX_DECODE_TOKENS = 32
LARGE_M_TOKENS = 128  # token counts from here on go to the tensor cores when the weights allow it


def _p(t: Tensor | None):
    return None if t is None else t.data_ptr()


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(device: torch.device) -> int:
    """The current CUDA stream of ``device`` as a raw handle (the torch-internal
    getter where it exists: it skips building a Python stream object per launch)."""
    if _RAW_STREAM is not None:
        return _RAW_STREAM(torch.cuda.current_device() if device.index is None else device.index)
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*tensors: Tensor) -> torch.device:
    device = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("bitdraft kernels take CUDA tensors")
        if not t.is_contiguous():
            raise ValueError("bitdraft kernels take contiguous tensors")
        device = t.device if device is None else device
        if t.device != device:
            raise ValueError("all tensors must be on one device")
    if device is None:
        raise ValueError("no device tensor given")
    return device


class Flags:
    """A device int32 word the kernels OR error bits into."""

    def __init__(self, device: torch.device):
        self.tensor = torch.zeros(1, dtype=torch.int32, device=device)

    @property
    def ptr(self) -> int:
        return self.tensor.data_ptr()

    def check(self) -> None:
        value = int(self.tensor.item())
        if value:
            self.tensor.zero_()
            _lib.raise_flags(value)


_workspaces: dict[tuple, Tensor] = {}


def workspace(device: torch.device, kind: str, nbytes: int) -> Tensor:
    """A cached byte buffer per (device, kind), zeroed when created; kernels that keep
    counters in their workspace leave them zeroed."""
    key = (device.index if device.index is not None else torch.cuda.current_device(), kind)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        _workspaces[key] = buf
    return buf


# --------------------------------------------------------------------------- signs


def pack_signs(latent: Tensor) -> Tensor:
    """GGUF sign words ``int32 [rows, ceil(cols/32)]`` (export.packed_signs, export.py:79-86)."""
    if latent.dtype != torch.float32 or latent.ndim != 2:
        raise ValueError("finite F32 sign matrix required")
    device = _require_cuda(latent)
    rows, cols = latent.shape
    words = torch.empty((rows, (cols + 31) // 32), dtype=torch.int32, device=device)
    flags = Flags(device)
    _lib.call("bd_pack_signs", _p(latent), rows, cols, _p(words), flags.ptr, _stream(device))
    flags.check()
    return words


def t16_words(rows: int, cols: int) -> int:
    return int(_lib.load().bd_t16_words(rows, cols))


def tile_t16(latent: Tensor, block_stride: int = 1, block_offset: int = 0, out: Tensor | None = None,
             flags: Flags | None = None) -> Tensor:
    """T16 decode-layout sign words of an F32 latent matrix (int32 storage)."""
    if latent.dtype != torch.float32 or latent.ndim != 2:
        raise ValueError("finite F32 sign matrix required")
    device = _require_cuda(latent)
    rows, cols = latent.shape
    if out is None:
        out = torch.zeros(t16_words(rows, cols) * block_stride, dtype=torch.int32, device=device)
    own = flags is None
    flags = flags or Flags(device)
    _lib.call("bd_tile_signs_t16", _p(latent), rows, cols, _p(out), block_stride, block_offset, flags.ptr,
              _stream(device))
    if own:
        flags.check()
    return out


def tile_gguf_t16(words: Tensor, rows: int, cols: int, block_stride: int = 1, block_offset: int = 0,
                  out: Tensor | None = None) -> Tensor:
    device = _require_cuda(words)
    if out is None:
        out = torch.zeros(t16_words(rows, cols) * block_stride, dtype=torch.int32, device=device)
    _lib.call("bd_tile_gguf_t16", _p(words), rows, cols, _p(out), block_stride, block_offset, _stream(device))
    return out


def tile_gate_up(gate: Tensor, up: Tensor, flags: Flags | None = None) -> Tensor:
    """Gate and up signs with their 16-row blocks interleaved (gate, up, gate, up, ...)."""
    if gate.shape != up.shape:
        raise ValueError("gate and up must have one shape")
    out = torch.zeros(t16_words(*gate.shape) * 2, dtype=torch.int32, device=gate.device)
    tile_t16(gate, 2, 0, out, flags)
    tile_t16(up, 2, 1, out, flags)
    return out


# --------------------------------------------------------------------------- projections


def codes_ld(cols: int) -> int:
    return int(_lib.load().bd_codes_ld(cols))


def quantize_codes(x: Tensor, gain: Tensor, bound: Tensor, bits: int, flags: Flags | None = None):
    """HE4 activation codes (int8, F8 fragment layout) and exact row sums (model.py:128-140)."""
    device = _require_cuda(x, gain, bound)
    rows, cols = x.shape
    ld = codes_ld(cols)
    codes = torch.zeros(int(_lib.load().bd_codes_bytes(rows, cols)), dtype=torch.int8, device=device)
    sums = torch.empty(rows, dtype=torch.int32, device=device)
    own = flags is None
    flags = flags or Flags(device)
    _lib.call("bd_quantize_codes", _p(x), rows, cols, ld, _p(gain), _p(bound), bits, _p(codes), _p(sums),
              flags.ptr, _stream(device))
    if own:
        flags.check()
    return codes, sums


def projection_he4(codes: Tensor, sums: Tensor, signs_t16: Tensor, in_features: int, scale: Tensor,
                   midpoint: Tensor, bound: Tensor, bits: int, residual: Tensor | None = None,
                   raw_dot: bool = False):
    """HE4 projection forward value from codes (model.py:141-150); optional exact dots."""
    device = _require_cuda(codes, sums, signs_t16, scale, midpoint, bound, residual)
    tokens = sums.shape[0]
    out_features = scale.shape[0]
    y = torch.empty((tokens, out_features), dtype=torch.float32, device=device)
    raw = torch.empty((tokens, out_features), dtype=torch.int32, device=device) if raw_dot else None
    nbytes = int(_lib.load().bd_projection_workspace_bytes(tokens, out_features))
    ws = workspace(device, "projection", nbytes)
    _lib.call("bd_projection_he4", _p(codes), _p(sums), tokens, in_features, out_features, _p(signs_t16),
              _p(scale), _p(midpoint), _p(bound), bits, _p(residual), _p(y), _p(raw), _p(ws), ws.numel(),
              _stream(device))
    return (y, raw) if raw_dot else y


@dataclass
class PackedProjection:
    scale: Tensor
    midpoint: Tensor


@dataclass
class PackedFFN:
    """Device-resident sign tiles and epilogue operands of one SwiGLU block."""

    hidden: int
    inter: int
    signs_gate_up: Tensor
    signs_down: Tensor
    scale_gate: Tensor
    scale_up: Tensor
    scale_down: Tensor
    midpoint_gate: Tensor | None = None
    midpoint_up: Tensor | None = None
    midpoint_down: Tensor | None = None
    gain_gate_up: Tensor | None = None
    bound_gate_up: Tensor | None = None
    gain_down: Tensor | None = None
    bound_down: Tensor | None = None
    signs_gate_up_i8: Tensor | None = None  # large-M copies (tensor-core path), see pack_ffn(large=True)
    signs_down_i8: Tensor | None = None
    signs_down_d8: Tensor | None = None  # down signs of the two-launch HE4 block (tokens <= 16)


def w8_words(rows: int, cols: int) -> int:
    return int(_lib.load().bd_w8_words(rows, cols))


def tile_w8(latent: Tensor, block_stride: int = 1, block_offset: int = 0, out: Tensor | None = None,
            flags: Flags | None = None) -> Tensor:
    """W8 sign words of an F32 latent matrix (the decode feed-forward's B-fragment layout)."""
    if latent.dtype != torch.float32 or latent.ndim != 2:
        raise ValueError("finite F32 sign matrix required")
    device = _require_cuda(latent)
    rows, cols = latent.shape
    if out is None:
        out = torch.zeros(w8_words(rows, cols) * block_stride, dtype=torch.int32, device=device)
    own = flags is None
    flags = flags or Flags(device)
    _lib.call("bd_tile_signs_w8", _p(latent), rows, cols, _p(out), block_stride, block_offset, flags.ptr,
              _stream(device))
    if own:
        flags.check()
    return out


def tile_d8(latent: Tensor, flags: Flags | None = None) -> Tensor | None:
    """D8 sign bytes of the down matrix ``[hidden, inter]`` for the two-launch HE4
    block: ``[hidden / 8][ceil(inter / 128)][32 lanes][4]``: lane ``4 g + t``,
    byte ``s % 4`` of 4-k-step group ``s / 4`` of n-tile ``n`` has bit ``4 r + j`` =
    ``latent[8 n + g, 32 s + 16 r + 4 t + j] >= 0``.  None when a dimension is not
    a multiple of 32 (the block then takes the three-kernel path)."""
    if latent.dtype != torch.float32 or latent.ndim != 2:
        raise ValueError("finite F32 sign matrix required")
    device = _require_cuda(latent)
    rows, cols = latent.shape
    if rows % 32 or cols % 32:
        return None
    out = torch.zeros(int(_lib.load().bd_d8_bytes(rows, cols)), dtype=torch.uint8, device=device)
    own = flags is None
    flags = flags or Flags(device)
    _lib.call("bd_tile_signs_d8", _p(latent), rows, cols, _p(out), flags.ptr, _stream(device))
    if own:
        flags.check()
    return out


def tile_gate_up_w8(gate: Tensor, up: Tensor, flags: Flags | None = None) -> Tensor:
    """Gate and up W8 signs with their 8-row n-tiles interleaved (gate, up, gate, up, ...)."""
    if gate.shape != up.shape:
        raise ValueError("gate and up must have one shape")
    out = torch.zeros(w8_words(*gate.shape) * 2, dtype=torch.int32, device=gate.device)
    tile_w8(gate, 2, 0, out, flags)
    tile_w8(up, 2, 1, out, flags)
    return out


def pack_ffn(gate: Tensor, up: Tensor, down: Tensor, scale_gate: Tensor | None = None,
             scale_up: Tensor | None = None, scale_down: Tensor | None = None, large: bool = False) -> PackedFFN:
    """Pack latent F32 matrices into W8 sign words; row scales default to ``mean|W|`` (model.py:123).
    ``large`` also keeps the +-1 int8 copies that the tensor-core path (token counts
    in the hundreds) reads."""
    flags = Flags(gate.device)
    signs_gate_up = tile_gate_up_w8(gate.contiguous(), up.contiguous(), flags)
    signs_down = tile_w8(down.contiguous(), flags=flags)
    signs_down_d8 = tile_d8(down.contiguous(), flags=flags)
    gu_i8 = tile_gate_up_i8(gate.contiguous(), up.contiguous(), flags) if large else None
    dn_i8 = tile_i8(down.contiguous(), flags=flags) if large else None
    flags.check()
    return PackedFFN(
        hidden=gate.shape[1], inter=gate.shape[0], signs_gate_up=signs_gate_up, signs_down=signs_down,
        scale_gate=(gate.abs().mean(-1) if scale_gate is None else scale_gate).contiguous(),
        scale_up=(up.abs().mean(-1) if scale_up is None else scale_up).contiguous(),
        scale_down=(down.abs().mean(-1) if scale_down is None else scale_down).contiguous(),
        signs_gate_up_i8=gu_i8, signs_down_i8=dn_i8, signs_down_d8=signs_down_d8,
    )


# --------------------------------------------------------------------------- tensor-core (large-M) path


def tile_i8(latent: Tensor, block_stride: int = 1, block_offset: int = 0, out: Tensor | None = None,
            flags: Flags | None = None) -> Tensor:
    """+-1 int8 copy of the signs [rows padded to 128, bd_i8_ld(cols)] (tensor-core B operand)."""
    if latent.dtype != torch.float32 or latent.ndim != 2:
        raise ValueError("finite F32 sign matrix required")
    device = _require_cuda(latent)
    rows, cols = latent.shape
    lib = _lib.load()
    if out is None:
        out = torch.zeros(int(lib.bd_i8_bytes(rows, cols)) * block_stride, dtype=torch.int8, device=device)
    own = flags is None
    flags = flags or Flags(device)
    _lib.call("bd_tile_signs_i8", _p(latent), rows, cols, _p(out), block_stride, block_offset, flags.ptr,
              _stream(device))
    if own:
        flags.check()
    return out


def tile_gate_up_i8(gate: Tensor, up: Tensor, flags: Flags | None = None) -> Tensor:
    """Gate and up int8 signs with their 128-row blocks interleaved."""
    out = torch.zeros(int(_lib.load().bd_i8_bytes(*gate.shape)) * 2, dtype=torch.int8, device=gate.device)
    tile_i8(gate, 2, 0, out, flags)
    tile_i8(up, 2, 1, out, flags)
    return out


def gemm_i8(codes: Tensor, k: int, signs_i8: Tensor, outs: int) -> Tensor:
    """Exact int32 dots of int8 codes [tokens, bd_i8_ld(k)] (the first k columns) with +-1 signs."""
    device = _require_cuda(codes, signs_i8)
    if codes.dtype != torch.int8 or codes.ndim != 2 or codes.shape[1] != int(_lib.load().bd_i8_ld(k)):
        raise ValueError("codes must be int8 [tokens, bd_i8_ld(k)]")
    tokens = codes.shape[0]
    dots = torch.empty((tokens, outs), dtype=torch.int32, device=device)
    _lib.call("bd_gemm_i8", _p(codes), tokens, k, _p(signs_i8), outs, _p(dots), _stream(device))
    return dots


def gemm_bf16(a: Tensor, b: Tensor, out: Tensor | None = None) -> Tensor:
    """``a @ b.T`` for bf16 ``a [m, k]`` and ``b [n, k]`` on the tensor cores (fp32 accumulators, fp32 result)."""
    if a.dtype != torch.bfloat16 or b.dtype != torch.bfloat16 or a.ndim != 2 or b.ndim != 2 or a.shape[1] != b.shape[1]:
        raise ValueError("gemm_bf16 takes bf16 [m, k] and [n, k]")
    m, k = a.shape
    n = b.shape[0]
    if a.stride(1) != 1 or b.stride(1) != 1 or a.stride(0) % 8 or b.stride(0) % 8:
        raise ValueError("gemm_bf16 operands need unit column stride and row strides that are multiples of 8")
    device = _require_cuda(a, b)
    c = torch.empty((m, n), dtype=torch.float32, device=device) if out is None else out
    nbytes = int(_lib.load().bd_gemm_split_workspace_bytes(m, n, k, 1))
    ws = workspace(device, "gemm_split", nbytes) if nbytes else None
    _lib.call("bd_gemm_bf16", _p(a), m, k, a.stride(0), _p(b), n, b.stride(0), _p(c), c.stride(0),
              None if ws is None else ws.data_ptr(), 0 if ws is None else ws.numel(), _stream(device))
    return c


def ffn_w1a1_large(x: Tensor, ffn: PackedFFN, hidden_out: bool = False, flags: Flags | None = None):
    """W1A1 SwiGLU block on the tensor cores (any token count; needs pack_ffn(large=True))."""
    if ffn.signs_gate_up_i8 is None or ffn.signs_down_i8 is None:
        raise ValueError("the tensor-core path needs pack_ffn(..., large=True)")
    device = _require_cuda(x)
    tokens = x.shape[0]
    y = torch.empty((tokens, ffn.hidden), dtype=torch.float32, device=device)
    h = torch.empty((tokens, ffn.inter), dtype=torch.float32, device=device) if hidden_out else None
    nbytes = int(_lib.load().bd_ffn_large_workspace_bytes(tokens, ffn.hidden, ffn.inter))
    ws = workspace(device, "ffn_large", nbytes)
    own = flags is None
    flags = flags or Flags(device)
    args = _lib.FfnLargeArgs(
        _p(x), _p(y), tokens, ffn.hidden, ffn.inter, _p(ffn.signs_gate_up_i8), _p(ffn.scale_gate),
        _p(ffn.scale_up), _p(ffn.signs_down_i8), _p(ffn.scale_down), _p(h), _p(ws), ws.numel(), flags.ptr,
    )
    _lib.call("bd_ffn_w1a1_large", _lib.ctypes.byref(args), _stream(device), kernels=4)
    if own:
        flags.check()
    return (y, h) if hidden_out else y


FUSED_MAX_TOKENS = 16


def ffn_he4(x: Tensor, ffn: PackedFFN, residual: Tensor | None = None, hidden_out: bool = False,
            flags: Flags | None = None, out: Tensor | None = None, norm: Tensor | None = None,
            epsilon: float = 1e-6, fused: bool = False):
    """HE4 SwiGLU block ``residual + down(silu(gate(n)) * up(n))`` (model.py:220-223).

    ``n = x``, or ``n = rms(x, norm, epsilon)`` when ``norm`` is given (then
    ``x`` is the residual stream itself).  Up to 16 tokens with D8 down signs
    run as two cluster launches (``bd_ffn_he4_fused``) when ``fused`` is
    True; otherwise the three-kernel path (``bd_ffn_he4``).
    """
    device = _require_cuda(x, residual, out)
    tokens = x.shape[0]
    if not 1 <= tokens <= MAX_DECODE_TOKENS:
        raise ValueError("decode feed-forward takes 1 to 32 tokens")
    y = torch.empty((tokens, ffn.hidden), dtype=torch.float32, device=device) if out is None else out
    h = torch.empty((tokens, ffn.inter), dtype=torch.float32, device=device) if hidden_out else None
    one_launch = fused and ffn.signs_down_d8 is not None and tokens <= FUSED_MAX_TOKENS
    if one_launch:
        nbytes = int(_lib.load().bd_ffn_fused_workspace_bytes(ffn.hidden, ffn.inter))
        ws = workspace(device, "ffn_fused", nbytes)
    else:
        nbytes = int(_lib.load().bd_ffn_workspace_bytes(tokens, ffn.hidden, ffn.inter))
        ws = workspace(device, "ffn", nbytes)
    own = flags is None
    flags = flags or Flags(device)
    args = _lib.FfnHe4Args(
        _p(x), _p(residual), _p(y), tokens, ffn.hidden, ffn.inter, _p(ffn.signs_gate_up), _p(ffn.scale_gate),
        _p(ffn.midpoint_gate), _p(ffn.scale_up), _p(ffn.midpoint_up), _p(ffn.gain_gate_up), _p(ffn.bound_gate_up),
        _p(ffn.signs_down), _p(ffn.scale_down), _p(ffn.midpoint_down), _p(ffn.gain_down), _p(ffn.bound_down),
        _p(h), _p(ws), ws.numel(), flags.ptr, _p(norm), float(epsilon),
    )
    if one_launch:
        _lib.call("bd_ffn_he4_fused", _lib.ctypes.byref(args), _p(ffn.signs_down_d8), _stream(device))
    else:
        _lib.call("bd_ffn_he4", _lib.ctypes.byref(args), _stream(device))
    if own:
        flags.check()
    return (y, h) if hidden_out else y


def ffn_w1(x: Tensor, ffn: PackedFFN, hidden_out: bool = False, flags: Flags | None = None):
    """Pure one-bit-weight SwiGLU with fp32 activations (16-bit fixed point inside)."""
    device = _require_cuda(x)
    tokens = x.shape[0]
    if not 1 <= tokens <= MAX_DECODE_TOKENS:
        raise ValueError("decode feed-forward takes 1 to 32 tokens")
    y = torch.empty((tokens, ffn.hidden), dtype=torch.float32, device=device)
    h = torch.empty((tokens, ffn.inter), dtype=torch.float32, device=device) if hidden_out else None
    nbytes = int(_lib.load().bd_ffn_workspace_bytes(tokens, ffn.hidden, ffn.inter))
    ws = workspace(device, "ffn", nbytes)
    own = flags is None
    flags = flags or Flags(device)
    args = _lib.FfnW1Args(
        _p(x), _p(y), tokens, ffn.hidden, ffn.inter, _p(ffn.signs_gate_up), _p(ffn.scale_gate), _p(ffn.scale_up),
        _p(ffn.signs_down), _p(ffn.scale_down), _p(h), _p(ws), ws.numel(), flags.ptr,
    )
    _lib.call("bd_ffn_w1", _lib.ctypes.byref(args), _stream(device))
    if own:
        flags.check()
    return (y, h) if hidden_out else y


# --------------------------------------------------------------------------- W1A1


def binarize_rows(x: Tensor, flags: Flags | None = None):
    """Sign words (bit j of word w = ``x[r, 32w+j] >= 0``) and fixed-order mean|x| per row."""
    device = _require_cuda(x)
    if x.dtype != torch.float32 or x.ndim != 2:
        raise ValueError("binarize_rows takes F32 [rows, cols]")
    rows, cols = x.shape
    words = torch.empty((rows, (cols + 31) // 32), dtype=torch.int32, device=device)
    mean = torch.empty(rows, dtype=torch.float32, device=device)
    own = flags is None
    flags = flags or Flags(device)
    _lib.call("bd_binarize_rows", _p(x), rows, cols, _p(words), _p(mean), flags.ptr, _stream(device))
    if own:
        flags.check()
    return words, mean


def projection_w1a1(x: Tensor, signs_t16: Tensor, scale: Tensor, raw_dot: bool = False,
                    flags: Flags | None = None):
    """W1A1 projection ``(D * scale[o]) * mean|x_t|`` with the exact +-1 dot D."""
    device = _require_cuda(x, signs_t16, scale)
    tokens, in_features = x.shape
    out_features = scale.shape[0]
    y = torch.empty((tokens, out_features), dtype=torch.float32, device=device)
    raw = torch.empty((tokens, out_features), dtype=torch.int32, device=device) if raw_dot else None
    nbytes = int(_lib.load().bd_projection_w1a1_workspace_bytes(in_features, out_features))
    ws = workspace(device, "w1a1", nbytes)
    own = flags is None
    flags = flags or Flags(device)
    _lib.call("bd_projection_w1a1", _p(x), tokens, in_features, out_features, _p(signs_t16), _p(scale), _p(y),
              _p(raw), _p(ws), ws.numel(), flags.ptr, _stream(device), kernels=2 * ((tokens + 31) // 32))
    if own:
        flags.check()
    return (y, raw) if raw_dot else y


def ffn_w1a1(x: Tensor, ffn: PackedFFN, hidden_out: bool = False, flags: Flags | None = None):
    """W1A1 SwiGLU: each projection input is re-binarised with its own mean|x|.  Token
    counts of 128 and more take the tensor-core path when the block was packed with it."""
    if x.shape[0] >= LARGE_M_TOKENS and ffn.signs_gate_up_i8 is not None:
        return ffn_w1a1_large(x, ffn, hidden_out, flags)
    device = _require_cuda(x)
    tokens = x.shape[0]
    y = torch.empty((tokens, ffn.hidden), dtype=torch.float32, device=device)
    h = torch.empty((tokens, ffn.inter), dtype=torch.float32, device=device) if hidden_out else None
    nbytes = int(_lib.load().bd_ffn_workspace_bytes(MAX_DECODE_TOKENS, ffn.hidden, ffn.inter))
    ws = workspace(device, "ffn", nbytes)
    own = flags is None
    flags = flags or Flags(device)
    args = _lib.FfnW1Args(
        _p(x), _p(y), tokens, ffn.hidden, ffn.inter, _p(ffn.signs_gate_up), _p(ffn.scale_gate), _p(ffn.scale_up),
        _p(ffn.signs_down), _p(ffn.scale_down), _p(h), _p(ws), ws.numel(), flags.ptr,
    )
    _lib.call("bd_ffn_w1a1", _lib.ctypes.byref(args), _stream(device), kernels=4 * ((tokens + 31) // 32))
    if own:
        flags.check()
    return (y, h) if hidden_out else y


# --------------------------------------------------------------------------- acceptance


def accept_greedy(logits: Tensor, drafts: Tensor, eog: Tensor | None = None, targets: bool = False,
                  flags: Flags | None = None):
    """Greedy block acceptance (benchmarks/verifier.py:107-113).

    ``logits`` bf16 ``[B, n+1, V]``, ``drafts`` int32 ``[B, n]``, ``eog`` int32.
    Returns ``(accepted [B], next_token [B])`` (+ ``targets [B, n+1]``).
    """
    if logits.dtype != torch.bfloat16 or logits.ndim != 3:
        raise ValueError("logits must be bf16 [requests, drafts + 1, vocab]")
    if drafts.dtype != torch.int32 or drafts.ndim != 2 or logits.shape[:2] != (drafts.shape[0], drafts.shape[1] + 1):
        raise ValueError("drafts must be int32 [requests, drafts]")
    device = _require_cuda(logits, drafts, eog)
    requests, n = drafts.shape
    accepted = torch.empty(requests, dtype=torch.int32, device=device)
    nxt = torch.empty(requests, dtype=torch.int32, device=device)
    tg = torch.empty((requests, n + 1), dtype=torch.int32, device=device) if targets else None
    nbytes = int(_lib.load().bd_accept_workspace_bytes(requests, n))
    ws = workspace(device, "accept", nbytes)
    own = flags is None
    flags = flags or Flags(device)
    n_eog = 0 if eog is None else eog.numel()
    _lib.call("bd_accept_greedy", _p(logits), requests, n, logits.shape[2], _p(drafts), _p(eog), n_eog,
              _p(accepted), _p(nxt), _p(tg), _p(ws), ws.numel(), flags.ptr, _stream(device))
    if own:
        flags.check()
    return (accepted, nxt, tg) if targets else (accepted, nxt)


def accept_rejection(target_logits: Tensor, draft_logits: Tensor, drafts: Tensor, seed: int, offset: int = 0,
                     eog: Tensor | None = None, flags: Flags | None = None):
    """Temperature-1 speculative rejection sampling under the deterministic contract
    of ``bd_accept_rejection``.  Returns ``(accepted [B], next_token [B])``."""
    if target_logits.dtype != torch.bfloat16 or draft_logits.dtype != torch.bfloat16:
        raise ValueError("logits must be bf16")
    if drafts.dtype != torch.int32 or drafts.ndim != 2:
        raise ValueError("drafts must be int32 [requests, drafts]")
    requests, n = drafts.shape
    if target_logits.shape[:2] != (requests, n + 1) or draft_logits.shape[:2] != (requests, n) \
            or target_logits.shape[2] != draft_logits.shape[2]:
        raise ValueError("logits must be [requests, drafts + 1, vocab] and [requests, drafts, vocab]")
    device = _require_cuda(target_logits, draft_logits, drafts, eog)
    accepted = torch.empty(requests, dtype=torch.int32, device=device)
    nxt = torch.empty(requests, dtype=torch.int32, device=device)
    ws = workspace(device, "rejection", int(_lib.load().bd_rejection_workspace_bytes(requests, n, target_logits.shape[2])))
    own = flags is None
    flags = flags or Flags(device)
    n_eog = 0 if eog is None else eog.numel()
    _lib.call("bd_accept_rejection", _p(target_logits), _p(draft_logits), requests, n, target_logits.shape[2],
              _p(drafts), _p(eog), n_eog, seed & 0xFFFFFFFFFFFFFFFF, offset & 0xFFFFFFFF, _p(accepted), _p(nxt),
              _p(ws), ws.numel(), flags.ptr, _stream(device))
    if own:
        flags.check()
    return accepted, nxt


_INGEST_OUT = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def ingest_taps(captures: Tensor, out_dtype: torch.dtype = torch.float16, device: torch.device | None = None,
                flags: Flags | None = None) -> Tensor:
    """Tap-major teacher captures ``[taps, rows, hidden]`` (fp16 or fp32, on the GPU or in
    pinned host memory) as token-major drafter features ``[rows, taps * hidden]``
    (captures.py:124-137), with the loader's ``nonfinite teacher features`` check."""
    if captures.ndim != 3 or captures.dtype not in (torch.float16, torch.float32) or out_dtype not in _INGEST_OUT:
        raise ValueError("captures must be fp16/fp32 [taps, rows, hidden]; features fp16, bf16 or fp32")
    taps, rows, hidden = captures.shape
    if hidden % 8:
        raise ValueError("capture hidden size must be a multiple of 8")
    if captures.device.type != "cuda":
        captures = captures.contiguous().to(device or torch.device("cuda", torch.cuda.current_device()),
                                            non_blocking=True)
    src = captures.contiguous()
    dev = _require_cuda(src)
    out = torch.empty((rows, taps * hidden), dtype=out_dtype, device=dev)
    own = flags is None
    flags = flags or Flags(dev)
    _lib.call("bd_ingest_taps", _p(src), 16 if src.dtype == torch.float16 else 32, taps, rows, hidden, _p(out),
              _INGEST_OUT[out_dtype], flags.ptr, _stream(dev))
    if own:
        flags.check()
    return out


def argmax_rows(logits: Tensor, flags: Flags | None = None) -> Tensor:
    """Row argmax of bf16 rows, lowest index on ties (contracts.py:130-137)."""
    if logits.dtype != torch.bfloat16:
        raise ValueError("logits must be bf16")
    device = _require_cuda(logits)
    rows = logits.numel() // logits.shape[-1]
    out = torch.empty(logits.shape[:-1], dtype=torch.int32, device=device)
    own = flags is None
    flags = flags or Flags(device)
    _lib.call("bd_argmax_rows_bf16", _p(logits), rows, logits.shape[-1], _p(out), flags.ptr, _stream(device))
    if own:
        flags.check()
    return out
