"""Drop-in mirror of the reference model API (``w1a1_eagle/model.py``).

Same names, constructor arguments, parameter names and ValueError messages as
the reference.  The binary projections run in ``libbitdraft.so``:

* ``Projection`` quantizes with ``bd_quantize_rows_i8``, multiplies int8 codes
  by the int8 signs on the tcgen05 tensor cores (exact s32 accumulation) with
  the HE4 epilogue in the same kernel, and back-propagates with the
  straight-through kernels and tcgen05 GEMMs (``bd_ste_*``);
* ``Layer`` runs its SwiGLU tail through the fused decode block
  (``bd_ffn_he4``) when no gradient is needed and at most 32 rows come in;
* ``hard_sign``, ``bound_latents`` and ``clamp_latents`` are kernels too;
* the training attention (``train_attention``), the norms, the per-head rms,
  rotary and fp16 storage (``rms``, ``head_post``) and the frozen products
  (``frozen_linear``) are kernels of this library, forward and backward;
* ``LatentGradients`` turns the latent gradients of many backward passes into
  one tensor-core product per projection.

A CUDA device is required for these paths: there is no CPU fallback (``rms`` and
the loss bookkeeping keep the reference's torch expressions for CPU tensors, for
host-side checks only).
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor, nn
from torch.nn import functional

from . import _lib, ops

MAX_DECODE_ROWS = ops.MAX_DECODE_TOKENS
_DEFERRED: list[ops.Flags] = []  # flags words of the active deferred_checks contexts
_LATENT: list["LatentGradients"] = []  # active latent-gradient accumulations


@dataclass(frozen=True)
class Geometry:
    """Drafter geometry (``w1a1_eagle/model.py:11-47``), validated the same way."""

    hidden: int = 2560
    intermediate: int = 9216
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    layers: int = 6
    slots: int = 16
    taps: int = 8
    window: int = 4096
    epsilon: float = 1e-6
    theta: float = 1e7

    def __post_init__(self) -> None:
        sizes = (self.hidden, self.intermediate, self.heads, self.kv_heads, self.head_dim, self.layers, self.slots,
                 self.taps, self.window)
        if any(type(v) is not int or v < 1 for v in sizes):
            raise ValueError("invalid geometry")
        if self.heads % self.kv_heads or self.head_dim % 2:
            raise ValueError("invalid grouped rotary geometry")
        if (not math.isfinite(self.epsilon) or self.epsilon <= 0 or not math.isfinite(self.theta)
                or self.theta <= 0):
            raise ValueError("invalid numerical constants")


# --------------------------------------------------------------------------- elementwise helpers


class _RmsFn(torch.autograd.Function):
    """``rms`` on the GPU: one kernel forward (``bd_rms_forward``), one backward
    (``bd_rms_backward``: input and weight gradients)."""

    @staticmethod
    def forward(ctx, value, weight, epsilon):
        cols = value.shape[-1]
        x = value.reshape(-1, cols).float().contiguous()
        w = weight.detach().float().contiguous()
        rows = x.shape[0]
        out = torch.empty_like(x)
        inv = torch.empty(rows, dtype=torch.float32, device=x.device)
        _lib.call("bd_rms_forward", x.data_ptr(), rows, cols, w.data_ptr(), float(epsilon), out.data_ptr(),
                  inv.data_ptr(), _stream(x.device))
        ctx.save_for_backward(x, w, inv)
        ctx.shape = value.shape
        return out.view(value.shape)

    @staticmethod
    def backward(ctx, grad):
        x, w, inv = ctx.saved_tensors
        rows, cols = x.shape
        g = grad.reshape(rows, cols).float().contiguous()
        dx = torch.empty_like(x)
        parts = torch.empty(_lib.size("bd_rms_partials", rows, cols), dtype=torch.float32, device=x.device)
        dw = torch.empty(cols, dtype=torch.float32, device=x.device)
        _lib.call("bd_rms_backward", x.data_ptr(), rows, cols, w.data_ptr(), inv.data_ptr(), g.data_ptr(),
                  dx.data_ptr(), parts.data_ptr(), dw.data_ptr(), _stream(x.device), kernels=3)
        return dx.view(ctx.shape), dw, None


def rms(value: Tensor, weight: Tensor, epsilon: float) -> Tensor:
    """``value / sqrt(mean(value^2) + eps) * weight`` over the last axis (``model.py:50-51``);
    on CUDA tensors one kernel each way (``_RmsFn``), on CPU tensors the reference's
    expression."""
    if value.is_cuda and value.numel() > 0:
        return _RmsFn.apply(value, weight, epsilon)
    return value * torch.rsqrt(value.square().mean(-1, keepdim=True) + epsilon) * weight


_FREQUENCIES: dict[tuple[int, float, torch.device], Tensor] = {}


def _frequencies(width: int, theta: float, device: torch.device) -> Tensor:
    """``theta^(-2i/width)`` in fp32, evaluated once on the host (as the reference does)
    and kept on ``device``: no host round trip per call."""
    key = (width, float(theta), device)
    hit = _FREQUENCIES.get(key)
    if hit is None:
        exponents = torch.arange(0, width, 2, dtype=torch.float32) / width
        hit = torch.tensor(theta, dtype=torch.float32).pow(-exponents).to(device)
        _FREQUENCIES[key] = hit
    return hit


def rope(value: Tensor, positions: Tensor, theta: float) -> Tensor:
    """Rotate-half rotary embedding with frequencies ``theta^(-2i/width)`` (``model.py:54-63``)."""
    width = value.shape[-1]
    frequency = _frequencies(width, theta, value.device)
    angle = positions.float()[:, None] * frequency
    angle = torch.cat((angle, angle), -1).unsqueeze(1)
    first, second = value[..., : width // 2], value[..., width // 2:]
    return value * angle.cos() + torch.cat((-second, first), -1) * angle.sin()


def cache_storage(value: Tensor) -> Tensor:
    """Round through fp16 storage with a straight-through gradient (``model.py:98-102``).
    Inside ``deferred_checks`` an overflow is recorded on the device and raised
    when the context ends."""
    rounded = value.half().float()
    if _DEFERRED and value.is_cuda and _DEFERRED[-1].tensor.device == value.device:
        flags = _DEFERRED[-1].tensor
        flags.bitwise_or_((~torch.isfinite(rounded)).any().to(torch.int32) * _lib.FLAG_CACHE_OVERFLOW)
    elif not bool(torch.isfinite(rounded).all()):
        raise ValueError("F16 cache storage overflow")
    return value + (rounded - value).detach()


class _HeadPostFn(torch.autograd.Function):
    """Per (row, head) of ``d`` values: the head rms with ``weight`` (or none), the
    rotary of the row's position (or none) and the fp16 storage rounding with a
    straight-through gradient (or none), one kernel each way (``bd_head_post``)."""

    @staticmethod
    def forward(ctx, value, weight, positions, frequencies, epsilon, fp16, heads, dim):
        rows = value.shape[0]
        x = value.reshape(rows, heads * dim).float().contiguous()
        device = x.device
        w = None if weight is None else weight.detach().float().contiguous()
        out = torch.empty((rows, heads, dim), dtype=torch.float32, device=device)
        inv = torch.empty((rows, heads), dtype=torch.float32, device=device) if w is not None else None
        flags, now = _flags(device)
        _lib.call("bd_head_post", x.data_ptr(), heads * dim, rows, heads, dim, None if w is None else w.data_ptr(),
                  float(epsilon), None if positions is None else positions.data_ptr(),
                  None if frequencies is None else frequencies.data_ptr(), int(fp16), out.data_ptr(),
                  None if inv is None else inv.data_ptr(), flags.ptr, _stream(device))
        if now:
            flags.check()
        ctx.save_for_backward(x, w, inv, positions, frequencies)
        ctx.sizes = (rows, heads, dim, value.shape)
        return out

    @staticmethod
    def backward(ctx, grad):
        x, w, inv, positions, frequencies = ctx.saved_tensors
        rows, heads, dim, shape = ctx.sizes
        device = x.device
        g = grad.reshape(rows, heads, dim).float().contiguous()
        if w is None and positions is None:  # the fp16 rounding alone: straight through
            return g.view(shape), None, None, None, None, None, None, None
        dx = torch.empty_like(x)
        parts = dw = None
        if w is not None:
            parts = torch.empty((_lib.size("bd_head_post_partials", rows, heads), dim), dtype=torch.float32,
                                device=device)
            dw = torch.empty(dim, dtype=torch.float32, device=device)
        _lib.call("bd_head_post_backward", x.data_ptr(), heads * dim, rows, heads, dim,
                  None if w is None else w.data_ptr(), None if inv is None else inv.data_ptr(),
                  None if positions is None else positions.data_ptr(),
                  None if frequencies is None else frequencies.data_ptr(), g.data_ptr(), dx.data_ptr(),
                  None if parts is None else parts.data_ptr(), None if dw is None else dw.data_ptr(),
                  _stream(device), kernels=1 if w is None else 2)
        return dx.view(shape), dw, None, None, None, None, None, None


def head_post(value: Tensor, heads: int, dim: int, weight: Tensor | None, epsilon: float,
              positions: Tensor | None, theta: float, fp16: bool) -> Tensor:
    """``[rows, heads * dim]`` -> ``[rows, heads, dim]``: ``rms`` with ``weight`` per head, then
    ``rope`` at ``positions``, then ``cache_storage`` when ``fp16`` (each step optional),
    as ``Layer.forward`` applies them to queries, keys and values (``model.py:196-218``)."""
    rows = value.shape[0]
    if not value.is_cuda:
        out = value.reshape(rows, heads, dim)
        if weight is not None:
            out = rms(out, weight, epsilon)
        if positions is not None:
            out = rope(out, positions, theta)
        return cache_storage(out) if fp16 else out
    frequencies = None
    if positions is not None:
        positions = positions.to(torch.int64).contiguous()
        frequencies = _frequencies(dim, theta, value.device)
    return _HeadPostFn.apply(value, weight, positions, frequencies, epsilon, fp16, heads, dim)


def _ids_valid(values: tuple, limit: int) -> bool:
    """Every value an ``int`` (not a ``bool``) in ``[0, limit)``, in C-level passes
    over the tuple (a per-item Python test costs milliseconds at 2048 tokens)."""
    return not values or (set(map(type, values)) == {int} and min(values) >= 0 and max(values) < limit)


def _to_device(values: list[int], device: torch.device) -> Tensor:
    """A small int64 tensor on ``device`` without a host synchronisation (pinned copy)."""
    host = torch.tensor(values, dtype=torch.int64)
    if device.type != "cuda":
        return host.to(device)
    return host.pin_memory().to(device, non_blocking=True)


def _need_cuda(t: Tensor) -> torch.device:
    if not t.is_cuda:
        raise RuntimeError("bitdraft runs on CUDA tensors only (no CPU fallback)")
    return t.device


_stream = ops._stream


class deferred_checks:
    """Within this context the projections OR their device error bits into one
    flags word instead of reading them back after every launch (each read is a
    host synchronisation); leaving the context reads it once and raises the same
    ``ValueError`` / ``RuntimeError`` the immediate checks would have raised."""

    def __init__(self, device: torch.device) -> None:
        self.flags = ops.Flags(device)

    def __enter__(self) -> "deferred_checks":
        _DEFERRED.append(self.flags)
        return self

    def __exit__(self, *exc) -> None:
        _DEFERRED.remove(self.flags)
        if exc[0] is None:
            self.flags.check()


def _flags(device: torch.device) -> tuple[ops.Flags, bool]:
    """The flags word to use and whether to check it right away."""
    if _DEFERRED and _DEFERRED[-1].tensor.device == device:
        return _DEFERRED[-1], False
    return ops.Flags(device), True


def _bump(t: Tensor) -> None:
    """Mark a tensor written by a kernel (raw pointer) as modified for autograd and caches."""
    torch.autograd.graph.increment_version(t)


class _Sign(torch.autograd.Function):
    """``SIGN`` (``model.py:66-73``): +-1 forward, ``grad * 1[|w| <= 1]`` backward, both kernels."""

    @staticmethod
    def forward(ctx, value: Tensor) -> Tensor:
        device = _need_cuda(value)
        x = value.contiguous()
        out = torch.empty_like(x)
        flags = ops.Flags(device)
        _lib.call("bd_sign_rows", x.data_ptr(), x.numel(), None, out.data_ptr(), flags.ptr, _stream(device))
        ctx.save_for_backward(x)
        return out.view_as(value)

    @staticmethod
    def backward(ctx, grad: Tensor):
        (x,) = ctx.saved_tensors
        g = grad.contiguous().float()
        out = torch.empty_like(x)
        _lib.call("bd_ste_sign_backward", g.data_ptr(), None, x.data_ptr(), x.numel(), 1.0, None, 0,
                  out.data_ptr(), None, _stream(x.device))
        return out.view_as(grad)


def hard_sign(value: Tensor) -> Tensor:
    """``+1`` where ``value >= 0`` else ``-1``, straight-through (``model.py:92-95``)."""
    if value.dtype != torch.float32:
        raise ValueError("latent signs must be F32")
    return _Sign.apply(value)


def _round8(n: int) -> int:
    return (n + 7) // 8 * 8


def _split(value: Tensor, transpose: bool = False) -> tuple[Tensor, Tensor, int]:
    """fp32 ``value [rows, cols]`` as bf16 halves ``hi + lo`` (``bd_split_bf16``), row
    stride a multiple of 8 (transposed: ``[cols, ld]``).  Returns ``(hi, lo, ld)``."""
    v = value.reshape(-1, value.shape[-1]).float().contiguous()
    rows, cols = v.shape
    ld = _round8(rows if transpose else cols)
    shape = (cols, ld) if transpose else (rows, ld)
    hi = torch.empty(shape, dtype=torch.bfloat16, device=v.device)
    lo = torch.empty_like(hi)
    _lib.call("bd_split_bf16", v.data_ptr(), rows, cols, cols, int(transpose), hi.data_ptr(), lo.data_ptr(), ld,
              _stream(v.device))
    return hi, lo, ld


class _FrozenOperand:
    """bf16 hi + lo halves of a frozen fp32 operand ``[out, in]`` (and, for the input
    gradient, of its transpose), made once; the buffer itself is never replaced
    or written.  ``lo`` is None when the operand is exactly representable in
    bf16 (the drafter's bf16 checkpoints)."""

    def __init__(self, operand: Tensor) -> None:
        self.source = operand
        self.version = operand._version
        self.hi, lo, self.ld = _split(operand.detach())
        self.lo = lo if bool(lo.any()) else None
        self._t: tuple[Tensor, Tensor | None, int] | None = None

    def transposed(self) -> tuple[Tensor, Tensor | None, int]:
        if self._t is None:
            hi, lo, ld = _split(self.source.detach(), transpose=True)
            self._t = (hi, lo if self.lo is not None else None, ld)
        return self._t

    def valid_for(self, operand: Tensor) -> bool:
        return self.source is operand and self.version == operand._version


def _frozen_halves(owner, operand: Tensor) -> _FrozenOperand:
    cache = owner.__dict__.get("_halves")
    if cache is None or not cache.valid_for(operand):
        cache = _FrozenOperand(operand)
        owner.__dict__["_halves"] = cache
    return cache


def _split_workspace(device: torch.device, m: int, n: int, k: int, parts: int) -> tuple[int | None, int]:
    """The split-K workspace of a bf16 split product (one per device, used in stream
    order), or (None, 0) when the shape runs unsplit."""
    nbytes = _lib.size("bd_gemm_split_workspace_bytes", m, n, k, parts)
    if nbytes == 0:
        return None, 0
    buf = ops.workspace(device, "gemm_split", nbytes)
    return buf.data_ptr(), buf.numel()


def _product(x: Tensor, b_hi: Tensor, b_lo: Tensor | None, ld_b: int, n: int) -> Tensor:
    """``x [m, k] @ (b_hi + b_lo)^T`` at fp32 accuracy on the tcgen05 tensor cores:
    ``x`` split into bf16 halves, ``b`` given as halves ``[n, ld_b]``
    (``bd_gemm_bf16_split3``: hi.hi + lo.hi + hi.lo, lo.lo left out)."""
    m, k = x.shape
    x_hi, x_lo, ld = _split(x)
    if ld != ld_b:
        raise ValueError("operand strides differ")
    out = torch.empty((m, n), dtype=torch.float32, device=x.device)
    ws, nbytes = _split_workspace(x.device, m, n, k, 2 if b_lo is None else 3)
    _lib.call("bd_gemm_bf16_split3", x_hi.data_ptr(), x_lo.data_ptr(), m, k, ld, b_hi.data_ptr(),
              None if b_lo is None else b_lo.data_ptr(), n, ld_b, out.data_ptr(), n, ws, nbytes, _stream(x.device))
    return out


class _FrozenLinearFn(torch.autograd.Function):
    """``linear(value, operand)`` of a frozen fp32 operand on the tcgen05 tensor
    cores (split-bf16 halves), forward and input gradient (the operand gets no
    gradient)."""

    @staticmethod
    def forward(ctx, value, operand, halves):
        x = value.reshape(-1, value.shape[-1]).float()
        y = _product(x, halves.hi, halves.lo, halves.ld, operand.shape[0])
        ctx.halves = halves
        ctx.in_shape = value.shape
        return y.reshape(*value.shape[:-1], operand.shape[0])

    @staticmethod
    def backward(ctx, grad):
        g = grad.reshape(-1, grad.shape[-1]).float()
        hi_t, lo_t, ld_t = ctx.halves.transposed()
        dx = _product(g, hi_t, lo_t, ld_t, ctx.in_shape[-1])
        return dx.reshape(ctx.in_shape), None, None


def frozen_linear(value: Tensor, operand: Tensor, owner) -> Tensor:
    """``functional.linear(value, operand)`` for a frozen operand held by ``owner``
    (its bf16 halves are cached on the owner, outside its parameters and buffers).

    CUDA tensors take the split-bf16 tcgen05 GEMMs.  CPU tensors (host-side
    checks of the loss head's bookkeeping; no kernel of this package runs on
    them, and the binary projections refuse them) get the reference's own fp32
    ``linear``."""
    if not value.is_cuda:
        return functional.linear(value, operand)
    return _FrozenLinearFn.apply(value, operand, _frozen_halves(owner, operand))


class FrozenLinear(nn.Module):
    """A frozen dense projection; the operand is a buffer (``model.py:105-113``).
    On the GPU the product runs on the tcgen05 tensor cores with split-bf16
    operands (``_product``), within ~1e-5 of the fp32 product."""

    operand: Tensor

    def __init__(self, weight: Tensor) -> None:
        super().__init__()
        self.register_buffer("operand", weight.detach().float().clone())

    def forward(self, value: Tensor) -> Tensor:
        return frozen_linear(value, self.operand, self)


# --------------------------------------------------------------------------- binary projection


class _ProjectionFn(torch.autograd.Function):
    """Forward value and straight-through gradients of ``Projection.forward``
    (``model.py:128-150``), every product on the tcgen05 tensor cores:

    * forward: int8 codes (``bd_quantize_rows_i8``) times the +-1 int8 signs,
      ``kind::i8`` with exact s32 accumulators and the HE4 epilogue in the TMEM
      drain (``bd_projection_he4_tc``), bit-identical to the reference's fp32
      ``linear`` of integers;
    * backward: ``dL = G * scale`` as bf16 hi + lo halves (``bd_ste_grad_prep``),
      the input-side product ``dL . signs`` (``bd_gemm_bf16_split``) into the
      quantizer's straight-through backward (``bd_ste_input_backward``), and the
      latent gradient ``dL^T . codes`` with the step scale and the clip-window
      mask of ``SIGN`` (``model.py:71-73``) in the GEMM's epilogue
      (``bd_ste_weight_grad``), which also sums the gradient of a learned window.
    """

    @staticmethod
    def forward(ctx, value, latent, scale, midpoint, log_gain, log_clip, log_window, module):
        device = _need_cuda(value)
        x = value.reshape(-1, value.shape[-1]).float().contiguous()
        tokens, inner = x.shape
        outer = latent.shape[0]
        bits = module.bits
        gain = log_gain.detach().exp().contiguous()
        bound = log_clip.detach().exp().reshape(1).contiguous()
        stream = _stream(device)
        flags, now = _flags(device)
        ld = _lib.size("bd_i8_ld", inner)
        codes = torch.empty((tokens, ld), dtype=torch.int8, device=device)
        sums = torch.empty(tokens, dtype=torch.int32, device=device)
        _lib.call("bd_quantize_rows_i8", x.data_ptr(), tokens, inner, gain.data_ptr(), bound.data_ptr(), bits,
                  codes.data_ptr(), ld, sums.data_ptr(), flags.ptr, stream)
        if now:
            flags.check()
        signs = module.signs_i8()
        y = torch.empty((tokens, outer), dtype=torch.float32, device=device)
        dot = torch.empty((tokens, outer), dtype=torch.float32, device=device)
        _lib.call("bd_projection_he4_tc", codes.data_ptr(), ld, sums.data_ptr(), tokens, inner, signs.data_ptr(), outer,
                  scale.detach().contiguous().data_ptr(), midpoint.detach().contiguous().data_ptr(), bound.data_ptr(),
                  bits, None, y.data_ptr(), dot.data_ptr(), flags.ptr, stream)
        if now:
            flags.check()
        window = None if log_window is None else log_window.detach().exp().reshape(1).contiguous()
        ctx.module = module
        ctx.value_shape = value.shape
        ctx.ld = ld
        ctx.learned = log_window is not None
        ctx.save_for_backward(x, latent, scale, midpoint, gain, bound, dot, codes, sums, window)
        return y.view(*value.shape[:-1], outer)

    @staticmethod
    def backward(ctx, grad_out):
        x, latent, scale, midpoint, gain, bound, dot, codes, sums, window = ctx.saved_tensors
        module = ctx.module
        device = x.device
        stream = _stream(device)
        tokens, inner = x.shape
        outer = latent.shape[0]
        bits = module.bits
        need = ctx.needs_input_grad
        need_latent = need[1] or (ctx.learned and need[6])
        # inside a LatentGradients context the latent-side operands go to its buffers
        acc = next((a for a in reversed(_LATENT) if a.owns(module)), None) if need_latent else None
        g = grad_out.reshape(tokens, outer).float().contiguous()
        ld_o, ld_t = _round8(outer), _round8(tokens)
        hi = torch.empty((tokens, ld_o), dtype=torch.bfloat16, device=device)
        lo = torch.empty_like(hi)
        hi_t = lo_t = None
        t_hi = t_lo = t_codes = None
        if acc is not None:
            t_hi, t_lo, t_codes, ld_t = acc.columns(module, tokens, latent, bound, window)
        elif need_latent:
            hi_t = torch.empty((outer, ld_t), dtype=torch.bfloat16, device=device)
            lo_t = torch.empty_like(hi_t)
            t_hi, t_lo = hi_t.data_ptr(), lo_t.data_ptr()
        d_scale = torch.empty(outer, dtype=torch.float32, device=device)
        d_mid = torch.empty_like(d_scale)
        gm = torch.empty(tokens, dtype=torch.float32, device=device)
        nbytes = _lib.size("bd_ste_workspace_bytes", tokens, outer, inner)
        ws = ops.workspace(device, "ste", nbytes)
        sc, mid = scale.detach().contiguous(), midpoint.detach().contiguous()
        _lib.call("bd_ste_grad_prep", g.data_ptr(), dot.data_ptr(), tokens, outer, sc.data_ptr(), mid.data_ptr(),
                  bound.data_ptr(), bits, sums.data_ptr(), hi.data_ptr(), lo.data_ptr(), ld_o, t_hi, t_lo, ld_t,
                  d_scale.data_ptr(), d_mid.data_ptr(), gm.data_ptr(), ws.data_ptr(), ws.numel(), stream)
        dx = d_gain = d_clip = d_latent = d_window = None
        if need[0] or need[4] or need[5]:
            signs_t = module.signs_t_bf16(ld_o)
            dv = torch.empty((tokens, inner), dtype=torch.float32, device=device)
            sws, snb = _split_workspace(device, tokens, inner, outer, 2)
            _lib.call("bd_gemm_bf16_split", hi.data_ptr(), lo.data_ptr(), tokens, outer, ld_o, signs_t.data_ptr(),
                      inner, ld_o, dv.data_ptr(), inner, sws, snb, stream)
            dx = torch.empty_like(x)
            d_gain = torch.empty(inner, dtype=torch.float32, device=device)
            d_clip = torch.empty(1, dtype=torch.float32, device=device)
            _lib.call("bd_ste_input_backward", dv.data_ptr(), None, gm.data_ptr(), x.data_ptr(), tokens, inner,
                      gain.data_ptr(), bound.data_ptr(), bits, dx.data_ptr(), d_gain.data_ptr(), d_clip.data_ptr(), 0,
                      ws.data_ptr(), ws.numel(), stream)
            dx = dx.view(ctx.value_shape)
            d_clip = d_clip.reshape(())
        if acc is not None:
            _lib.call("bd_codes_transpose_bf16", codes.data_ptr(), tokens, inner, ctx.ld, t_codes, ld_t, stream)
        elif need_latent:
            codes_t = torch.empty((inner, ld_t), dtype=torch.bfloat16, device=device)
            _lib.call("bd_codes_transpose_bf16", codes.data_ptr(), tokens, inner, ctx.ld, codes_t.data_ptr(), ld_t,
                      stream)
            d_latent = torch.empty((outer, inner), dtype=torch.float32, device=device)
            partials = None
            if ctx.learned:
                partials = torch.empty(_lib.size("bd_ste_weight_grad_partials", outer, inner), dtype=torch.float32,
                                       device=device)
            flags, now = _flags(device)
            _lib.call("bd_ste_weight_grad", hi_t.data_ptr(), lo_t.data_ptr(), outer, tokens, ld_t, codes_t.data_ptr(),
                      inner, latent.detach().contiguous().data_ptr(),
                      None if window is None else window.data_ptr(), float(module.window), bound.data_ptr(), bits,
                      d_latent.data_ptr(), None if partials is None else partials.data_ptr(), flags.ptr, stream)
            if now:
                flags.check()
            if ctx.learned:
                # d/d(log window) = window * sum over |w| > window of the unmasked gradient * sign(w)
                d_window = (partials.view(-1, 2)[:, 1].sum() * window[0]).reshape(1)
        return (dx if need[0] else None, d_latent if need[1] else None, d_scale if need[2] else None,
                d_mid if need[3] else None, d_gain if need[4] else None, d_clip if need[5] else None,
                d_window if ctx.learned and need[6] else None, None)


class Projection(nn.Module):
    """HE4 binary projection (``model.py:116-150``) with the reference's parameters
    ``latent_sign``, ``scale``, ``midpoint``, ``log_gain``, ``log_clip``.

    ``window`` is the sign straight-through window: the reference's fixed 1.0
    (``model.py:71-73``), or, with ``learned_window=True``, the initial value of a
    learned clip ``|w| <= alpha`` held as the parameter ``log_window`` (``alpha =
    exp(log_window)``); its gradient is the sum over the latents outside the
    window of their straight-through gradient times ``sign(w)``, the weight-side
    counterpart of the learned activation clip of ``model.py:136-139``.  Packed
    and expanded signs are caches outside the module's parameters and buffers,
    keyed by the latent's version counter.
    """

    def __init__(self, weight: Tensor, bits: int, gain: nn.Parameter, clip: nn.Parameter,
                 window: float = 1.0, learned_window: bool = False) -> None:
        super().__init__()
        if bits not in (4, 8) or weight.ndim != 2 or not bool(torch.isfinite(weight).all()):
            raise ValueError("invalid HE4 projection")
        if not (math.isfinite(window) and window > 0):
            raise ValueError("the straight-through window must be positive and finite")
        self.bits = bits
        self.window = float(window)
        self.latent_sign = nn.Parameter(weight.detach().float().clone())
        self.scale = nn.Parameter(weight.detach().float().abs().mean(-1))
        self.midpoint = nn.Parameter(torch.zeros(weight.shape[0]))
        self.log_gain = gain
        self.log_clip = clip
        self.log_window = nn.Parameter(torch.tensor(math.log(window))) if learned_window else None
        self._signs: dict[str, tuple[tuple[int, int], Tensor]] = {}

    def _key(self) -> tuple[int, int]:
        return self.latent_sign.data_ptr(), self.latent_sign._version

    def signs_i8(self) -> Tensor:
        """+-1 int8 copy of the signs, rows padded to 128 (the tensor-core forward's
        operand; cached per latent version)."""
        key = self._key()
        hit = self._signs.get("i8")
        if hit is not None and hit[0] == key:
            return hit[1]
        latent = self.latent_sign.detach().contiguous()
        flags, now = _flags(latent.device)
        out = ops.tile_i8(latent, flags=flags)
        if now:
            flags.check()
        self._signs["i8"] = (key, out)
        return out

    def signs_t_bf16(self, ld: int) -> Tensor:
        """+-1 bf16 signs transposed ``[in][ld]`` (the input-gradient GEMM's operand;
        cached per latent version)."""
        key = self._key()
        hit = self._signs.get("t_bf16")
        if hit is not None and hit[0] == key and hit[1].shape[1] == ld:
            return hit[1]
        latent = self.latent_sign.detach().contiguous()
        device = _need_cuda(latent)
        rows, cols = latent.shape
        out = torch.empty((cols, ld), dtype=torch.bfloat16, device=device)
        flags, now = _flags(device)
        _lib.call("bd_sign_cols_bf16", latent.data_ptr(), rows, cols, out.data_ptr(), ld, flags.ptr, _stream(device))
        if now:
            flags.check()
        self._signs["t_bf16"] = (key, out)
        return out

    def signs_w8(self) -> Tensor:
        """W8 decode-layout sign words (cached per latent version)."""
        key = self._key()
        hit = self._signs.get("w8")
        if hit is not None and hit[0] == key:
            return hit[1]
        out = ops.tile_w8(self.latent_sign.detach().contiguous())
        self._signs["w8"] = (key, out)
        return out

    def adopt_w8(self, tiled: Tensor) -> None:
        """Install W8 words re-packed by the optimizer for the current latent version."""
        self._signs = {"w8": (self._key(), tiled)}

    def forward(self, value: Tensor) -> Tensor:
        return _ProjectionFn.apply(value, self.latent_sign, self.scale, self.midpoint, self.log_gain, self.log_clip,
                                   self.log_window, self)


def _projections(model: nn.Module):
    return [m for m in model.modules() if isinstance(m, Projection)]


def _add_grad(parameter: nn.Parameter, grad: Tensor) -> None:
    if parameter.grad is None:
        parameter.grad = grad
    else:
        parameter.grad.add_(grad)


class LatentGradients:
    """Gradient accumulation of the binary projections' latents over several
    backward passes (one update over many sequences) as one tensor-core product
    per projection.

    Inside ``with LatentGradients(model, rows):`` a projection's backward writes
    the transposed bf16 halves of its output gradient and its transposed codes
    side by side into per-projection buffers of ``rows`` columns instead of
    running its latent-gradient GEMM.  Leaving the context runs one
    ``bd_ste_weight_grad`` per projection over all the columns, so the
    clip-window mask, the fp32 latent read and the gradient write happen once
    per update instead of once per sequence, and no gradient is added between
    passes.  The product over the concatenated columns is the sum of the
    per-sequence products (the mask, the step scale and the window do not depend
    on the sequence), accumulated in fp32 by the tensor cores in one pass.

    A buffer that would overflow, or a latent that changed since the columns were
    written, is flushed first, so the result does not depend on ``rows``; ``rows``
    only sizes the buffers (the sum of the rows of the backward passes).  At a
    flush ``latent_sign.grad`` and ``log_window.grad`` are set or added to, and
    ``on_ready(parameter)`` is called for each, in module order (every rank flushes
    in the same order, so a data-parallel exchange issues the same collectives).
    Buffers are kept for the next use of the same object."""

    def __init__(self, model: nn.Module, rows: int, on_ready=None) -> None:
        if rows < 1:
            raise ValueError("rows must be positive")
        self.modules = _projections(model)
        self.rows = _round8(int(rows))
        self.on_ready = on_ready
        self._owned = {id(m) for m in self.modules}
        self._slots: dict[int, dict] = {}

    def __enter__(self) -> "LatentGradients":
        _LATENT.append(self)
        return self

    def __exit__(self, *exc) -> None:
        _LATENT.remove(self)
        if exc[0] is None:
            self.flush()
        else:
            for s in self._slots.values():
                s["filled"] = 0

    def owns(self, module: "Projection") -> bool:
        return id(module) in self._owned

    def columns(self, module: "Projection", tokens: int, latent: Tensor, bound: Tensor,
                window: Tensor | None) -> tuple[int, int, int, int]:
        """Device addresses of ``tokens`` free columns in the module's dL^T hi, dL^T lo
        and codes^T buffers, and the buffers' row stride (elements)."""
        width = _round8(tokens)
        key = (latent.data_ptr(), latent._version)
        s = self._slots.get(id(module))
        if s is not None and s["filled"] and (s["key"] != key or s["filled"] + width > s["cap"]):
            self._flush_one(module, s)
        if s is None or s["cap"] < width:
            cap = max(self.rows, width)
            outer, inner = latent.shape
            s = {"hi": torch.empty((outer, cap), dtype=torch.bfloat16, device=latent.device),
                 "codes": torch.empty((inner, cap), dtype=torch.bfloat16, device=latent.device),
                 "cap": cap, "filled": 0}
            s["lo"] = torch.empty_like(s["hi"])
            self._slots[id(module)] = s
        s["key"], s["bound"], s["window"] = key, bound, window
        off = s["filled"]
        s["filled"] = off + width
        if width != tokens:  # padding columns take part in the product: zero on both sides
            for name in ("hi", "lo", "codes"):
                s[name][:, off + tokens:off + width].zero_()
        return (s["hi"].data_ptr() + 2 * off, s["lo"].data_ptr() + 2 * off, s["codes"].data_ptr() + 2 * off,
                s["cap"])

    def _flush_one(self, module: "Projection", s: dict) -> None:
        filled, s["filled"] = s["filled"], 0
        if not filled:
            return
        latent = module.latent_sign
        outer, inner = latent.shape
        device = latent.device
        window = s["window"]
        learned = module.log_window is not None and window is not None
        partials = None
        if learned:
            partials = torch.empty(_lib.size("bd_ste_weight_grad_partials", outer, inner), dtype=torch.float32,
                                   device=device)
        d_latent = torch.empty((outer, inner), dtype=torch.float32, device=device)
        flags, now = _flags(device)
        _lib.call("bd_ste_weight_grad", s["hi"].data_ptr(), s["lo"].data_ptr(), outer, filled, s["cap"],
                  s["codes"].data_ptr(), inner, latent.detach().data_ptr(),
                  window.data_ptr() if learned else None, float(module.window), s["bound"].data_ptr(), module.bits,
                  d_latent.data_ptr(), None if partials is None else partials.data_ptr(), flags.ptr,
                  _stream(device))
        if now:
            flags.check()
        ready = []
        if latent.requires_grad:
            _add_grad(latent, d_latent)
            ready.append(latent)
        if learned and module.log_window.requires_grad:
            # d/d(log window) = window * sum over |w| > window of the unmasked gradient * sign(w)
            d_window = (partials.view(-1, 2)[:, 1].sum() * window[0]).reshape(module.log_window.shape)
            _add_grad(module.log_window, d_window)
            ready.append(module.log_window)
        if self.on_ready is not None:
            for p in ready:
                self.on_ready(p)

    def flush(self) -> None:
        """Run the pending latent-gradient products (module order)."""
        for module in self.modules:
            s = self._slots.get(id(module))
            if s is not None:
                self._flush_one(module, s)


def bound_latents(model: nn.Module, multiple: float) -> None:
    """``latent <- clamp(latent / (multiple * mean|row|), -1, 1)`` for every projection
    (``model.py:153-164``); refuses (before writing) a change of any sign."""
    with torch.no_grad():
        for module in _projections(model):
            latent = module.latent_sign
            device = _need_cuda(latent)
            out = torch.empty_like(latent)
            flags = ops.Flags(device)
            _lib.call("bd_bound_latents", latent.data_ptr(), latent.shape[0], latent.shape[1], float(multiple),
                      out.data_ptr(), flags.ptr, _stream(device))
            flags.check()
            latent.copy_(out)


def clamp_latents(model: nn.Module) -> None:
    """``latent.clamp_(-1, 1)`` for every projection (``model.py:167-169``)."""
    with torch.no_grad():
        for module in _projections(model):
            latent = module.latent_sign
            device = _need_cuda(latent)
            _lib.call("bd_clamp", latent.data_ptr(), latent.numel(), -1.0, 1.0, _stream(device))
            _bump(latent)


# --------------------------------------------------------------------------- layers


class _Stacked:
    """Several frozen operands stacked along their output rows, as one frozen
    operand (one split-bf16 GEMM computes all of them); rebuilt when any source
    buffer is replaced or written."""

    def __init__(self, operands: tuple[Tensor, ...]) -> None:
        self.key = tuple((id(o), o._version) for o in operands)
        self.operand = torch.cat([o.detach() for o in operands], 0)
        self.sizes = tuple(o.shape[0] for o in operands)


def _stacked(owner, name: str, operands: tuple[Tensor, ...]) -> _Stacked:
    cache = owner.__dict__.get(name)
    key = tuple((id(o), o._version) for o in operands)
    if cache is None or cache.key != key:
        cache = _Stacked(operands)
        owner.__dict__[name] = cache
    return cache


def _stacked_linear(value: Tensor, owner, name: str, operands: tuple[Tensor, ...]) -> tuple[Tensor, ...]:
    """``(linear(value, o) for o in operands)`` as one product of the stacked operands."""
    stack = _stacked(owner, name, operands)
    return frozen_linear(value, stack.operand, stack).split(stack.sizes, -1)


def _padded_dim(head_dim: int) -> int:
    for size in (16, 32, 64, 128):
        if head_dim <= size:
            return size
    raise ValueError("training attention supports head_dim up to 128")


class _TrainAttentionFn(torch.autograd.Function):
    """The windows' attention on the training-attention kernels
    (``bd_train_attention_forward`` / ``_backward``): fp16 tensor-core products with
    the fp32 operands as hi + lo halves, the row log-sum-exp saved for the backward.
    The operand layouts are made on the device (``bd_train_attention_pack``,
    ``bd_train_attention_pack_grad``)."""

    @staticmethod
    def forward(ctx, query, ctx_k, ctx_v, slot_k, slot_v, ctx_allowed, slot_allowed):
        windows, slots, kvh, groups, dim = query.shape
        length = ctx_k.shape[0]
        dp = _padded_dim(dim)
        device = query.device
        padded = (length + 63) // 64 * 64
        f16 = dict(dtype=torch.float16, device=device)
        q_hi = torch.empty((kvh, windows, groups, 16, dp), **f16)
        q_lo = torch.empty_like(q_hi)
        kc = torch.empty((kvh, padded, dp), **f16)
        vc = torch.empty_like(kc)
        ks = torch.empty((kvh, windows, 16, dp), **f16)
        vs = torch.empty_like(ks)
        ctx_mask = torch.empty((windows, 16, padded), dtype=torch.uint8, device=device)
        slot_mask = torch.empty((16, 16), dtype=torch.uint8, device=device)
        lse = torch.empty((kvh, windows, groups, 16), dtype=torch.float32, device=device)
        q = query.detach().float().contiguous()
        kk, vv = ctx_k.detach().float().contiguous(), ctx_v.detach().float().contiguous()
        sk, sv = slot_k.detach().float().contiguous(), slot_v.detach().float().contiguous()
        allowed = ctx_allowed.to(torch.bool).expand(windows, slots, length)
        slot_ok = None if slot_allowed is None else slot_allowed.to(torch.bool).expand(slots, slots)
        stream = _stream(device)
        _lib.call("bd_train_attention_pack", q.data_ptr(), kk.data_ptr() if length else None,
                  vv.data_ptr() if length else None, sk.data_ptr(), sv.data_ptr(),
                  allowed.data_ptr() if length else None, *allowed.stride(),
                  None if slot_ok is None else slot_ok.data_ptr(), *((0, 0) if slot_ok is None else slot_ok.stride()),
                  windows, slots, kvh, groups, dim, length, q_hi.data_ptr(), q_lo.data_ptr(),
                  kc.data_ptr() if length else None, vc.data_ptr() if length else None, ks.data_ptr(), vs.data_ptr(),
                  ctx_mask.data_ptr() if length else None, slot_mask.data_ptr(), lse.data_ptr(), stream,
                  kernels=4 if length else 3)
        out = torch.empty((windows, slots, kvh, groups, dim), dtype=torch.float32, device=device)
        live = torch.empty((windows, padded // 64 + 1), dtype=torch.uint8, device=device)
        scale = 1.0 / math.sqrt(dim)
        _lib.call("bd_train_attention_forward", q_hi.data_ptr(), q_lo.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                  ks.data_ptr(), vs.data_ptr(), ctx_mask.data_ptr(), slot_mask.data_ptr(), windows, slots, kvh, groups,
                  dim, length, scale, out.data_ptr(), lse.data_ptr(), live.data_ptr(), stream)
        ctx.save_for_backward(q_hi, q_lo, kc, vc, ks, vs, ctx_mask, slot_mask, out, lse, live)
        ctx.sizes = (windows, slots, kvh, groups, dim, length, dp, scale)
        return out

    @staticmethod
    def backward(ctx, grad):
        q_hi, q_lo, kc, vc, ks, vs, ctx_mask, slot_mask, out, lse, live = ctx.saved_tensors
        windows, slots, kvh, groups, dim, length, dp, scale = ctx.sizes
        device = out.device
        stream = _stream(device)
        grad = grad.float().contiguous()
        # the output gradient times a power of two with its largest magnitude in
        # (1/2, 1], so that its fp16 halves keep their precision; undone exactly
        # on the results (scalars: the maximum, the factor, its inverse)
        d_hi = torch.empty_like(q_hi)
        d_lo = torch.empty_like(q_hi)
        dr = torch.empty((kvh, windows, groups, 16), dtype=torch.float32, device=device)
        scalars = torch.empty(4, dtype=torch.float32, device=device)
        _lib.call("bd_train_attention_pack_grad", grad.data_ptr(), out.data_ptr(), windows, slots, kvh, groups, dim,
                  d_hi.data_ptr(), d_lo.data_ptr(), dr.data_ptr(), scalars.data_ptr(), stream, kernels=4)
        dq = torch.empty_like(out)
        dkc = torch.empty((length, kvh, dim), dtype=torch.float32, device=device)
        dvc = torch.empty_like(dkc)
        dks = torch.empty((windows, slots, kvh, dim), dtype=torch.float32, device=device)
        dvs = torch.empty_like(dks)
        parts = torch.empty((8, length, kvh, dim), dtype=torch.float32, device=device) if length else None
        _lib.call("bd_train_attention_backward", q_hi.data_ptr(), q_lo.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                  ks.data_ptr(), vs.data_ptr(), ctx_mask.data_ptr(), slot_mask.data_ptr(), d_hi.data_ptr(),
                  d_lo.data_ptr(), lse.data_ptr(), dr.data_ptr(), scalars[2:].data_ptr(), live.data_ptr(), windows,
                  slots, kvh, groups, dim, length, scale, dq.data_ptr(), dkc.data_ptr() if length else None,
                  dvc.data_ptr() if length else None, dks.data_ptr(), dvs.data_ptr(),
                  parts.data_ptr() if length else None, stream, kernels=3 if length else 2)
        return dq, dkc, dvc, dks, dvs, None, None


def train_attention(query: Tensor, ctx_k: Tensor, ctx_v: Tensor, slot_k: Tensor, slot_v: Tensor,
                    ctx_allowed: Tensor, slot_allowed: Tensor | None) -> Tensor:
    """Block attention of ``group`` on the GPU kernels: ``query [W, k, kvh, g, d]``,
    ``ctx_k/ctx_v [L, kvh, d]`` and ``slot_k/slot_v [W, k, kvh, d]`` holding fp16
    values (``cache_storage``), ``ctx_allowed`` broadcastable to ``[W, k, L]``,
    ``slot_allowed [k, k]`` or None.  Returns ``[W, k, kvh, g, d]``."""
    slots, groups = query.shape[1], query.shape[3]
    if slots > 16 or groups > 4:
        raise ValueError("training attention supports up to 16 slots and 4 query heads per kv head")
    _padded_dim(query.shape[-1])
    return _TrainAttentionFn.apply(query, ctx_k, ctx_v, slot_k, slot_v, ctx_allowed, slot_allowed)


def _window_attention(query: Tensor, ctx_k: Tensor, ctx_v: Tensor, slot_k: Tensor, slot_v: Tensor,
                      ctx_allowed: Tensor, slot_allowed: Tensor | None, head_dim: int) -> Tensor:
    """Grouped-query attention of a block of windows: ``query [W, k, kvh, g, d]`` over the
    shared context ``ctx_k/ctx_v [L, kvh, d]`` (rows allowed by ``ctx_allowed
    [W, k, L]``) and each window's own slots ``slot_k/slot_v [W, k, kvh, d]``
    (``slot_allowed [k, k]`` or all; both masks broadcast), one softmax over both parts.  Returns
    ``[W * k, kvh * g * d]``.  CUDA tensors run the training-attention kernels; CPU
    tensors the reference's eager expression."""
    windows, slots = query.shape[:2]
    if query.is_cuda:
        return train_attention(query, ctx_k, ctx_v, slot_k, slot_v, ctx_allowed, slot_allowed).reshape(
            windows * slots, -1)
    scale = 1.0 / math.sqrt(head_dim)
    logits = torch.cat((torch.einsum("wshgd,lhd->whgsl", query, ctx_k),
                        torch.einsum("wshgd,wthd->whgst", query, slot_k)), -1) * scale
    length = ctx_k.shape[0]
    ctx_mask = ctx_allowed.expand(windows, slots, length)[:, None, None]
    if slot_allowed is None:
        slot_mask = torch.ones((windows, 1, 1, slots, slots), dtype=torch.bool, device=query.device)
    else:
        slot_mask = slot_allowed.expand(slots, slots)[None, None, None].expand(windows, 1, 1, slots, slots)
    mask = torch.cat((ctx_mask, slot_mask), -1)
    weights = functional.softmax(logits.masked_fill(~mask, -torch.inf), -1)
    ctx_w, slot_w = weights.split((ctx_k.shape[0], slots), -1)
    out = torch.einsum("whgsl,lhd->wshgd", ctx_w, ctx_v) + torch.einsum("whgst,wthd->wshgd", slot_w, slot_v)
    return out.reshape(windows * slots, -1)


class Layer(nn.Module):
    """One drafter block (``model.py:172-274``): attention over cached context plus
    the block's slots, then the binary SwiGLU ``down(silu(gate(n)) * up(n))``.

    The context keys and values of a block come from one stacked frozen product
    (``k|v``), the slots' queries, keys and values from another (``q|k|v``);
    the single-window ``forward`` is the window-block ``group`` with one window."""

    def __init__(self, tensors: dict[str, Tensor], prefix: str, geometry: Geometry, window: float = 1.0,
                 learned_window: bool = False) -> None:
        super().__init__()
        self.geometry = geometry
        self.attn_norm = nn.Parameter(tensors[prefix + "attn_norm.weight"].clone())
        self.q_norm = nn.Parameter(tensors[prefix + "attn_q_norm.weight"].clone())
        self.k_norm = nn.Parameter(tensors[prefix + "attn_k_norm.weight"].clone())
        self.ffn_norm = nn.Parameter(tensors[prefix + "ffn_norm.weight"].clone())
        self.query = FrozenLinear(tensors[prefix + "attn_q.weight"])
        self.key = FrozenLinear(tensors[prefix + "attn_k.weight"])
        self.value = FrozenLinear(tensors[prefix + "attn_v.weight"])
        self.output = FrozenLinear(tensors[prefix + "attn_output.weight"])
        gain = nn.Parameter(torch.zeros(geometry.hidden))
        clip = nn.Parameter(torch.tensor(0.0))
        straight = dict(window=window, learned_window=learned_window)
        self.gate = Projection(tensors[prefix + "ffn_gate.weight"], 4, gain, clip, **straight)
        self.up = Projection(tensors[prefix + "ffn_up.weight"], 4, gain, clip, **straight)
        self.down = Projection(tensors[prefix + "ffn_down.weight"], 8, nn.Parameter(torch.zeros(geometry.intermediate)),
                               nn.Parameter(torch.tensor(0.0)), **straight)
        self._packed: tuple[tuple, ops.PackedFFN] | None = None

    def _heads(self, flat: Tensor, heads: int) -> Tensor:
        return flat.reshape(-1, heads, self.geometry.head_dim)

    def _keys(self, key: Tensor, positions: Tensor) -> Tensor:
        """Head rms, rotary, fp16 storage of raw keys ``[n, kvh, d]`` (``model.py:196-200, 211-213``)."""
        cfg = self.geometry
        return head_post(key.reshape(key.shape[0], -1), cfg.kv_heads, cfg.head_dim, self.k_norm, cfg.epsilon, positions,
                         cfg.theta, True)

    def context(self, encoded: Tensor, positions: Tensor) -> tuple[Tensor, Tensor]:
        """Context keys (normed, rotated) and values through fp16 storage (``model.py:195-200``)."""
        cfg = self.geometry
        key, value = _stacked_linear(encoded, self, "_kv", (self.key.operand, self.value.operand))
        return self._keys(key, positions), head_post(value, cfg.kv_heads, cfg.head_dim, None, 0.0, None, 0.0, True)

    def packed_ffn(self) -> ops.PackedFFN:
        """The SwiGLU operands in the fused decode block's layout (cached per parameter versions)."""
        params = (self.gate.latent_sign, self.up.latent_sign, self.down.latent_sign, self.gate.scale, self.up.scale,
                  self.down.scale, self.gate.midpoint, self.up.midpoint, self.down.midpoint, self.gate.log_gain,
                  self.gate.log_clip, self.down.log_gain, self.down.log_clip)
        key = tuple((p.data_ptr(), p._version) for p in params)
        if self._packed is not None and self._packed[0] == key:
            return self._packed[1]
        with torch.no_grad():
            gate, up, down = (p.latent_sign.detach().contiguous() for p in (self.gate, self.up, self.down))
            flags = ops.Flags(gate.device)
            packed = ops.PackedFFN(
                hidden=gate.shape[1], inter=gate.shape[0], signs_gate_up=ops.tile_gate_up_w8(gate, up, flags),
                signs_down=self.down.signs_w8(), signs_down_d8=ops.tile_d8(down, flags),
                scale_gate=self.gate.scale.detach().contiguous(),
                scale_up=self.up.scale.detach().contiguous(), scale_down=self.down.scale.detach().contiguous(),
                midpoint_gate=self.gate.midpoint.detach().contiguous(),
                midpoint_up=self.up.midpoint.detach().contiguous(),
                midpoint_down=self.down.midpoint.detach().contiguous(),
                gain_gate_up=self.gate.log_gain.detach().exp().contiguous(),
                bound_gate_up=self.gate.log_clip.detach().exp().reshape(1).contiguous(),
                gain_down=self.down.log_gain.detach().exp().contiguous(),
                bound_down=self.down.log_clip.detach().exp().reshape(1).contiguous())
            flags.check()
        self._packed = (key, packed)
        return packed

    def feed_forward(self, residual: Tensor) -> Tensor:
        """``residual + down(silu(gate(n)) * up(n))``, ``n = rms(residual, ffn_norm)`` (``model.py:220-223``)."""
        cfg = self.geometry
        rows = residual.reshape(-1, residual.shape[-1])
        grad = torch.is_grad_enabled() and any(p.requires_grad for p in self.parameters())
        if not grad and not residual.requires_grad and rows.shape[0] <= MAX_DECODE_ROWS:
            x = rows.float().contiguous()
            norm = self.ffn_norm.detach().float().contiguous()
            y = ops.ffn_he4(x, self.packed_ffn(), residual=x, norm=norm, epsilon=cfg.epsilon)
            return y.view_as(residual)
        norm = rms(residual, self.ffn_norm, cfg.epsilon)
        return residual + self.down.forward(functional.silu(self.gate.forward(norm)) * self.up.forward(norm))

    def forward(self, state: Tensor, context: tuple[Tensor, Tensor], positions: Tensor, allowed: Tensor) -> Tensor:
        """One block over a single window's slots (``model.py:202-223``): ``allowed
        [k, L + k]`` over the context keys and then the slots."""
        length = context[0].shape[0]
        return self.group(state, context, positions[None], allowed[None, :, :length], allowed[:, length:])

    def group(self, state: Tensor, context: tuple[Tensor, Tensor], positions: Tensor, allowed: Tensor,
              slot_allowed: Tensor | None) -> Tensor:
        """Several windows at once (``model.py:225-274``): ``positions [W, k]``, the shared
        context of length L, ``allowed [W, k, L]``, ``slot_allowed [k, k]`` or None."""
        cfg = self.geometry
        windows, slots = positions.shape
        groups = cfg.heads // cfg.kv_heads
        norm = rms(state, self.attn_norm, cfg.epsilon)
        query, key, value = _stacked_linear(norm, self, "_qkv",
                                            (self.query.operand, self.key.operand, self.value.operand))
        flat = positions.reshape(-1)
        query = head_post(query, cfg.heads, cfg.head_dim, self.q_norm, cfg.epsilon, flat, cfg.theta, False)
        key = self._keys(self._heads(key, cfg.kv_heads), flat)
        value = head_post(value, cfg.kv_heads, cfg.head_dim, None, 0.0, None, 0.0, True)
        attended = _window_attention(
            query.view(windows, slots, cfg.kv_heads, groups, cfg.head_dim), context[0], context[1],
            key.view(windows, slots, cfg.kv_heads, cfg.head_dim), value.view(windows, slots, cfg.kv_heads, cfg.head_dim),
            allowed, slot_allowed, cfg.head_dim)
        return self.feed_forward(state.reshape(windows * slots, -1) + self.output.forward(attended))


class HE4(nn.Module):
    """The block drafter (``model.py:277-396``): fused target features, ``layers``
    blocks, tied vocabulary head.  ``window`` / ``learned_window`` set the
    straight-through window of every binary projection (the reference's fixed
    1.0 by default; see ``Projection``)."""

    vocabulary: Tensor

    def __init__(self, tensors: dict[str, Tensor], vocabulary: Tensor, mask: int,
                 geometry: Geometry = Geometry(), window: float = 1.0, learned_window: bool = False) -> None:
        super().__init__()
        self.geometry = geometry
        self.mask = mask
        self.origin: tuple[str, str] | None = None
        self.native_codes: tuple[tuple[str, tuple[int, ...], bytes], ...] = ()
        if (vocabulary.ndim != 2 or vocabulary.shape[1] != geometry.hidden or type(mask) is not int
                or not 0 <= mask < vocabulary.shape[0] or not bool(torch.isfinite(vocabulary).all())):
            raise ValueError("invalid frozen vocabulary geometry or mask")
        self.register_buffer("vocabulary", vocabulary.detach().float().clone())
        self.fusion = FrozenLinear(tensors["fc.weight"])
        self.encoder_norm = nn.Parameter(tensors["enc.output_norm.weight"].clone())
        self.output_norm = nn.Parameter(tensors["output_norm.weight"].clone())
        self.blocks = nn.ModuleList([Layer(tensors, f"blk.{i}.", geometry, window, learned_window)
                                     for i in range(geometry.layers)])

    def check(self, features: Tensor, tokens: tuple[int, ...], anchors: tuple[int, ...]) -> None:
        cfg = self.geometry
        if (not anchors or not _ids_valid(anchors, len(tokens))
                or features.ndim != 2 or features.dtype not in (torch.float16, torch.float32)
                or features.shape != (len(tokens), cfg.taps * cfg.hidden)
                or not _ids_valid(tokens, self.vocabulary.shape[0])):
            raise ValueError("invalid model inputs")

    def block(self, slots: int | None) -> int:
        size = self.geometry.slots if slots is None else slots
        if type(size) is not int or not 1 <= size <= self.geometry.slots:
            raise ValueError("block size must be between one slot and the model's slots")
        return size

    def _encode(self, features: Tensor, length: int) -> Tensor:
        """Fused, normalised target features of the first ``length`` positions (``model.py:349-351``)."""
        fused = self.fusion.forward(features[:length].to(self.vocabulary.device).float())
        return rms(fused, self.encoder_norm, self.geometry.epsilon)

    def _contexts(self, encoded: Tensor, positions: Tensor) -> list[tuple[Tensor, Tensor]]:
        """Every layer's context keys and values (``Layer.context``), all layers' k|v rows
        as one stacked frozen product of the encoded context."""
        cfg = self.geometry
        operands = tuple(o for b in self.blocks for o in (b.key.operand, b.value.operand))
        parts = _stacked_linear(encoded, self, "_context_kv", operands)
        out = []
        for index, block in enumerate(self.blocks):
            key, value = parts[2 * index], parts[2 * index + 1]
            out.append((block._keys(key, positions),
                        head_post(value, cfg.kv_heads, cfg.head_dim, None, 0.0, None, 0.0, True)))
        return out

    def group_hidden(self, features: Tensor, tokens: tuple[int, ...], anchors: tuple[int, ...],
                     slots: int | None = None) -> Tensor:
        """Hidden states ``[W, k, hidden]`` of several windows (``model.py:329-367``): each
        window is its anchor token then ``k - 1`` mask slots at positions anchor ..
        anchor + k - 1, attending to the context before its anchor (and, except in
        the last layer, within the sliding window) and to its own slots."""
        self.check(features, tokens, anchors)
        cfg = self.geometry
        size = self.block(slots)
        device = self.vocabulary.device
        windows = len(anchors)
        first = _to_device([tokens[a] for a in anchors], device)
        ids = torch.cat((first[:, None], torch.full((windows, size - 1), self.mask, device=device)), 1)
        state = functional.embedding(ids.reshape(-1), self.vocabulary)
        start = _to_device(list(anchors), device)
        offset = torch.arange(size, device=device)
        positions = start[:, None] + offset[None, :]
        length = max(anchors)
        keys = torch.arange(length, device=device)
        visible = keys[None, None, :] < start[:, None, None]
        near = (positions[:, :, None] - keys[None, None, :]).abs() < cfg.window
        slot_near = (offset[:, None] - offset[None, :]).abs() < cfg.window
        contexts = self._contexts(self._encode(features, length), keys)
        for index, block in enumerate(self.blocks):
            last = index == cfg.layers - 1
            state = block.group(state, contexts[index], positions, visible if last else visible & near,
                                None if last else slot_near)
        return rms(state, self.output_norm, cfg.epsilon).view(windows, size, cfg.hidden)

    def forward(self, features: Tensor, tokens: tuple[int, ...], anchor: int, slots: int | None = None) -> Tensor:
        """Logits ``[k, vocabulary]`` of one block anchored at ``anchor`` (``model.py:369-396``):
        the one-window case of ``group_hidden`` (the reference checks the two agree,
        ``tests/numerical/test_model.py:586-604``), then the tied vocabulary head."""
        if type(anchor) is not int:
            raise ValueError("invalid model inputs")
        hidden = self.group_hidden(features, tokens, (anchor,), slots)[0]
        return frozen_linear(hidden, self.vocabulary, self)
