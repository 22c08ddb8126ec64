"""Drop-in mirror of the reference model API (``w1a1_eagle/model.py``).

Same names, constructor arguments, parameter names and ValueError messages as
the reference.  The binary projections run in ``libbitdraft.so``:

* ``Projection`` quantizes with ``bd_quantize_rows_i8``, multiplies int8 codes
  by the int8 signs on the tcgen05 tensor cores (exact s32 accumulation) with
  the HE4 epilogue in the same kernel, and back-propagates with the
  straight-through kernels and tcgen05 GEMMs (``bd_ste_*``);
* ``Layer`` runs its SwiGLU tail through the fused decode block
  (``bd_ffn_he4``) when no gradient is needed and at most 32 rows come in;
* ``hard_sign``, ``bound_latents`` and ``clamp_latents`` are kernels too.

Attention, norms and rotary embedding stay torch expressions of the same
mathematics (the serving path has kernels for them in ``drafter.py``).  A CUDA
device is required: there is no CPU fallback.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
from torch import Tensor, nn
from torch.nn import functional

from . import _lib, ops

MAX_DECODE_ROWS = ops.MAX_DECODE_TOKENS


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


def rms(value: Tensor, weight: Tensor, epsilon: float) -> Tensor:
    """``value / sqrt(mean(value^2) + eps) * weight`` over the last axis (``model.py:50-51``)."""
    return value * torch.rsqrt(value.square().mean(-1, keepdim=True) + epsilon) * weight


def rope(value: Tensor, positions: Tensor, theta: float) -> Tensor:
    """Rotate-half rotary embedding with frequencies ``theta^(-2i/width)`` (``model.py:54-63``)."""
    width = value.shape[-1]
    exponents = torch.arange(0, width, 2, dtype=torch.float32, device=value.device) / width
    frequency = torch.tensor(theta, dtype=torch.float32, device=value.device).pow(-exponents)
    angle = positions.float()[:, None] * frequency
    angle = torch.cat((angle, angle), -1).unsqueeze(1)
    first, second = value[..., : width // 2], value[..., width // 2:]
    return value * angle.cos() + torch.cat((-second, first), -1) * angle.sin()


def cache_storage(value: Tensor) -> Tensor:
    """Round through fp16 storage with a straight-through gradient (``model.py:98-102``)."""
    rounded = value.half().float()
    if not bool(torch.isfinite(rounded).all()):
        raise ValueError("F16 cache storage overflow")
    return value + (rounded - value).detach()


def _need_cuda(t: Tensor) -> torch.device:
    if not t.is_cuda:
        raise RuntimeError("bitdraft runs on CUDA tensors only (no CPU fallback)")
    return t.device


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


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


def _bf16_split(value: Tensor) -> tuple[Tensor, Tensor]:
    """fp32 ``value`` as bf16 hi + lo halves (value ~= hi + lo to ~16 bits)."""
    hi = value.to(torch.bfloat16)
    return hi, (value - hi.float()).to(torch.bfloat16)


class _FrozenOperand:
    """bf16 hi + lo halves of a frozen fp32 operand ``[out, in]``, made once (the
    buffer itself is never replaced or written).  ``lo`` is None when the operand
    is exactly representable in bf16 (the drafter's bf16 checkpoints)."""

    def __init__(self, operand: Tensor) -> None:
        self.source = operand
        self.version = operand._version
        self.hi, lo = _bf16_split(operand.detach())
        self.lo = lo if bool(lo.any()) else None

    def valid_for(self, operand: Tensor) -> bool:
        return self.source is operand and self.version == operand._version


def _frozen_halves(owner, operand: Tensor) -> _FrozenOperand:
    cache = owner.__dict__.get("_halves")
    if cache is None or not cache.valid_for(operand):
        cache = _FrozenOperand(operand)
        owner.__dict__["_halves"] = cache
    return cache


def _mm_split(a_hi: Tensor, a_lo: Tensor, b_hi: Tensor, b_lo: Tensor | None) -> Tensor:
    """(a_hi + a_lo) @ (b_hi + b_lo) on bf16 tensor cores with fp32 accumulation,
    leaving out only lo x lo (fp32-level accuracy: ~2^-16 relative per product)."""
    out = torch.mm(a_hi, b_hi, out_dtype=torch.float32)
    out += torch.mm(a_lo, b_hi, out_dtype=torch.float32)
    if b_lo is not None:
        out += torch.mm(a_hi, b_lo, out_dtype=torch.float32)
    return out


class _FrozenLinearFn(torch.autograd.Function):
    """``linear(value, operand)`` of a frozen fp32 operand as split-bf16 tensor-core
    GEMMs, forward and input gradient (the operand gets no gradient)."""

    @staticmethod
    def forward(ctx, value, operand, halves):
        x = value.reshape(-1, value.shape[-1]).float()
        x_hi, x_lo = _bf16_split(x)
        y = _mm_split(x_hi, x_lo, halves.hi.t(), None if halves.lo is None else halves.lo.t())
        ctx.halves = halves
        ctx.in_shape = value.shape
        return y.reshape(*value.shape[:-1], operand.shape[0])

    @staticmethod
    def backward(ctx, grad):
        g = grad.reshape(-1, grad.shape[-1]).float()
        g_hi, g_lo = _bf16_split(g)
        dx = _mm_split(g_hi, g_lo, ctx.halves.hi, ctx.halves.lo)
        return dx.reshape(ctx.in_shape), None, None


def frozen_linear(value: Tensor, operand: Tensor, owner) -> Tensor:
    """``functional.linear(value, operand)`` for a frozen operand held by ``owner``
    (its bf16 halves are cached on the owner, outside its parameters and buffers).

    CUDA tensors take the split-bf16 tensor-core GEMMs.  CPU tensors (host-side
    checks of the loss head's bookkeeping; no kernel of this package runs on
    them, and the binary projections refuse them) get the reference's own fp32
    ``linear``, since torch has no bf16 -> fp32 ``mm`` on the CPU."""
    if not value.is_cuda:
        return functional.linear(value, operand)
    return _FrozenLinearFn.apply(value, operand, _frozen_halves(owner, operand))


class FrozenLinear(nn.Module):
    """A frozen dense projection; the operand is a buffer (``model.py:105-113``).
    On the GPU the product runs on bf16 tensor cores with split operands
    (``_mm_split``), within ~1e-5 of the fp32 product."""

    operand: Tensor

    def __init__(self, weight: Tensor) -> None:
        super().__init__()
        self.register_buffer("operand", weight.detach().float().clone())

    def forward(self, value: Tensor) -> Tensor:
        return frozen_linear(value, self.operand, self)


# --------------------------------------------------------------------------- binary projection


def _round8(n: int) -> int:
    return (n + 7) // 8 * 8


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
        lib = _lib.load()
        gain = log_gain.detach().exp().contiguous()
        bound = log_clip.detach().exp().reshape(1).contiguous()
        stream = _stream(device)
        flags = ops.Flags(device)
        ld = int(lib.bd_i8_ld(inner))
        codes = torch.empty((tokens, ld), dtype=torch.int8, device=device)
        sums = torch.empty(tokens, dtype=torch.int32, device=device)
        _lib.call("bd_quantize_rows_i8", x.data_ptr(), tokens, inner, gain.data_ptr(), bound.data_ptr(), bits,
                  codes.data_ptr(), ld, sums.data_ptr(), flags.ptr, stream)
        flags.check()
        signs = module.signs_i8()
        y = torch.empty((tokens, outer), dtype=torch.float32, device=device)
        dot = torch.empty((tokens, outer), dtype=torch.float32, device=device)
        _lib.call("bd_projection_he4_tc", codes.data_ptr(), ld, sums.data_ptr(), tokens, inner, signs.data_ptr(), outer,
                  scale.detach().contiguous().data_ptr(), midpoint.detach().contiguous().data_ptr(), bound.data_ptr(),
                  bits, None, y.data_ptr(), dot.data_ptr(), flags.ptr, stream)
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
        lib = _lib.load()
        tokens, inner = x.shape
        outer = latent.shape[0]
        bits = module.bits
        need = ctx.needs_input_grad
        need_latent = need[1] or (ctx.learned and need[6])
        g = grad_out.reshape(tokens, outer).float().contiguous()
        ld_o, ld_t = _round8(outer), _round8(tokens)
        hi = torch.empty((tokens, ld_o), dtype=torch.bfloat16, device=device)
        lo = torch.empty_like(hi)
        hi_t = torch.empty((outer, ld_t), dtype=torch.bfloat16, device=device) if need_latent else None
        lo_t = torch.empty_like(hi_t) if need_latent else None
        d_scale = torch.empty(outer, dtype=torch.float32, device=device)
        d_mid = torch.empty_like(d_scale)
        gm = torch.empty(tokens, dtype=torch.float32, device=device)
        nbytes = int(lib.bd_ste_workspace_bytes(tokens, outer, inner))
        ws = ops.workspace(device, "ste", nbytes)
        sc, mid = scale.detach().contiguous(), midpoint.detach().contiguous()
        _lib.call("bd_ste_grad_prep", g.data_ptr(), dot.data_ptr(), tokens, outer, sc.data_ptr(), mid.data_ptr(),
                  bound.data_ptr(), bits, sums.data_ptr(), hi.data_ptr(), lo.data_ptr(), ld_o,
                  None if hi_t is None else hi_t.data_ptr(), None if lo_t is None else lo_t.data_ptr(), ld_t,
                  d_scale.data_ptr(), d_mid.data_ptr(), gm.data_ptr(), ws.data_ptr(), ws.numel(), stream)
        dx = d_gain = d_clip = d_latent = d_window = None
        if need[0] or need[4] or need[5]:
            signs_t = module.signs_t_bf16(ld_o)
            dv = torch.empty((tokens, inner), dtype=torch.float32, device=device)
            _lib.call("bd_gemm_bf16_split", hi.data_ptr(), lo.data_ptr(), tokens, outer, ld_o, signs_t.data_ptr(),
                      inner, ld_o, dv.data_ptr(), inner, stream)
            dx = torch.empty_like(x)
            d_gain = torch.empty(inner, dtype=torch.float32, device=device)
            d_clip = torch.empty(1, dtype=torch.float32, device=device)
            _lib.call("bd_ste_input_backward", dv.data_ptr(), None, gm.data_ptr(), x.data_ptr(), tokens, inner,
                      gain.data_ptr(), bound.data_ptr(), bits, dx.data_ptr(), d_gain.data_ptr(), d_clip.data_ptr(), 0,
                      ws.data_ptr(), ws.numel(), stream)
            dx = dx.view(ctx.value_shape)
            d_clip = d_clip.reshape(())
        if need_latent:
            codes_t = torch.empty((inner, ld_t), dtype=torch.bfloat16, device=device)
            _lib.call("bd_codes_transpose_bf16", codes.data_ptr(), tokens, inner, ctx.ld, codes_t.data_ptr(), ld_t,
                      stream)
            d_latent = torch.empty((outer, inner), dtype=torch.float32, device=device)
            partials = None
            if ctx.learned:
                partials = torch.empty(int(lib.bd_ste_weight_grad_partials(outer, inner)), dtype=torch.float32,
                                       device=device)
            flags = ops.Flags(device)
            _lib.call("bd_ste_weight_grad", hi_t.data_ptr(), lo_t.data_ptr(), outer, tokens, ld_t, codes_t.data_ptr(),
                      inner, latent.detach().contiguous().data_ptr(),
                      None if window is None else window.data_ptr(), float(module.window), bound.data_ptr(), bits,
                      d_latent.data_ptr(), None if partials is None else partials.data_ptr(), flags.ptr, stream)
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
        out = ops.tile_i8(self.latent_sign.detach().contiguous())
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
        flags = ops.Flags(device)
        _lib.call("bd_sign_cols_bf16", latent.data_ptr(), rows, cols, out.data_ptr(), ld, flags.ptr, _stream(device))
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


def _attend(query: Tensor, keys: Tensor, values: Tensor, allowed: Tensor, head_dim: int) -> Tensor:
    """Grouped-query attention.  ``query [n, kvh, g, d]``, ``keys/values [m, kvh, d]``,
    ``allowed [n, m]`` -> ``[n, kvh * g * d]``."""
    scores = torch.einsum("nhgd,mhd->hgnm", query, keys) / math.sqrt(head_dim)
    scores = scores.masked_fill(~allowed[None, None], -torch.inf)
    weights = functional.softmax(scores, -1)
    return torch.einsum("hgnm,mhd->nhgd", weights, values).reshape(query.shape[0], -1)


class Layer(nn.Module):
    """One drafter block (``model.py:172-274``): attention over cached context plus
    the block's slots, then the binary SwiGLU ``down(silu(gate(n)) * up(n))``."""

    def __init__(self, tensors: dict[str, Tensor], prefix: str, geometry: Geometry) -> None:
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
        self.gate = Projection(tensors[prefix + "ffn_gate.weight"], 4, gain, clip)
        self.up = Projection(tensors[prefix + "ffn_up.weight"], 4, gain, clip)
        self.down = Projection(tensors[prefix + "ffn_down.weight"], 8, nn.Parameter(torch.zeros(geometry.intermediate)),
                               nn.Parameter(torch.tensor(0.0)))
        self._packed: tuple[tuple, ops.PackedFFN] | None = None

    def context(self, encoded: Tensor, positions: Tensor) -> tuple[Tensor, Tensor]:
        """Context keys (normed, rotated) and values through fp16 storage (``model.py:195-200``)."""
        cfg = self.geometry
        key = self.key.forward(encoded).view(-1, cfg.kv_heads, cfg.head_dim)
        value = self.value.forward(encoded).view(-1, cfg.kv_heads, cfg.head_dim)
        key = rope(rms(key, self.k_norm, cfg.epsilon), positions, cfg.theta)
        return cache_storage(key), cache_storage(value)

    def _slot_qkv(self, state: Tensor, positions: Tensor):
        cfg = self.geometry
        norm = rms(state, self.attn_norm, cfg.epsilon)
        query = self.query.forward(norm).view(-1, cfg.heads, cfg.head_dim)
        key = self.key.forward(norm).view(-1, cfg.kv_heads, cfg.head_dim)
        value = self.value.forward(norm).view(-1, cfg.kv_heads, cfg.head_dim)
        query = rope(rms(query, self.q_norm, cfg.epsilon), positions, cfg.theta)
        key = rope(rms(key, self.k_norm, cfg.epsilon), positions, cfg.theta)
        return query, cache_storage(key), cache_storage(value)

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
        """One block over a single window's slots (``model.py:202-223``)."""
        cfg = self.geometry
        query, key, value = self._slot_qkv(state, positions)
        keys = torch.cat((context[0], key), 0)
        values = torch.cat((context[1], value), 0)
        groups = cfg.heads // cfg.kv_heads
        query = query.view(positions.shape[0], cfg.kv_heads, groups, cfg.head_dim)
        attended = _attend(query, keys, values, allowed, cfg.head_dim)
        return self.feed_forward(state + self.output.forward(attended))

    def group(self, state: Tensor, context: tuple[Tensor, Tensor], positions: Tensor, allowed: Tensor,
              slot_allowed: Tensor | None) -> Tensor:
        """Several windows at once (``model.py:225-274``): ``positions [W, k]``, the shared
        context of length L, ``allowed [W, k, L]``, ``slot_allowed [k, k]`` or None."""
        cfg = self.geometry
        windows, slots = positions.shape
        length = context[0].shape[0]
        groups, kvh, d = cfg.heads // cfg.kv_heads, cfg.kv_heads, cfg.head_dim
        query, key, value = self._slot_qkv(state, positions.reshape(-1))
        query = query.view(windows, slots, kvh, groups, d)
        key = key.view(windows, slots, kvh, d)
        value = value.view(windows, slots, kvh, d)
        scale = math.sqrt(d)
        ctx_scores = torch.einsum("wshgd,lhd->whgsl", query, context[0]) / scale
        ctx_scores = ctx_scores.masked_fill(~allowed[:, None, None], -torch.inf)
        slot_scores = torch.einsum("wshgd,wthd->whgst", query, key) / scale
        if slot_allowed is not None:
            slot_scores = slot_scores.masked_fill(~slot_allowed, -torch.inf)
        weights = functional.softmax(torch.cat((ctx_scores, slot_scores), -1), -1)
        ctx_w, slot_w = weights.split((length, slots), -1)
        attended = (torch.einsum("whgsl,lhd->wshgd", ctx_w, context[1])
                    + torch.einsum("whgst,wthd->wshgd", slot_w, value))
        attended = attended.reshape(windows * slots, -1)
        return self.feed_forward(state + self.output.forward(attended))


class HE4(nn.Module):
    """The block drafter (``model.py:277-396``): fused target features, ``layers``
    blocks, tied vocabulary head."""

    vocabulary: Tensor

    def __init__(self, tensors: dict[str, Tensor], vocabulary: Tensor, mask: int,
                 geometry: Geometry = Geometry()) -> None:
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
        self.blocks = nn.ModuleList([Layer(tensors, f"blk.{i}.", geometry) for i in range(geometry.layers)])

    def check(self, features: Tensor, tokens: tuple[int, ...], anchors: tuple[int, ...]) -> None:
        cfg = self.geometry
        if (not anchors
                or any(type(anchor) is not int or not 0 <= anchor < len(tokens) for anchor in anchors)
                or features.ndim != 2 or features.dtype not in (torch.float16, torch.float32)
                or features.shape != (len(tokens), cfg.taps * cfg.hidden)
                or any(type(token) is not int or not 0 <= token < self.vocabulary.shape[0] for token in tokens)):
            raise ValueError("invalid model inputs")

    def block(self, slots: int | None) -> int:
        size = self.geometry.slots if slots is None else slots
        if type(size) is not int or not 1 <= size <= self.geometry.slots:
            raise ValueError("block size must be between one slot and the model's slots")
        return size

    def _encode(self, features: Tensor, length: int) -> Tensor:
        device = self.vocabulary.device
        fused = self.fusion.forward(features[:length].to(device).float())
        return rms(fused, self.encoder_norm, self.geometry.epsilon)

    def group_hidden(self, features: Tensor, tokens: tuple[int, ...], anchors: tuple[int, ...],
                     slots: int | None = None) -> Tensor:
        """Hidden states ``[W, k, hidden]`` of several windows (``model.py:329-367``)."""
        self.check(features, tokens, anchors)
        cfg = self.geometry
        size = self.block(slots)
        device = self.vocabulary.device
        starts = torch.tensor(anchors, device=device)
        offsets = torch.arange(size, device=device)
        positions = starts[:, None] + offsets[None, :]
        last = max(anchors)
        ctx_positions = torch.arange(last, device=device)
        ids = torch.full((len(anchors), size), self.mask, device=device)
        ids[:, 0] = torch.tensor([tokens[a] for a in anchors], device=device)
        state = functional.embedding(ids.reshape(-1), self.vocabulary)
        encoded = self._encode(features, last)
        visible = ctx_positions[None, None, :] < starts[:, None, None]
        local = visible & ((positions[:, :, None] - ctx_positions[None, None, :]).abs() < cfg.window)
        slot_local = (offsets[:, None] - offsets[None, :]).abs() < cfg.window
        for index, block in enumerate(self.blocks):
            final = index == cfg.layers - 1
            state = block.group(state, block.context(encoded, ctx_positions), positions,
                                visible if final else local, None if final else slot_local)
        return rms(state, self.output_norm, cfg.epsilon).view(len(anchors), size, cfg.hidden)

    def forward(self, features: Tensor, tokens: tuple[int, ...], anchor: int, slots: int | None = None) -> Tensor:
        """Logits ``[k, vocabulary]`` of one block anchored at ``anchor`` (``model.py:369-396``)."""
        cfg = self.geometry
        if type(anchor) is not int:
            raise ValueError("invalid model inputs")
        self.check(features, tokens, (anchor,))
        size = self.block(slots)
        device = self.vocabulary.device
        positions = torch.arange(anchor, anchor + size, device=device)
        ctx_positions = torch.arange(anchor, device=device)
        ids = torch.tensor((tokens[anchor],) + (self.mask,) * (size - 1), device=device)
        state = functional.embedding(ids, self.vocabulary)
        encoded = self._encode(features, anchor)
        keys = torch.cat((ctx_positions, positions))
        for index, block in enumerate(self.blocks):
            allowed = torch.ones((size, anchor + size), dtype=torch.bool, device=device)
            if index < cfg.layers - 1:
                allowed &= (positions[:, None] - keys[None, :]).abs() < cfg.window
            state = block.forward(state, block.context(encoded, ctx_positions), positions, allowed)
        return frozen_linear(rms(state, self.output_norm, cfg.epsilon), self.vocabulary, self)
