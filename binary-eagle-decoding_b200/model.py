"""Drop-in mirror of the reference model API (``w1a1_eagle/model.py``).

Same names, constructor arguments, parameter names and ValueError messages as
the reference.  The binary projections run in ``libbitdraft.so``:

* ``Projection`` quantizes with ``bd_quantize_rows_bf16``, multiplies exact
  bf16 codes by exact bf16 signs on the tensor cores (fp32 accumulation, so the
  integer dot is exact), applies ``bd_he4_epilogue``, and back-propagates with
  the straight-through kernels (``bd_ste_*``);
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


class _ProjectionFn(torch.autograd.Function):
    """Forward value and straight-through gradients of ``Projection.forward``
    (``model.py:128-150``); see ``csrc/ste.cu`` for the operation order."""

    @staticmethod
    def forward(ctx, value, latent, scale, midpoint, log_gain, log_clip, module):
        device = _need_cuda(value)
        x = value.reshape(-1, value.shape[-1]).float().contiguous()
        tokens, inner = x.shape
        outer = latent.shape[0]
        bits = module.bits
        gain = log_gain.detach().exp().contiguous()
        bound = log_clip.detach().exp().reshape(1).contiguous()
        stream = _stream(device)
        flags = ops.Flags(device)
        codes = torch.empty((tokens, inner), dtype=torch.bfloat16, device=device)
        sums = torch.empty(tokens, dtype=torch.int32, device=device)
        _lib.call("bd_quantize_rows_bf16", x.data_ptr(), tokens, inner, gain.data_ptr(), bound.data_ptr(), bits,
                  codes.data_ptr(), sums.data_ptr(), flags.ptr, stream)
        flags.check()
        signs = module.signs_bf16()
        dot = torch.mm(codes, signs.t(), out_dtype=torch.float32)
        y = torch.empty((tokens, outer), dtype=torch.float32, device=device)
        _lib.call("bd_he4_epilogue", dot.data_ptr(), tokens, outer, scale.detach().contiguous().data_ptr(),
                  midpoint.detach().contiguous().data_ptr(), bound.data_ptr(), bits, sums.data_ptr(), None,
                  y.data_ptr(), stream)
        ctx.module = module
        ctx.value_shape = value.shape
        ctx.save_for_backward(x, latent, scale, midpoint, gain, bound, dot, codes, sums)
        return y.view(*value.shape[:-1], outer)

    @staticmethod
    def backward(ctx, grad_out):
        x, latent, scale, midpoint, gain, bound, dot, codes, sums = ctx.saved_tensors
        module = ctx.module
        device = x.device
        stream = _stream(device)
        tokens, inner = x.shape
        outer = latent.shape[0]
        bits = module.bits
        g = grad_out.reshape(tokens, outer).float().contiguous()
        hi = torch.empty((tokens, outer), dtype=torch.bfloat16, device=device)
        lo = torch.empty_like(hi)
        d_scale = torch.empty(outer, dtype=torch.float32, device=device)
        d_mid = torch.empty_like(d_scale)
        gm = torch.empty(tokens, dtype=torch.float32, device=device)
        nbytes = int(_lib.load().bd_ste_workspace_bytes(tokens, outer, inner))
        ws = ops.workspace(device, "ste", nbytes)
        sc, mid = scale.detach().contiguous(), midpoint.detach().contiguous()
        _lib.call("bd_ste_grad_prep", g.data_ptr(), dot.data_ptr(), tokens, outer, sc.data_ptr(), mid.data_ptr(),
                  bound.data_ptr(), bits, sums.data_ptr(), hi.data_ptr(), lo.data_ptr(), d_scale.data_ptr(),
                  d_mid.data_ptr(), gm.data_ptr(), ws.data_ptr(), ws.numel(), stream)
        need = ctx.needs_input_grad
        dx = d_gain = d_clip = d_latent = None
        if need[0] or need[4] or need[5]:
            signs = module.signs_bf16()
            dv1 = torch.mm(hi, signs, out_dtype=torch.float32)
            dv2 = torch.mm(lo, signs, out_dtype=torch.float32)
            dx = torch.empty_like(x)
            d_gain = torch.empty(inner, dtype=torch.float32, device=device)
            d_clip = torch.empty(1, dtype=torch.float32, device=device)
            _lib.call("bd_ste_input_backward", dv1.data_ptr(), dv2.data_ptr(), gm.data_ptr(), x.data_ptr(), tokens,
                      inner, gain.data_ptr(), bound.data_ptr(), bits, dx.data_ptr(), d_gain.data_ptr(),
                      d_clip.data_ptr(), 0, ws.data_ptr(), ws.numel(), stream)
            dx = dx.view(ctx.value_shape)
            d_clip = d_clip.reshape(())
        if need[1]:
            ds1 = torch.mm(hi.t(), codes, out_dtype=torch.float32)
            ds2 = torch.mm(lo.t(), codes, out_dtype=torch.float32)
            d_latent = torch.empty((outer, inner), dtype=torch.float32, device=device)
            _lib.call("bd_ste_sign_backward", ds1.data_ptr(), ds2.data_ptr(), latent.data_ptr(), outer * inner,
                      float(module.window), bound.data_ptr(), bits, d_latent.data_ptr(), None, stream)
        return (dx if need[0] else None, d_latent, d_scale if need[2] else None, d_mid if need[3] else None,
                d_gain if need[4] else None, d_clip if need[5] else None, None)


class Projection(nn.Module):
    """HE4 binary projection (``model.py:116-150``) with the reference's parameters
    ``latent_sign``, ``scale``, ``midpoint``, ``log_gain``, ``log_clip``.

    ``window`` is the sign straight-through window (1.0 in the reference).  Packed
    and expanded signs are caches outside the module's parameters and buffers,
    keyed by the latent's version counter.
    """

    def __init__(self, weight: Tensor, bits: int, gain: nn.Parameter, clip: nn.Parameter,
                 window: float = 1.0) -> None:
        super().__init__()
        if bits not in (4, 8) or weight.ndim != 2 or not bool(torch.isfinite(weight).all()):
            raise ValueError("invalid HE4 projection")
        self.bits = bits
        self.window = float(window)
        self.latent_sign = nn.Parameter(weight.detach().float().clone())
        self.scale = nn.Parameter(weight.detach().float().abs().mean(-1))
        self.midpoint = nn.Parameter(torch.zeros(weight.shape[0]))
        self.log_gain = gain
        self.log_clip = clip
        self._signs: dict[str, tuple[tuple[int, int], Tensor]] = {}

    def _key(self) -> tuple[int, int]:
        return self.latent_sign.data_ptr(), self.latent_sign._version

    def signs_bf16(self) -> Tensor:
        """+-1 bf16 copy of the signs [out, in] (cached per latent version)."""
        key = self._key()
        hit = self._signs.get("bf16")
        if hit is not None and hit[0] == key:
            return hit[1]
        latent = self.latent_sign.detach()
        device = _need_cuda(latent)
        out = torch.empty(latent.shape, dtype=torch.bfloat16, device=device)
        flags = ops.Flags(device)
        _lib.call("bd_sign_rows", latent.contiguous().data_ptr(), latent.numel(), out.data_ptr(), None, flags.ptr,
                  _stream(device))
        flags.check()
        self._signs["bf16"] = (key, out)
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
                                   self)


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
                signs_down=self.down.signs_w8(), scale_gate=self.gate.scale.detach().contiguous(),
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
