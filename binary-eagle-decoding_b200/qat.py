"""QAT update of the binary drafter (``w1a1_eagle/numerical/worker.py:300-392``).

One update is: the windows' hidden states (``HE4.group_hidden``), the weighted
cross-entropy of the drafted positions against the frozen vocabulary head in
128-row chunks (``group_loss``), the straight-through backward of the binary
projections (kernels in ``csrc/ste.cu``), an optional data-parallel gradient
average (NCCL all-reduce of flat buckets), the global gradient-norm clip, and
the fused AdamW + sign re-pack (``csrc/optim.cu``).

The optimizer takes the caller's ``Optimization`` (``w1a1_eagle/training.py:151-170``)
or :class:`UpdatePolicy`; ``label_weights`` gives the label weights of
``worker.py:41-50``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.distributed as dist
from torch import Tensor, nn

from . import _lib, ops
from .model import (HE4, Projection, _bump, _flags, _frozen_halves, _need_cuda, _split, _split_workspace, _stream,
                    _to_device, deferred_checks, frozen_linear)

PARAMETER_GROUPS = ("sign", "scale", "midpoint", "gain", "clip", "norm")
HEAD_ROWS = 128
SUFFIX_GROUPS = {"latent_sign": "sign", "scale": "scale", "midpoint": "midpoint", "log_gain": "gain",
                 "log_clip": "clip", "log_window": "clip"}
# The reference's default AdamW step size per parameter group (training.py:108-109).
REFERENCE_STEP_SIZES = {"sign": 1e-3, "scale": 1e-5, "midpoint": 1e-5, "gain": 1e-5, "clip": 1e-5, "norm": 1e-5}


class _Constant:
    def multiplier(self, updates: int) -> float:
        return 1.0


@dataclass(frozen=True)
class UpdatePolicy:
    """What the optimizer reads from the reference's ``Optimization``
    (``training.py:151-170``): ``step_sizes`` per group, ``schedule.multiplier(n)``
    and ``latent_multiple``.  The caller's own ``Optimization`` object can be
    passed to :class:`BitAdamW` instead; this default has the reference's step
    sizes and a constant schedule."""

    step_sizes: dict[str, float] = field(default_factory=lambda: dict(REFERENCE_STEP_SIZES))
    schedule: object = field(default_factory=_Constant)
    latent_multiple: float | None = None


def label_weights(lengths: tuple[int, ...], positions: tuple[float, ...] | None = None) -> Tensor:
    """Weights of the concatenated labels of several windows (``worker.py:41-50``):
    within a window, label ``i`` weighs ``exp(-i / 7)`` (or ``positions[i]``),
    normalised to sum 1 over the window, and every window counts ``1 / #windows``."""
    if not lengths or min(lengths) < 1:
        raise ValueError("every window needs at least one label")
    offsets = torch.cat([torch.arange(n) for n in lengths])
    window = torch.repeat_interleave(torch.arange(len(lengths)), torch.tensor(lengths))
    raw = (torch.exp(-offsets / 7) if positions is None
           else torch.tensor(positions, dtype=torch.float32)[offsets])
    totals = torch.zeros(len(lengths)).index_add_(0, window, raw)
    return raw / totals[window] / len(lengths)


def parameter_groups(model: nn.Module) -> dict[str, list[tuple[str, nn.Parameter]]]:
    """Trainable parameters by group, keyed on the name suffix (``worker.py:111-121``)."""
    groups: dict[str, list[tuple[str, nn.Parameter]]] = {key: [] for key in PARAMETER_GROUPS}
    for name, parameter in model.named_parameters():
        if parameter.requires_grad:
            groups[SUFFIX_GROUPS.get(name.rsplit(".", 1)[-1], "norm")].append((name, parameter))
    return groups


# --------------------------------------------------------------------------- gradient norm


def clip_grad_norm(parameters, max_norm: float = 1.0) -> tuple[Tensor, Tensor]:
    """Global L2 norm of the gradients and the clip coefficient ``min(1, max / (norm + 1e-6))``
    (``torch.nn.utils.clip_grad_norm_``, ``worker.py:372``), both device scalars.

    The gradients are not rescaled here: the optimizer applies the coefficient as
    it reads them.  A non-finite norm raises ``ValueError`` like ``error_if_nonfinite``.
    """
    grads = [p.grad for p in parameters if p.grad is not None]
    if not grads:
        raise ValueError("no gradients to clip")
    device = _need_cuda(grads[0])
    lib = _lib.load()
    counts = [int(lib.bd_sum_squares_count(g.numel())) for g in grads]
    partials = torch.empty(sum(counts), dtype=torch.float32, device=device)
    stream = _stream(device)
    offset = 0
    for g, n in zip(grads, counts):
        gc = g.contiguous()
        _lib.call("bd_sum_squares", gc.data_ptr(), gc.numel(), partials.data_ptr() + 4 * offset, stream)
        offset += n
    total = torch.empty(1, dtype=torch.float32, device=device)
    coef = torch.empty(1, dtype=torch.float32, device=device)
    flags = ops.Flags(device)
    _lib.call("bd_grad_norm", partials.data_ptr(), partials.numel(), float(max_norm), total.data_ptr(),
              coef.data_ptr(), flags.ptr, stream)
    if int(flags.tensor.item()):
        raise ValueError("non-finite total norm of gradients")
    return total, coef


# --------------------------------------------------------------------------- optimizer


class BitAdamW:
    """``torch.optim.AdamW(groups, weight_decay=0, fused=True)`` over the drafter's
    parameter groups (``worker.py:122-130``), with the post-step clamps of
    ``worker.py:377-382`` fused in: ``scale`` is clamped at 0, latents optionally to
    [-1, 1], and each latent's new signs are re-packed into its projection's W8
    cache in the same pass."""

    def __init__(self, model: nn.Module, optimization=None, betas=(0.9, 0.999), eps: float = 1e-8) -> None:
        self.model = model
        self.optimization = optimization or UpdatePolicy()
        if set(self.optimization.step_sizes) != set(PARAMETER_GROUPS):
            raise ValueError("a step size for every parameter group is required")
        self.betas = betas
        self.eps = eps
        self.groups = parameter_groups(model)
        self.owner = {id(m.latent_sign): m for m in model.modules() if isinstance(m, Projection)}
        self.state: dict[int, dict] = {}
        self.lr = dict(self.optimization.step_sizes)

    def zero_grad(self) -> None:
        for params in self.groups.values():
            for _, p in params:
                p.grad = None

    def set_multiplier(self, multiplier: float) -> None:
        self.lr = {k: v * multiplier for k, v in self.optimization.step_sizes.items()}

    @torch.no_grad()
    def step(self, clip_coef: Tensor | None = None) -> None:
        clamp = self.optimization.latent_multiple is not None
        flags = None
        for group, params in self.groups.items():
            lr = float(self.lr[group])
            for _, p in params:
                if p.grad is None:
                    continue
                device = _need_cuda(p)
                flags = flags or ops.Flags(device)
                st = self.state.get(id(p))
                if st is None:
                    st = {"step": 0, "exp_avg": torch.zeros_like(p), "exp_avg_sq": torch.zeros_like(p)}
                    self.state[id(p)] = st
                st["step"] += 1
                grad = p.grad.contiguous()
                coef = None if clip_coef is None else clip_coef.data_ptr()
                owner = self.owner.get(id(p))
                stream = _stream(device)
                if owner is not None:
                    tiled = torch.zeros(ops.w8_words(*p.shape), dtype=torch.int32, device=device)
                    _lib.call("bd_adamw_latent", p.data_ptr(), grad.data_ptr(), st["exp_avg"].data_ptr(),
                              st["exp_avg_sq"].data_ptr(), p.shape[0], p.shape[1], lr, self.betas[0], self.betas[1],
                              self.eps, st["step"], coef, int(clamp), tiled.data_ptr(), 1, 0, flags.ptr, stream)
                    _bump(p)
                    owner.adopt_w8(tiled)
                else:
                    lower = 0.0 if group == "scale" else -math.inf
                    _lib.call("bd_adamw", p.data_ptr(), grad.data_ptr(), st["exp_avg"].data_ptr(),
                              st["exp_avg_sq"].data_ptr(), p.numel(), lr, self.betas[0], self.betas[1], self.eps,
                              st["step"], coef, lower, flags.ptr, stream)
                    _bump(p)
        if flags is not None and int(flags.tensor.item()):
            raise ValueError("nonfinite post-update state")


# --------------------------------------------------------------------------- data parallel


def average_gradients(parameters, group=None, bucket_bytes: int = 256 << 20) -> None:
    """Average gradients over the process group with NCCL all-reduces of flat fp32
    buckets (sum, then divide by the world size), in parameter order."""
    if not dist.is_available() or not dist.is_initialized():
        return
    world = dist.get_world_size(group)
    if world == 1:
        return
    grads = [p.grad for p in parameters if p.grad is not None]
    bucket: list[Tensor] = []
    size = 0

    def flush() -> None:
        nonlocal bucket, size
        if not bucket:
            return
        flat = torch.cat([g.reshape(-1) for g in bucket])
        dist.all_reduce(flat, group=group)
        flat.div_(world)
        offset = 0
        for g in bucket:
            n = g.numel()
            g.copy_(flat[offset:offset + n].view_as(g))
            offset += n
        bucket, size = [], 0

    for g in grads:
        bucket.append(g)
        size += g.numel() * 4
        if size >= bucket_bytes:
            flush()
    flush()


class GradientExchange:
    """Data-parallel gradient average overlapped with the backward pass.

    Each trainable parameter gets a post-accumulate hook; while the exchange is
    ``armed`` (during the last backward pass of an update), every gradient that
    becomes final joins the current bucket, and a full bucket (``bucket_bytes``
    of fp32) is flattened and all-reduced asynchronously (NCCL on GPUs, gloo on
    CPUs) while autograd goes on with the earlier layers.  ``finish()`` flushes
    the last bucket, waits for every reduction and writes back the averages
    (sum / world size), before the gradient-norm clip (``worker.py:372``).  All
    ranks build the same graph, so their hooks fire in the same order and they
    issue the same collectives."""

    def __init__(self, parameters, group=None, bucket_bytes: int = 64 << 20) -> None:
        self.group = group
        self.bucket_bytes = bucket_bytes
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.armed = False
        self._bucket: list[nn.Parameter] = []
        self._size = 0
        self._pending: list[tuple[object, Tensor, list[Tensor]]] = []
        self.buckets = 0
        self._hooks = [p.register_post_accumulate_grad_hook(self.ready) for p in parameters if p.requires_grad]

    def ready(self, parameter: nn.Parameter) -> None:
        """A gradient became final (the post-accumulate hook, or a ``LatentGradients``
        flush): add it to the bucket while the exchange is armed."""
        if not self.armed or self.world == 1 or parameter.grad is None:
            return
        self._bucket.append(parameter)
        self._size += parameter.grad.numel() * 4
        if self._size >= self.bucket_bytes:
            self._flush()

    def _flush(self) -> None:
        if not self._bucket:
            return
        grads = [p.grad for p in self._bucket]
        flat = torch.cat([g.reshape(-1) for g in grads])
        handle = dist.all_reduce(flat, group=self.group, async_op=True)
        self._pending.append((handle, flat, grads))
        self._bucket, self._size = [], 0
        self.buckets += 1

    def finish(self) -> None:
        self._flush()
        for handle, flat, grads in self._pending:
            handle.wait()
            flat.div_(self.world)
            offset = 0
            for g in grads:
                n = g.numel()
                g.copy_(flat[offset:offset + n].view_as(g))
                offset += n
        self._pending = []
        self.armed = False

    def remove(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []


# --------------------------------------------------------------------------- one update


@dataclass(frozen=True)
class Window:
    """One supervised window: the anchor position and the labels of its drafted slots."""

    anchor: int
    labels: tuple[int, ...]


def group_loss(model: HE4, features: Tensor, tokens: tuple[int, ...], windows: tuple[Window, ...],
               slots: int | None = None, positions: tuple[float, ...] | None = None, scale: float = 1.0) -> Tensor:
    """Weighted cross-entropy of the drafted positions (``worker.py:315-363``); runs the
    backward of the vocabulary head in 128-row chunks, then through the drafter.
    ``scale`` multiplies the label weights (1/n to average n sequences into one update)."""
    if not windows or any(not w.labels for w in windows):
        raise ValueError("an update requires supervised windows")
    device = model.vocabulary.device
    size = model.block(slots)
    if size < 2:
        raise ValueError("an update requires at least one drafted position")
    hidden = model.group_hidden(features, tokens, tuple(w.anchor for w in windows), size)
    lengths = tuple(min(len(w.labels), size - 1) for w in windows)
    rows = _to_device([i * size + 1 + o for i, n in enumerate(lengths) for o in range(n)], device)
    labels = _to_device([l for w, n in zip(windows, lengths) for l in w.labels[:n]], device)
    weights = label_weights(lengths, positions) * scale
    weights = weights.pin_memory().to(device, non_blocking=True) if device.type == "cuda" else weights.to(device)
    selected = hidden.view(-1, hidden.shape[-1]).index_select(0, rows)
    if not selected.is_cuda:
        # host-side bookkeeping checks only: the reference's own chunked expression
        head = selected.detach().requires_grad_()
        total = torch.zeros((), device=device)
        for start in range(0, labels.numel(), HEAD_ROWS):
            end = start + HEAD_ROWS
            logits = frozen_linear(head[start:end], model.vocabulary, model)
            losses = torch.nn.functional.cross_entropy(logits, labels[start:end], reduction="none")
            loss = (losses * weights[start:end]).sum()
            torch.autograd.backward(loss)
            total = total + loss.detach()
        if not bool(torch.isfinite(total)) or head.grad is None:
            raise ValueError("nonfinite loss")
        torch.autograd.backward(selected, head.grad)
        return total
    total, d_head = loss_head(selected.detach(), model, labels, weights)
    torch.autograd.backward(selected, d_head)
    return total


def group_loss_deferred(model: HE4, features: Tensor, tokens: tuple[int, ...], windows: tuple[Window, ...],
                        slots: int | None = None, positions: tuple[float, ...] | None = None,
                        scale: float = 1.0) -> Tensor:
    """``group_loss`` with the projections' device error checks read once at the end
    (``model.deferred_checks``) instead of after every launch."""
    with deferred_checks(model.vocabulary.device):
        return group_loss(model, features, tokens, windows, slots, positions, scale)


def loss_head(head: Tensor, model: HE4, labels: Tensor, weights: Tensor) -> tuple[Tensor, Tensor]:
    """``sum_r w_r cross_entropy(head_r . vocabulary^T, label_r)`` and its gradient with
    respect to ``head`` (``worker.py:350-359``), on the tcgen05 tensor cores
    without writing the logits: ``bd_loss_head_forward`` keeps per-row softmax
    statistics in the GEMM epilogue, ``bd_loss_head_grad`` recomputes the logits
    into ``w (softmax - onehot)`` as bf16 halves, and one split GEMM with the
    transposed vocabulary gives the gradient.  Raises ``ValueError("nonfinite
    loss")`` like the reference (``worker.py:360-361``)."""
    device = _need_cuda(head)
    lib = _lib.load()
    halves = _frozen_halves(model, model.vocabulary)
    rows, hidden = head.shape
    vocab = model.vocabulary.shape[0]
    h_hi, h_lo, ld_h = _split(head)
    lab = labels.to(device=device, dtype=torch.int32).contiguous()
    w = weights.to(device=device, dtype=torch.float32).contiguous()
    stats = torch.empty(int(lib.bd_loss_head_stats_count(rows, vocab)), dtype=torch.float32, device=device)
    target = torch.empty(rows, dtype=torch.float32, device=device)
    lse = torch.empty(rows, dtype=torch.float32, device=device)
    loss_rows = torch.empty(rows, dtype=torch.float32, device=device)
    total = torch.empty(1, dtype=torch.float32, device=device)
    flags, now = _flags(device)
    stream = _stream(device)
    v_lo = None if halves.lo is None else halves.lo.data_ptr()
    _lib.call("bd_loss_head_forward", h_hi.data_ptr(), h_lo.data_ptr(), rows, hidden, ld_h, halves.hi.data_ptr(), v_lo,
              vocab, lab.data_ptr(), w.data_ptr(), stats.data_ptr(), target.data_ptr(), lse.data_ptr(),
              loss_rows.data_ptr(), total.data_ptr(), flags.ptr, stream)
    if now:
        flags.check()
    hi_t, lo_t, ld_v = halves.transposed()
    dl_hi = torch.empty((rows, ld_v), dtype=torch.bfloat16, device=device)
    dl_lo = torch.empty_like(dl_hi)
    _lib.call("bd_loss_head_grad", h_hi.data_ptr(), h_lo.data_ptr(), rows, hidden, ld_h, halves.hi.data_ptr(), v_lo,
              vocab, lab.data_ptr(), w.data_ptr(), lse.data_ptr(), dl_hi.data_ptr(), dl_lo.data_ptr(), ld_v, stream)
    d_head = torch.empty((rows, hidden), dtype=torch.float32, device=device)
    ws, nbytes = _split_workspace(device, rows, hidden, vocab, 2 if lo_t is None else 3)
    _lib.call("bd_gemm_bf16_split3", dl_hi.data_ptr(), dl_lo.data_ptr(), rows, vocab, ld_v, hi_t.data_ptr(),
              None if lo_t is None else lo_t.data_ptr(), hidden, ld_v, d_head.data_ptr(), hidden, ws, nbytes, stream)
    return total.reshape(()), d_head


def update(model: HE4, optimizer: BitAdamW, features: Tensor, tokens: tuple[int, ...], windows: tuple[Window, ...],
           updates: int = 0, slots: int | None = None, group=None) -> tuple[float, float]:
    """One QAT update (``worker.py:365-392``).  Returns ``(loss, gradient norm)``; with an
    initialised process group the gradients are averaged across ranks first."""
    optimizer.zero_grad()
    loss = group_loss_deferred(model, features, tokens, windows, slots)
    params = [p for ps in optimizer.groups.values() for _, p in ps]
    average_gradients(params, group)
    norm, coef = clip_grad_norm(params, 1.0)
    optimizer.set_multiplier(optimizer.optimization.schedule.multiplier(updates))
    optimizer.step(coef)
    return float(loss), float(norm)
