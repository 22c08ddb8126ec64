"""Training-size block attention (``Layer.group``'s attention, w1a1_eagle/model.py:225-270)
on the ``bd_train_attention_*`` kernels against the reference's eager expression
evaluated in float64 on the CPU (forward and every input gradient)."""

from __future__ import annotations

import pytest
import torch

from conftest import package, submodule

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")

# fp16 hi + lo halves carry ~22 bits of each fp32 operand and the products
# accumulate in fp32: the outputs and gradients sit within a few 1e-6 (relative
# to the tensor's norm) of the float64 evaluation; 1e-4 leaves a wide margin.
RTOL = 1e-4


@pytest.fixture(scope="module")
def model():
    package()
    return submodule("model")


def rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def case(windows, slots, kvh, groups, dim, length, seed, windowed):
    g = torch.Generator().manual_seed(seed)
    half = lambda *s: torch.randn(*s, generator=g).half().float()  # fp16 values, as cache_storage leaves them
    query = torch.randn(windows, slots, kvh, groups, dim, generator=g)
    ctx_k, ctx_v = half(length, kvh, dim), half(length, kvh, dim)
    slot_k, slot_v = half(windows, slots, kvh, dim), half(windows, slots, kvh, dim)
    anchors = torch.randint(0, length + 1, (windows,), generator=g)
    anchors[0] = length  # one window sees the whole context
    positions = anchors[:, None] + torch.arange(slots)[None]
    keys = torch.arange(length)
    allowed = keys[None, None, :] < anchors[:, None, None]
    slot_allowed = None
    if windowed:
        allowed = allowed & ((positions[:, :, None] - keys[None, None, :]).abs() < windowed)
        offset = torch.arange(slots)
        slot_allowed = (offset[:, None] - offset[None, :]).abs() < windowed
    upstream = torch.randn(windows, slots, kvh, groups, dim, generator=g) * 1e-3
    return query, ctx_k, ctx_v, slot_k, slot_v, allowed, slot_allowed, upstream


@pytest.mark.parametrize("shape", [
    (3, 16, 2, 4, 128, 200, 0),     # config geometry per kv head, ragged context
    (2, 5, 1, 2, 2, 70, 6),         # the tiny test model: head_dim 2, 2 query heads per kv head, sliding window
    (4, 16, 2, 3, 64, 64, 0),       # three query heads per kv head, one exact key tile
    (2, 16, 1, 4, 128, 0, 0),       # no context: the slots alone
])
def test_train_attention_matches_float64(model, shape):
    windows, slots, kvh, groups, dim, length, windowed = shape
    query, ctx_k, ctx_v, slot_k, slot_v, allowed, slot_allowed, upstream = case(
        windows, slots, kvh, groups, dim, length, 31 + windows * dim + length, windowed)

    ref_in = [t.double().requires_grad_() for t in (query, ctx_k, ctx_v, slot_k, slot_v)]
    ref = model._window_attention(*ref_in, allowed, slot_allowed, dim).view(windows, slots, kvh, groups, dim)
    (ref * upstream.double()).sum().backward()

    gpu_in = [t.to(DEV).requires_grad_() for t in (query, ctx_k, ctx_v, slot_k, slot_v)]
    out = model.train_attention(*gpu_in, allowed.to(DEV), None if slot_allowed is None else slot_allowed.to(DEV))
    (out * upstream.to(DEV)).sum().backward()
    torch.cuda.synchronize()

    assert rel(out.detach(), ref.detach()) < RTOL
    names = ("query", "ctx_k", "ctx_v", "slot_k", "slot_v")
    for name, a, b in zip(names, gpu_in, ref_in):
        if b.grad is None or b.grad.numel() == 0:
            continue
        assert torch.isfinite(a.grad).all(), name
        assert rel(a.grad, b.grad) < RTOL, (name, rel(a.grad, b.grad))


def test_train_attention_is_deterministic(model):
    query, ctx_k, ctx_v, slot_k, slot_v, allowed, slot_allowed, upstream = case(3, 16, 2, 4, 128, 150, 9, 0)
    grads = []
    for _ in range(2):
        gpu_in = [t.to(DEV).requires_grad_() for t in (query, ctx_k, ctx_v, slot_k, slot_v)]
        out = model.train_attention(*gpu_in, allowed.to(DEV), None)
        (out * upstream.to(DEV)).sum().backward()
        grads.append([out.detach()] + [t.grad for t in gpu_in])
    for a, b in zip(*grads):
        assert torch.equal(a, b)
