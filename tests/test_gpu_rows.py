"""The fused row-wise kernels of the training forward (``bd_rms_*``, ``bd_head_post*``)
against the reference's torch expressions (``rms``, ``rope``, ``cache_storage`` of
w1a1_eagle/model.py:50-63, 98-102) evaluated in float64 on the CPU, forward and
backward."""

from __future__ import annotations

import pytest
import torch

from conftest import package, submodule

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def model():
    package()
    return submodule("model")


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-300))


def ref_rms(x, w, eps):
    return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * w


def ref_rope(x, positions, theta):
    # the angles in fp32 as the reference forms them (fp32 frequencies times the
    # position), the rotation in float64
    width = x.shape[-1]
    exponents = torch.arange(0, width, 2, dtype=torch.float32) / width
    angle = (positions.float()[:, None] * torch.tensor(theta, dtype=torch.float32).pow(-exponents)).double()
    angle = torch.cat((angle, angle), -1).unsqueeze(1)
    first, second = x[..., : width // 2], x[..., width // 2:]
    return x * angle.cos() + torch.cat((-second, first), -1) * angle.sin()


@pytest.mark.parametrize("shape", [(37, 2560), (300, 10240), (5, 4)])
def test_rms_forward_backward(model, shape):
    g = torch.Generator().manual_seed(shape[0])
    x = torch.randn(shape, generator=g) * 3
    w = torch.randn(shape[1], generator=g)
    up = torch.randn(shape, generator=g)
    xd, wd = x.double().requires_grad_(), w.double().requires_grad_()
    ref = ref_rms(xd, wd, 1e-6)
    (ref * up.double()).sum().backward()
    xg, wg = x.to(DEV).requires_grad_(), w.to(DEV).requires_grad_()
    out = model.rms(xg, wg, 1e-6)
    (out * up.to(DEV)).sum().backward()
    assert rel(out.detach(), ref.detach()) < 1e-6
    assert rel(xg.grad, xd.grad) < 1e-5
    assert rel(wg.grad, wd.grad) < 1e-5


@pytest.mark.parametrize("heads,dim,weighted,rotary,fp16", [
    (32, 128, True, True, False),   # queries
    (8, 128, True, True, True),     # keys: rms, rotary, fp16 storage
    (8, 128, False, False, True),   # values: fp16 storage only
    (2, 2, True, True, True),       # the tiny test model's head_dim 2
])
def test_head_post_forward_backward(model, heads, dim, weighted, rotary, fp16):
    rows, theta, eps = 96, 1e6, 1e-6
    g = torch.Generator().manual_seed(heads * dim)
    x = torch.randn((rows, heads * dim), generator=g) * 2
    w = torch.randn(dim, generator=g) if weighted else None
    positions = torch.randint(0, 4096, (rows,), generator=g)
    up = torch.randn((rows, heads, dim), generator=g)

    xd = x.double().requires_grad_()
    wd = w.double().requires_grad_() if weighted else None
    ref = xd.view(rows, heads, dim)
    if weighted:
        ref = ref_rms(ref, wd, eps)
    if rotary:
        ref = ref_rope(ref, positions, theta)
    (ref * up.double()).sum().backward()  # the fp16 rounding passes the gradient straight through

    xg = x.to(DEV).requires_grad_()
    wg = w.to(DEV).requires_grad_() if weighted else None
    out = model.head_post(xg, heads, dim, wg, eps, positions.to(DEV) if rotary else None, theta, fp16)
    (out * up.to(DEV)).sum().backward()
    torch.cuda.synchronize()
    if fp16:
        # fp16 storage: within half an fp16 ulp of the exact value (plus the fp32 path's error)
        ulp = torch.clamp(ref.detach().abs(), min=2.0 ** -14) * 2.0 ** -10
        assert bool(((out.detach().double().cpu() - ref.detach()).abs() <= 0.5 * ulp + 1e-5).all())
        assert bool((out.detach().half().float() == out.detach()).all())
    else:
        assert rel(out.detach(), ref.detach()) < 1e-5
    assert rel(xg.grad, xd.grad) < 1e-5
    if weighted:
        assert rel(wg.grad, wd.grad) < 1e-5


def test_head_post_fp16_overflow_raises(model):
    x = torch.full((4, 8 * 128), 1e6, device=DEV)
    with pytest.raises(ValueError, match="F16 cache storage overflow"):
        model.head_post(x, 8, 128, None, 0.0, None, 0.0, True)
