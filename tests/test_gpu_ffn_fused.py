"""The two-launch HE4 SwiGLU block (``bd_ffn_he4_fused``, tokens <= 16) on the GPU:
its D8 down signs against the oracle's layout, and the block against the
oracle's ``Projection.forward`` composition and against the three-kernel path
(needs a B200)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import package
from oracle import core

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
FIELDS = ("latent", "scale", "midpoint", "gain", "bound")


@pytest.fixture(scope="module")
def ops():
    return package().ops


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a, np.float64) - b) / max(np.linalg.norm(np.asarray(b, np.float64)), 1e-30))


def he4_case(H, F, seed, bounds=(2.0, 0.05)):
    rng = np.random.default_rng(seed)
    params = {}
    for name, shape in (("gate", (F, H)), ("up", (F, H)), ("down", (H, F))):
        w = (rng.standard_normal(shape) * 0.02).astype(np.float32)
        w.reshape(-1)[::97] = -0.0
        params[name] = {"latent": w, "scale": np.abs(w).mean(-1, dtype=np.float32),
                        "midpoint": (rng.standard_normal(shape[0]) * 1e-3).astype(np.float32),
                        "gain": np.exp(rng.standard_normal(shape[1]).astype(np.float32) * 0.1).astype(np.float32),
                        "bound": np.float32(bounds[0] if name != "down" else bounds[1])}
    params["up"]["gain"], params["up"]["bound"] = params["gate"]["gain"], params["gate"]["bound"]
    return params


def pack(ops, p):
    ffn = ops.pack_ffn(dev(p["gate"]["latent"]), dev(p["up"]["latent"]), dev(p["down"]["latent"]),
                       dev(p["gate"]["scale"]), dev(p["up"]["scale"]), dev(p["down"]["scale"]))
    ffn.midpoint_gate, ffn.midpoint_up = dev(p["gate"]["midpoint"]), dev(p["up"]["midpoint"])
    ffn.midpoint_down = dev(p["down"]["midpoint"])
    ffn.gain_gate_up = dev(p["gate"]["gain"])
    ffn.bound_gate_up = dev(np.atleast_1d(p["gate"]["bound"]))
    ffn.gain_down = dev(p["down"]["gain"])
    ffn.bound_down = dev(np.atleast_1d(p["down"]["bound"]))
    return ffn


@pytest.mark.parametrize("rows,cols", [(2560, 9728), (64, 96), (32, 32), (96, 160)])
def test_d8_layout_matches_oracle(ops, rows, cols):
    w = torch.randn((rows, cols), generator=torch.Generator().manual_seed(rows + cols))
    w.view(-1)[::13] = -0.0
    got = ops.tile_d8(w.to(DEV)).cpu().numpy()
    assert np.array_equal(got, core.tile_signs_d8(w.numpy()))


@pytest.mark.parametrize("H,F,tokens", [(2560, 9728, 16), (2560, 9728, 1), (2560, 9728, 9), (64, 96, 5),
                                        (96, 160, 16), (32, 32, 3), (256, 512, 12)])
def test_fused_block_against_oracle(ops, H, F, tokens):
    """Without the rms the input codes are the oracle's exactly: the hidden state
    matches to rounding of silu, and the down projection of the kernel's own
    hidden state is bit-exact (exact integer dot, the reference's op order)."""
    p = he4_case(H, F, seed=H + F + tokens)
    ffn = pack(ops, p)
    assert ffn.signs_down_d8 is not None
    rng = np.random.default_rng(tokens)
    x = rng.standard_normal((tokens, H)).astype(np.float32)
    res = rng.standard_normal((tokens, H)).astype(np.float32)
    y, h = ops.ffn_he4(dev(x), ffn, dev(res), hidden_out=True, fused=True)
    torch.cuda.synchronize()
    g = core.projection_forward(x, **{k: p["gate"][k] for k in FIELDS}, bits=4)
    u = core.projection_forward(x, **{k: p["up"][k] for k in FIELDS}, bits=4)
    assert rel(h.cpu().numpy(), (core.silu(g) * u).astype(np.float32)) < 1e-6
    down = core.projection_forward(h.cpu().numpy(), **{k: p["down"][k] for k in FIELDS}, bits=8)
    assert np.array_equal(y.cpu().numpy(), (res + down).astype(np.float32))
    want = core.he4_ffn(x, res, p["gate"], p["up"], p["down"])
    assert rel(y.cpu().numpy() - res, want - res) < 1e-3


@pytest.mark.parametrize("tokens", [16, 4])
def test_fused_block_with_rms_matches_three_kernel_path_twice(ops, tokens):
    """The drafter's call (rms of the residual stream inside the block): the
    two-launch block against the three-kernel block on the same operands, two
    calls in a row (the accumulator and counters are left zeroed)."""
    H, F = 2560, 9728
    p = he4_case(H, F, seed=7, bounds=(4.0, 1.0))
    ffn = pack(ops, p)
    rng = np.random.default_rng(3)
    x = dev(rng.standard_normal((tokens, H)).astype(np.float32))
    norm = dev((1 + 0.1 * rng.standard_normal(H)).astype(np.float32))
    base = ops.ffn_he4(x, ffn, x, norm=norm, epsilon=1e-6, fused=False)
    first = ops.ffn_he4(x, ffn, x, norm=norm, epsilon=1e-6, fused=True)
    second = ops.ffn_he4(x, ffn, x, norm=norm, epsilon=1e-6, fused=True)
    torch.cuda.synchronize()
    assert torch.equal(first, second)
    xr = x.cpu().numpy()
    assert rel(first.cpu().numpy() - xr, base.cpu().numpy() - xr) < 1e-3
    # against the oracle: rms, then the HE4 composition
    n = core.rms(xr, norm.cpu().numpy(), 1e-6)
    want = core.he4_ffn(n, xr, p["gate"], p["up"], p["down"])
    assert rel(first.cpu().numpy() - xr, want - xr) < 1e-2


def test_fused_block_reports_nonfinite_input(ops):
    p = he4_case(64, 96, seed=1)
    ffn = pack(ops, p)
    x = torch.zeros((2, 64), device=DEV)
    x[1, 5] = float("inf")
    with pytest.raises(ValueError):
        ops.ffn_he4(x, ffn, x, fused=True)
    # the workspace is still left clean for the next call
    x[1, 5] = 0.5
    y = ops.ffn_he4(x, ffn, x, fused=True)
    base = ops.ffn_he4(x, ffn, x, fused=False)
    assert torch.equal(y, base)
