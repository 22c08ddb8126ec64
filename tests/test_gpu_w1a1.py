"""W1A1 kernels on the GPU: bit-exact sign words, mean|x|, +-1 dots (popcounts)
and projection outputs; SwiGLU block within tolerance (needs a B200)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN, package
from oracle import core

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
H, F = 2560, 9728


@pytest.fixture(scope="module")
def ops():
    return package().ops


def randn(shape, seed, std=1.0):
    return torch.randn(shape, generator=torch.Generator().manual_seed(seed)) * std


@pytest.mark.parametrize("rows,cols", [(1, 1), (5, 31), (37, 2600), (16, 9728)])
def test_binarize_rows_words_and_mean_bit_exact(ops, rows, cols):
    x = randn((rows, cols), rows * 7 + cols)
    x.view(-1)[::11] = 0.0
    x.view(-1)[5::13] = -0.0
    words, mean = ops.binarize_rows(x.to(DEV))
    want = core.pack_bits_rows(x.numpy()).view(np.int32)
    assert np.array_equal(words.cpu().numpy(), want)
    assert np.array_equal(mean.cpu().numpy(), core.fixed_mean_abs(x.numpy()))
    # the popcount identity on the packed words, against the +-1 dot
    w = randn((3, cols), 99)
    dots = core.popcount_dot(want.view(np.uint32), core.pack_bits_rows(w.numpy()), cols)
    xs, ws = np.where(x.numpy() >= 0, 1, -1), np.where(w.numpy() >= 0, 1, -1)
    assert np.array_equal(dots, xs @ ws.T)


def test_binarize_rejects_nonfinite(ops):
    x = torch.zeros((2, 64))
    x[1, 3] = float("inf")
    with pytest.raises(ValueError, match="nonfinite quantizer input"):
        ops.binarize_rows(x.to(DEV))


@pytest.mark.parametrize("tokens,out_f,in_f", [(16, F, H), (40, H, F), (3, 77, 300)])
def test_projection_w1a1_dots_and_outputs_bit_exact(ops, tokens, out_f, in_f):
    x = randn((tokens, in_f), 4)
    latent = randn((out_f, in_f), 1, 0.02)
    scale = latent.abs().mean(-1)
    signs = ops.tile_t16(latent.to(DEV))
    y, raw = ops.projection_w1a1(x.to(DEV), signs, scale.to(DEV), raw_dot=True)
    want_y, want_d, _ = core.w1a1_projection(x.numpy(), latent.numpy(), scale.numpy())
    assert np.array_equal(raw.cpu().numpy(), want_d)
    assert np.array_equal(y.cpu().numpy(), want_y)


@pytest.mark.parametrize("tokens", [16, 1024])
def test_ffn_w1a1_config3_shapes(ops, tokens):
    x = randn((tokens, H), 4)
    gate, up, down = randn((F, H), 1, 0.02), randn((F, H), 2, 0.02), randn((H, F), 3, 0.02)
    ffn = ops.pack_ffn(gate.to(DEV), up.to(DEV), down.to(DEV))
    y, h = ops.ffn_w1a1(x.to(DEV), ffn, hidden_out=True)
    want, dots = core.w1a1_ffn(x.numpy(), gate.numpy(), up.numpy(), down.numpy())
    hidden = dots["hidden"]
    err_h = np.linalg.norm(h.cpu().numpy() - hidden) / np.linalg.norm(hidden)
    err_y = np.linalg.norm(y.cpu().numpy() - want) / np.linalg.norm(want)
    assert err_h < 1e-5, err_h
    assert err_y < 1e-2, err_y
    # the down projection re-binarises the kernel's own hidden: its dots are exact
    _, raw = ops.projection_w1a1(h, ops.tile_t16(down.to(DEV)), ffn.scale_down, raw_dot=True)
    _, want_d, _ = core.w1a1_projection(h.cpu().numpy(), down.numpy(), ffn.scale_down.cpu().numpy())
    assert np.array_equal(raw.cpu().numpy(), want_d)


@pytest.mark.parametrize("repeat", [1, 40])
def test_ffn_w1a1_against_reference_fixture(ops, repeat):
    """The W1A1 block on the fixture made from the reference's hard_sign /
    packed_signs / linear: decode rows (5 tokens) and, repeated to 200 rows, the
    tcgen05 large-M path.  Gate and up dots are exact, so the hidden state equals
    the fixture's to the last bit of the fixed-order mean; y within 1e-5."""
    f = np.load(GOLDEN / "w1a1_ffn.npz")
    x = torch.from_numpy(np.tile(f["x"], (repeat, 1)))
    gate, up, down = (torch.from_numpy(f[k]).to(DEV) for k in ("w_gate", "w_up", "w_down"))
    ffn = ops.pack_ffn(gate, up, down, large=repeat > 1)
    y, h = ops.ffn_w1a1(x.to(DEV), ffn, hidden_out=True)
    want_h, want_y = np.tile(f["hidden"], (repeat, 1)), np.tile(f["y"], (repeat, 1))
    np.testing.assert_allclose(h.cpu().numpy(), want_h, rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(y.cpu().numpy(), want_y, rtol=1e-5, atol=1e-7)
    _, raw = ops.projection_w1a1(x[:5].to(DEV), ops.tile_t16(gate), ffn.scale_gate, raw_dot=True)
    assert np.array_equal(raw.cpu().numpy(), f["gate_dot"])
