"""Tensor-core (tcgen05) large-M path on the GPU: exact integer dots on ragged shapes
and the W1A1 SwiGLU block at config-3 size (needs a B200)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import package
from oracle import core

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def ops():
    return package().ops


def codes_tensor(ops, codes):
    tokens, k = codes.shape
    ld = int(ops._lib.load().bd_i8_ld(k))
    buf = np.zeros((tokens, ld), np.int8)
    buf[:, :k] = codes
    return torch.from_numpy(buf).to(DEV), k


@pytest.mark.parametrize("tokens,k,outs", [(128, 128, 256), (1, 300, 77), (300, 2560, 1000), (1024, 2560, 512),
                                           (200, 9728, 384)])
def test_gemm_i8_exact(ops, tokens, k, outs):
    rng = np.random.default_rng(tokens + k + outs)
    codes = rng.integers(-127, 128, size=(tokens, k)).astype(np.int8)
    latent = rng.standard_normal((outs, k)).astype(np.float32)
    latent.reshape(-1)[::5] = -0.0
    signs = ops.tile_i8(torch.from_numpy(latent).to(DEV))
    cbuf, _ = codes_tensor(ops, codes)
    dots = ops.gemm_i8(cbuf, k, signs, outs)
    want = codes.astype(np.float64) @ np.where(latent >= 0, 1.0, -1.0).T
    assert np.array_equal(dots.cpu().numpy(), want.astype(np.int64))


def test_ffn_w1a1_large_config3(ops):
    H, F, M = 2560, 9728, 1024
    g = torch.Generator().manual_seed(4)
    x = torch.randn((M, H), generator=g)
    gate, up, down = (torch.randn(s, generator=torch.Generator().manual_seed(i)) * 0.02
                      for i, s in ((1, (F, H)), (2, (F, H)), (3, (H, F))))
    ffn = ops.pack_ffn(gate.to(DEV), up.to(DEV), down.to(DEV), large=True)
    y, h = ops.ffn_w1a1(x.to(DEV), ffn, hidden_out=True)
    want, dots = core.w1a1_ffn(x.numpy(), gate.numpy(), up.numpy(), down.numpy(), ffn.scale_gate.cpu().numpy(),
                               ffn.scale_up.cpu().numpy(), ffn.scale_down.cpu().numpy())
    hidden = dots["hidden"]
    assert np.linalg.norm(h.cpu().numpy() - hidden) / np.linalg.norm(hidden) < 1e-5
    assert np.linalg.norm(y.cpu().numpy() - want) / np.linalg.norm(want) < 1e-2
    # the down projection of the kernel's own hidden state: exact popcount dots and values
    _, want_d, s = core.w1a1_projection(h.cpu().numpy(), down.numpy(), ffn.scale_down.cpu().numpy())
    want_y = (want_d.astype(np.float32) * ffn.scale_down.cpu().numpy()) * s[:, None]
    assert np.array_equal(y.cpu().numpy(), want_y.astype(np.float32))
    # and the decode path (32-token chunks) gives the same block output
    y_small = ops.ffn_w1a1(x[:40].to(DEV), ops.pack_ffn(gate.to(DEV), up.to(DEV), down.to(DEV)))
    assert np.array_equal(y_small.cpu().numpy(), y[:40].cpu().numpy())


# (2048, 2560, 10240) and (1000, 8192, 2560): products that fill the GPU run on SM pairs
# (256-row tiles over two CTAs, tcgen05 cta_group::2); 1000 rows end inside a pair's second half
@pytest.mark.parametrize("m,n,k", [(512, 2560, 10240), (100, 200, 72), (1, 8, 8), (300, 2048, 5120),
                                   (2048, 2560, 10240), (1000, 8192, 2560)])
def test_gemm_bf16(ops, m, n, k):
    g = torch.Generator().manual_seed(m + n + k)
    a = torch.randn((m, k), generator=g).to(torch.bfloat16)
    b = torch.randn((n, k), generator=g).to(torch.bfloat16)
    got = ops.gemm_bf16(a.to(DEV), b.to(DEV)).cpu().double().numpy()
    want = a.double().numpy() @ b.double().numpy().T  # bf16 inputs are exact in float64
    # fp32 accumulation of up to 10240 products: relative error of the norm about 1e-5
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 3e-5
    assert np.abs(got - want).max() <= 1e-4 * np.abs(want).max() + 1e-6
