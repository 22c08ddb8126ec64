"""Split-K of the bf16 split products (``bd_gemm_bf16_split3``): a product whose
128 x 256 output tiles leave most of the GPU idle is cut into K slices whose fp32
partial tiles the last slice adds in slice order.  Checked against a float64
product, against the same call without a workspace (unsplit), and for
run-to-run determinism; the workspace counters are left zero."""

from __future__ import annotations

import pytest
import torch

from conftest import package, submodule

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def mods():
    package()
    return submodule("_lib"), submodule("model")


def product(lib, model, x, b, workspace):
    m, k = x.shape
    n = b.shape[0]
    x_hi, x_lo, ld = model._split(x)
    b_hi, b_lo, ld_b = model._split(b)
    out = torch.empty((m, n), dtype=torch.float32, device=DEV)
    ws, nbytes = workspace
    lib.call("bd_gemm_bf16_split3", x_hi.data_ptr(), x_lo.data_ptr(), m, k, ld, b_hi.data_ptr(), b_lo.data_ptr(), n,
             ld_b, out.data_ptr(), n, ws, nbytes, torch.cuda.current_stream().cuda_stream)
    return out


@pytest.mark.parametrize("shape", [(480, 2560, 20000), (512, 2560, 9728), (100, 300, 4000)])
def test_split_k_matches_float64_and_unsplit(mods, shape):
    lib, model = mods
    m, n, k = shape
    nbytes = int(lib.load().bd_gemm_split_workspace_bytes(m, n, k, 3))
    assert nbytes > 0  # these shapes leave most SMs idle: they are split
    g = torch.Generator().manual_seed(m + n + k)
    x = torch.randn((m, k), generator=g)
    b = torch.randn((n, k), generator=g) * 0.02
    ref = (x.double() @ b.double().T)
    xd, bd = x.to(DEV), b.to(DEV)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    split = product(lib, model, xd, bd, (ws.data_ptr(), nbytes))
    again = product(lib, model, xd, bd, (ws.data_ptr(), nbytes))
    plain = product(lib, model, xd, bd, (None, 0))
    torch.cuda.synchronize()
    err_split = (split.double().cpu() - ref)
    err_plain = (plain.double().cpu() - ref)
    # split bf16 (lo x lo left out) with the tensor cores' fp32 accumulation over
    # up to 3 x 20000 products: a few 1e-5 of the result in norm.  Slicing K
    # shortens the accumulation chains and adds the slices in IEEE fp32: no worse.
    assert float(err_split.norm() / ref.norm()) < 1e-4
    assert float(err_split.norm()) <= 1.05 * float(err_plain.norm())
    assert float(err_split.abs().max()) <= 1.5 * float(err_plain.abs().max())
    assert torch.equal(split, again)
    counters = ws[: ((m + 127) // 128) * ((n + 255) // 256) * 8 * 4].view(torch.int32)
    assert int(counters.abs().sum()) == 0


def test_split_k_workspace_shared_across_shapes(mods):
    """One workspace serves products of different shapes in turn (the partial sums
    of one call never land where the next keeps its counters)."""
    lib, model = mods
    shapes = [(40, 2560, 9728), (300, 2560, 9728), (100, 300, 4000), (300, 2560, 9728)]
    nbytes = max(int(lib.load().bd_gemm_split_workspace_bytes(m, n, k, 3)) for m, n, k in shapes)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=DEV)
    g = torch.Generator().manual_seed(7)
    for m, n, k in shapes:
        x = torch.randn((m, k), generator=g).to(DEV)
        b = (torch.randn((n, k), generator=g) * 0.02).to(DEV)
        split = product(lib, model, x, b, (ws.data_ptr(), nbytes))
        plain = product(lib, model, x, b, (None, 0))
        torch.cuda.synchronize()
        ref = (x.double() @ b.double().T)
        assert float((split.double() - ref).norm()) <= 1.05 * float((plain.double() - ref).norm()), (m, n, k)
