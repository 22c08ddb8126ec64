"""Teacher-feature ingestion on the GPU (needs a B200): tap-major captures become
the token-major features of captures.py:124-137, bit-exact, with its finiteness check."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import package

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def ops():
    return package().ops


@pytest.mark.parametrize("taps,rows,hidden", [(8, 2048, 2560), (4, 1, 8), (3, 37, 24)])
@pytest.mark.parametrize("src_dtype", [np.float16, np.float32])
def test_tap_interleave_is_exact(ops, taps, rows, hidden, src_dtype):
    rng = np.random.default_rng(taps * 1000 + rows)
    caps = (rng.standard_normal((taps, rows, hidden)) * 4).astype(src_dtype)
    want = np.ascontiguousarray(caps.transpose(1, 0, 2)).reshape(rows, taps * hidden)
    for out_dtype in (torch.float16, torch.float32, torch.bfloat16):
        got = ops.ingest_taps(torch.from_numpy(caps).to(DEV), out_dtype)
        ref = torch.from_numpy(want).to(out_dtype)  # torch's own rounding (round to nearest even)
        assert torch.equal(got.cpu(), ref), out_dtype


def test_host_pinned_captures(ops):
    caps = torch.randn((4, 64, 2560)).half().pin_memory()
    got = ops.ingest_taps(caps, torch.float32, device=DEV)
    assert torch.equal(got.cpu(), caps.permute(1, 0, 2).reshape(64, 4 * 2560).float())


@pytest.mark.parametrize("bad", [float("nan"), float("inf"), float("-inf")])
def test_nonfinite_teacher_features(ops, bad):
    caps = torch.randn((8, 5, 16))
    caps[6, 3, 11] = bad
    for dtype in (torch.float16, torch.float32):
        with pytest.raises(ValueError, match="nonfinite teacher features"):
            ops.ingest_taps(caps.to(dtype).to(DEV))
