"""Greedy acceptance through the allocation-free entry point (needs a B200).

``bd_accept_greedy_noalloc`` serves callers that cannot allocate device memory
(a verifier living inside a serving runtime that only lends it a stream and
tensor pointers): its scratch is a fixed device array inside the library.  Its
results are checked against the CPU oracle of the reference's greedy rule and
against the workspace entry point, on calls made back to back.  This file is
collected last so that a run stopping at the first failure has run every other
test first; it also passes alone in a fresh process.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import package
from oracle import acceptance

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")
TOO_LARGE = 6


def planted(logits: torch.Tensor, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    B, P, V = logits.shape
    targets = logits.float().argmax(-1).numpy()
    drafts = rng.integers(0, V, size=(B, P - 1)).astype(np.int32)
    for b in range(B):
        cut = int(rng.integers(0, P))
        drafts[b, :cut] = targets[b, :cut]
    return drafts


def with_workspace(lib, logits, drafts, eog):
    B, P, V = logits.shape
    n = P - 1
    acc = torch.empty(B, dtype=torch.int32, device=DEV)
    nxt = torch.empty(B, dtype=torch.int32, device=DEV)
    tg = torch.empty(B * P, dtype=torch.int32, device=DEV)
    ws = torch.zeros(int(lib.load().bd_accept_workspace_bytes(B, n)), dtype=torch.uint8, device=DEV)
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    lib.call("bd_accept_greedy", logits.data_ptr(), B, n, V, drafts.data_ptr(), eog.data_ptr(), eog.numel(),
             acc.data_ptr(), nxt.data_ptr(), tg.data_ptr(), ws.data_ptr(), ws.numel(), flags.data_ptr(),
             torch.cuda.current_stream().cuda_stream)
    return acc, nxt, tg, flags


def without_allocation(lib, logits, drafts, eog, targets: bool):
    B, P, V = logits.shape
    acc = torch.empty(B, dtype=torch.int32, device=DEV)
    nxt = torch.empty(B, dtype=torch.int32, device=DEV)
    tg = torch.empty(B * P, dtype=torch.int32, device=DEV) if targets else None
    flags = torch.zeros(1, dtype=torch.int32, device=DEV)
    lib.call("bd_accept_greedy_noalloc", logits.data_ptr(), B, P - 1, V, drafts.data_ptr(), eog.data_ptr(),
             eog.numel(), acc.data_ptr(), nxt.data_ptr(), None if tg is None else tg.data_ptr(), flags.data_ptr(),
             torch.cuda.current_stream().cuda_stream)
    return acc, nxt, tg, flags


def test_noalloc_greedy_matches_workspace_entry_point_twice():
    lib = package()._lib
    shapes = [(32, 17, 151936, 5), (7, 4, 1001, 11)]
    for call, (B, P, V, seed) in enumerate(shapes):
        logits = (torch.randn((B, P, V), generator=torch.Generator().manual_seed(seed)) * 3).to(torch.bfloat16)
        drafts = torch.from_numpy(planted(logits, seed + 1))
        eog = torch.tensor([int(drafts[0, 0]), V - 1], dtype=torch.int32)
        ld, dd, ed = logits.to(DEV), drafts.to(DEV), eog.to(DEV)
        ref = with_workspace(lib, ld, dd, ed)
        got = without_allocation(lib, ld, dd, ed, targets=call == 0)
        torch.cuda.synchronize()
        bits = logits.view(torch.int16).numpy().view(np.uint16)
        want_acc, want_next, want_tg = acceptance.accept_greedy(acceptance.bf16_to_f32(bits), drafts.numpy(),
                                                                eog.tolist())
        assert np.array_equal(got[0].cpu().numpy(), want_acc), call
        assert np.array_equal(got[1].cpu().numpy(), want_next), call
        if got[2] is not None:
            assert np.array_equal(got[2].cpu().numpy().reshape(B, P), want_tg)
        assert torch.equal(got[0], ref[0]) and torch.equal(got[1], ref[1]), call
        if got[2] is not None:
            assert torch.equal(got[2], ref[2])
        assert int(got[3].item()) == 0 and int(ref[3].item()) == 0
    # the same inputs again: the shared scratch keeps no state between calls
    again = without_allocation(lib, ld, dd, ed, targets=False)
    torch.cuda.synchronize()
    assert np.array_equal(again[0].cpu().numpy(), want_acc) and np.array_equal(again[1].cpu().numpy(), want_next)
    assert torch.equal(again[0], ref[0]) and torch.equal(again[1], ref[1])


def test_noalloc_greedy_rejects_sizes_beyond_its_scratch():
    lib = package()._lib
    logits = torch.zeros((257, 2, 8), dtype=torch.bfloat16, device=DEV)
    drafts = torch.zeros((257, 1), dtype=torch.int32, device=DEV)
    out = torch.zeros(257, dtype=torch.int32, device=DEV)
    status = lib.load().bd_accept_greedy_noalloc(logits.data_ptr(), 257, 1, 8, drafts.data_ptr(), None, 0,
                                                 out.data_ptr(), out.data_ptr(), None, None,
                                                 torch.cuda.current_stream().cuda_stream)
    assert status == TOO_LARGE
    assert b"scratch capacity" in lib.load().bd_status_string(status)
    logits = torch.zeros((1, 34, 8), dtype=torch.bfloat16, device=DEV)
    drafts = torch.zeros((1, 33), dtype=torch.int32, device=DEV)
    status = lib.load().bd_accept_greedy_noalloc(logits.data_ptr(), 1, 33, 8, drafts.data_ptr(), None, 0,
                                                 out.data_ptr(), out.data_ptr(), None, None,
                                                 torch.cuda.current_stream().cuda_stream)
    assert status == TOO_LARGE
