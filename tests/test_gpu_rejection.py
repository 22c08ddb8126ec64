"""Rejection sampling on the GPU: bit-exact against the contract's CPU restatement,
and statistically against the reference's sampler check (needs a B200)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import package
from oracle import acceptance

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def ops():
    return package().ops


def run_both(ops, target, draft, drafts, seed, offset=0, eog=()):
    eog_t = torch.tensor(list(eog), dtype=torch.int32, device=DEV) if eog else None
    acc, nxt = ops.accept_rejection(target.to(DEV), draft.to(DEV), torch.from_numpy(drafts).to(DEV), seed, offset,
                                    eog_t)
    w_acc, w_nxt = acceptance.accept_rejection(target.float().numpy(), draft.float().numpy(), drafts, seed, offset,
                                               eog)
    return acc.cpu().numpy(), nxt.cpu().numpy(), w_acc, w_nxt


def test_config4_bit_exact_with_acceptances_rejections_and_bonus(ops):
    B, n, V = 32, 16, 151936
    target = (torch.randn((B, n + 1, V), generator=torch.Generator().manual_seed(5)) * 3).to(torch.bfloat16)
    draft = (torch.randn((B, n, V), generator=torch.Generator().manual_seed(7)) * 3).to(torch.bfloat16)
    # requests 0..11 draft with the target's own distribution (accepted), 12..15 for a prefix
    draft[:12] = target[:12, :n]
    draft[12:16, :6] = target[12:16, :6]
    drafts = torch.randint(0, V, (B, n), generator=torch.Generator().manual_seed(6)).to(torch.int32).numpy()
    for b in range(16):  # draft the most likely tokens so acceptances are likely
        drafts[b] = target[b, :n].float().argmax(-1).numpy()
    acc, nxt, w_acc, w_nxt = run_both(ops, target, draft, drafts, seed=8)
    assert np.array_equal(acc, w_acc), (acc, w_acc)
    assert np.array_equal(nxt, w_nxt), (nxt, w_nxt)
    assert (acc == n).sum() >= 8 and (acc < n).sum() >= 8  # both paths exercised
    # another seed / offset changes the draw but stays bit-exact
    acc, nxt, w_acc, w_nxt = run_both(ops, target, draft, drafts, seed=(1 << 40) + 3, offset=17, eog=(int(drafts[2, 3]),))
    assert np.array_equal(acc, w_acc) and np.array_equal(nxt, w_nxt)


@pytest.mark.parametrize("V", [1, 7, 4097, 9000])
def test_small_and_ragged_vocabularies(ops, V):
    B, n = 6, 3
    g = torch.Generator().manual_seed(V)
    target = (torch.randn((B, n + 1, V), generator=g) * 2).to(torch.bfloat16)
    draft = (torch.randn((B, n, V), generator=g) * 2).to(torch.bfloat16)
    draft[:3] = target[:3, :n]
    drafts = torch.randint(0, V, (B, n), generator=g).to(torch.int32).numpy()
    acc, nxt, w_acc, w_nxt = run_both(ops, target, draft, drafts, seed=11)
    assert np.array_equal(acc, w_acc) and np.array_equal(nxt, w_nxt)


def test_zero_drafts_samples_the_bonus(ops):
    target = (torch.randn((4, 1, 3000), generator=torch.Generator().manual_seed(2)) * 2).to(torch.bfloat16)
    draft = torch.zeros((4, 0, 3000), dtype=torch.bfloat16)
    drafts = np.zeros((4, 0), np.int32)
    acc, nxt, w_acc, w_nxt = run_both(ops, target, draft, drafts, seed=3)
    assert not acc.any() and np.array_equal(nxt, w_nxt)


def test_eog_stop_case(ops):
    # native/verifier-test.cpp:84-97 of the reference: drafts [eos, eos] under a point mass
    lp = torch.full((1, 3, 8), -60.0)
    lp[..., 2] = 0.0
    target = lp.to(torch.bfloat16)
    draft = lp[:, :2].to(torch.bfloat16)
    acc, nxt, _, _ = run_both(ops, target, draft, np.array([[2, 2]], np.int32), seed=1, eog=(2,))
    assert (int(acc[0]), int(nxt[0])) == (0, 2)


def test_statistics_match_reference_sampler_check(ops):
    # native/verifier-test.cpp:43-80: marginals within 0.035 of p, acceptance within 0.035 of sum(min(p, q))
    cases = [((0.55, 0.35, 0.10), (0.10, 0.70, 0.20)), ((0.55, 0.35, 0.10), (1.00, 0.00, 0.00)),
             ((0.55, 0.35, 0.10), (0.55, 0.35, 0.10)), ((0.00, 0.60, 0.40), (0.50, 0.50, 0.00))]
    rng = np.random.default_rng(9101)
    trials = 20000
    for p, q in cases:
        p, q = np.array(p), np.array(q)
        lp = torch.tensor(np.where(p > 0, np.log(np.maximum(p, 1e-30)), -60.0), dtype=torch.float32)
        lq = torch.tensor(np.where(q > 0, np.log(np.maximum(q, 1e-30)), -60.0), dtype=torch.float32)
        drafts = rng.choice(3, size=(trials, 1), p=q).astype(np.int32)
        target = lp.expand(trials, 2, 3).contiguous().to(torch.bfloat16)
        draft = lq.expand(trials, 1, 3).contiguous().to(torch.bfloat16)
        acc, nxt = ops.accept_rejection(target.to(DEV), draft.to(DEV), torch.from_numpy(drafts).to(DEV), seed=8101)
        acc, nxt = acc.cpu().numpy(), nxt.cpu().numpy()
        first = np.where(acc == 1, drafts[:, 0], nxt)
        observed = np.bincount(first, minlength=3) / trials
        pb = torch.softmax(lp.to(torch.bfloat16).float(), 0).numpy()
        assert np.abs(observed - pb).max() <= 0.035, (p, q, observed)
        qb = torch.softmax(lq.to(torch.bfloat16).float(), 0).numpy()
        assert abs(acc.mean() - np.minimum(pb, qb).sum()) <= 0.035


def test_nonfinite_logits_and_bad_tokens_raise(ops):
    target = torch.zeros((1, 2, 16), dtype=torch.bfloat16)
    draft = torch.zeros((1, 1, 16), dtype=torch.bfloat16)
    target[0, 1, 3] = float("nan")
    with pytest.raises(ValueError, match="nonfinite verifier logits"):
        ops.accept_rejection(target.to(DEV), draft.to(DEV), torch.zeros((1, 1), dtype=torch.int32, device=DEV), 1)
    target[0, 1, 3] = 0.0
    with pytest.raises(ValueError, match="outside the vocabulary"):
        ops.accept_rejection(target.to(DEV), draft.to(DEV), torch.full((1, 1), 99, dtype=torch.int32, device=DEV), 1)
