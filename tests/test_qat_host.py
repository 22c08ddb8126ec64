"""Host logic of the QAT update (no GPU): schedule, step sizes, label weights,
parameter grouping, and the data-parallel gradient average over gloo ranks."""

from __future__ import annotations

import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

from conftest import submodule


@pytest.fixture(scope="module")
def qat():
    return submodule("qat")


def test_update_policy_defaults_and_duck_typing(qat):
    """The optimizer reads step sizes, a schedule multiplier and the latent bound
    from the caller's Optimization object; the default has the reference's
    step sizes (training.py:108-109) and a constant schedule."""
    policy = qat.UpdatePolicy()
    assert policy.step_sizes == {"sign": 1e-3, "scale": 1e-5, "midpoint": 1e-5, "gain": 1e-5, "clip": 1e-5,
                                 "norm": 1e-5}
    assert policy.schedule.multiplier(0) == 1.0 and policy.schedule.multiplier(12345) == 1.0
    assert policy.latent_multiple is None

    class Halving:
        def multiplier(self, updates):
            return 0.5 ** updates

    class CallerOptimization:  # the reference's Optimization, as the optimizer sees it
        step_sizes = {**qat.REFERENCE_STEP_SIZES, "sign": 2e-3}
        schedule = Halving()
        latent_multiple = None

    model = nn.Module()
    model.norm = nn.Parameter(torch.zeros(2))
    opt = qat.BitAdamW(model, CallerOptimization())
    opt.set_multiplier(opt.optimization.schedule.multiplier(2))
    assert opt.lr["sign"] == pytest.approx(5e-4) and opt.lr["norm"] == pytest.approx(2.5e-6)

    class Partial:
        step_sizes = {"sign": 1e-3}
        schedule = Halving()
        latent_multiple = None

    with pytest.raises(ValueError, match="every parameter group"):
        qat.BitAdamW(model, Partial())


def test_label_weights(qat):
    w = qat.label_weights((3, 1))
    first = torch.exp(-torch.arange(3) / 7)
    torch.testing.assert_close(w[:3], first / first.sum() / 2)
    assert w[3].item() == pytest.approx(0.5)
    assert w.sum().item() == pytest.approx(1.0)
    p = qat.label_weights((2,), (1.0, 3.0, 5.0))
    torch.testing.assert_close(p, torch.tensor([0.25, 0.75]))
    many = qat.label_weights((15, 7, 1, 15))
    for at, n in ((0, 15), (15, 7), (22, 1), (23, 15)):
        assert many[at:at + n].sum().item() == pytest.approx(0.25)
    with pytest.raises(ValueError):
        qat.label_weights((2, 0))


def test_parameter_groups_by_suffix(qat):
    class P(nn.Module):
        def __init__(self):
            super().__init__()
            for name in ("latent_sign", "scale", "midpoint", "log_gain", "log_clip", "attn_norm"):
                setattr(self, name, nn.Parameter(torch.zeros(2)))

    m = nn.Module()
    m.a = P()
    m.frozen = nn.Parameter(torch.zeros(1), requires_grad=False)
    groups = qat.parameter_groups(m)
    assert {k: [n for n, _ in v] for k, v in groups.items()} == {
        "sign": ["a.latent_sign"], "scale": ["a.scale"], "midpoint": ["a.midpoint"], "gain": ["a.log_gain"],
        "clip": ["a.log_clip"], "norm": ["a.attn_norm"]}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out: dict) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        qat = submodule("qat")
        params = [nn.Parameter(torch.zeros(s)) for s in ((3, 4), (5,), (1000,))]
        for i, p in enumerate(params):
            p.grad = torch.full(p.shape, float(rank + 1) * (i + 1))
        # a small bucket size forces several all-reduces
        qat.average_gradients(params, bucket_bytes=64)
        out[rank] = [p.grad.clone() for p in params]
    finally:
        dist.destroy_process_group()


def test_average_gradients_two_gloo_ranks(qat):
    port = _free_port()
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_rank_main, args=(2, port, out), nprocs=2, join=True)
    for rank in range(2):
        for i, g in enumerate(out[rank]):
            assert torch.all(g == 1.5 * (i + 1)), (rank, i)


def _exchange_rank_main(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        qat = submodule("qat")
        torch.manual_seed(0)
        model = nn.Sequential(nn.Linear(6, 5), nn.Tanh(), nn.Linear(5, 3))
        params = list(model.parameters())
        exchange = qat.GradientExchange(params, bucket_bytes=32)  # several buckets
        x = torch.randn(4, 6, generator=torch.Generator().manual_seed(10 + rank))
        for step in range(2):  # two backward passes; only the last one is exchanged
            exchange.armed = step == 1
            model(x * (step + 1)).square().sum().backward()
        exchange.finish()
        out[rank] = ([p.grad.clone() for p in params], exchange.buckets)
    finally:
        dist.destroy_process_group()


def test_gradient_exchange_overlapped_two_gloo_ranks(qat):
    """The hook-driven exchange equals the average of the ranks' accumulated
    gradients, reduced in several buckets during the last backward pass."""
    port = _free_port()
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_exchange_rank_main, args=(2, port, out), nprocs=2, join=True)
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(6, 5), nn.Tanh(), nn.Linear(5, 3))
    expected = [torch.zeros_like(p) for p in model.parameters()]
    for rank in range(2):
        model.zero_grad()
        x = torch.randn(4, 6, generator=torch.Generator().manual_seed(10 + rank))
        for step in range(2):
            model(x * (step + 1)).square().sum().backward()
        for e, p in zip(expected, model.parameters()):
            e += p.grad / 2
    for rank in range(2):
        grads, buckets = out[rank]
        assert buckets >= 2
        for g, e in zip(grads, expected):
            torch.testing.assert_close(g, e)


def test_average_gradients_without_process_group_is_a_no_op(qat):
    p = nn.Parameter(torch.zeros(3))
    p.grad = torch.ones(3)
    qat.average_gradients([p])
    assert torch.equal(p.grad, torch.ones(3))


def test_latent_gradients_context_bookkeeping():
    """``LatentGradients`` host side: it owns the model's projections only, refuses a
    non-positive size, and leaves the active-context stack clean on exit, also
    when the block raises (nothing pending is flushed then)."""
    model_mod = submodule("model")
    gain, clip = nn.Parameter(torch.zeros(8)), nn.Parameter(torch.tensor(0.0))
    inner = model_mod.Projection(torch.randn(4, 8), 4, gain, clip)
    other = model_mod.Projection(torch.randn(4, 8), 4, gain, clip)
    holder = nn.Module()
    holder.proj = inner
    with pytest.raises(ValueError):
        model_mod.LatentGradients(holder, 0)
    acc = model_mod.LatentGradients(holder, 13)
    assert acc.rows == 16 and acc.owns(inner) and not acc.owns(other)
    with acc:
        assert model_mod._LATENT == [acc]
    assert model_mod._LATENT == []
    with pytest.raises(RuntimeError, match="boom"):
        with acc:
            raise RuntimeError("boom")
    assert model_mod._LATENT == [] and inner.latent_sign.grad is None


class _TableDrafter(nn.Module):
    """A stand-in for ``HE4`` exposing what the loss head uses: ``block``,
    ``group_hidden`` (here a trainable table of hidden states per anchor) and the
    frozen ``vocabulary``.  On CPU tensors the head is the reference's fp32 linear."""

    def __init__(self, anchors: int, slots: int, hidden: int, vocab: int, seed: int = 5) -> None:
        super().__init__()
        g = torch.Generator().manual_seed(seed)
        self.slots = slots
        self.table = nn.Parameter(torch.randn(anchors, slots, hidden, generator=g))
        self.register_buffer("vocabulary", torch.randn(vocab, hidden, generator=g))

    def block(self, slots):
        size = self.slots if slots is None else slots
        if type(size) is not int or not 1 <= size <= self.slots:
            raise ValueError("block size must be between one slot and the model's slots")
        return size

    def group_hidden(self, features, tokens, anchors, size):
        return self.table[list(anchors), :size]


def _closed_form_loss(model, windows, size, positions, scale):
    """Weighted cross-entropy of the label rows and its gradient w.r.t. the table, in fp64
    (``worker.py:41-50, 315-363``)."""
    table = model.table.detach().double()
    vocab = model.vocabulary.double()
    grad = torch.zeros_like(table)
    lengths = [min(len(labels), size - 1) for _, labels in windows]
    total = 0.0
    for (anchor, labels), length in zip(windows, lengths):
        if positions is None:
            w = torch.exp(-torch.arange(length, dtype=torch.float64) / 7)
        else:
            w = torch.tensor(positions[:length], dtype=torch.float64)
        w = w / w.sum() / len(windows) * scale
        for offset in range(length):
            row = table[anchor, 1 + offset]
            logits = vocab @ row
            p = torch.softmax(logits, 0)
            total += float(w[offset] * (torch.logsumexp(logits, 0) - logits[labels[offset]]))
            p[labels[offset]] -= 1
            grad[anchor, 1 + offset] += w[offset] * (vocab.t() @ p)
    return total, grad


@pytest.mark.parametrize("slots,positions,scale", [(6, None, 1.0), (None, tuple(0.9 ** i for i in range(15)), 0.5)])
def test_group_loss_bookkeeping_matches_closed_form(qat, slots, positions, scale):
    # 12 windows x up to 15 label rows: 150+ rows cross the 128-row head chunks
    model = _TableDrafter(anchors=24, slots=16, hidden=8, vocab=37)
    g = torch.Generator().manual_seed(11)
    windows = tuple((2 * i, tuple(int(v) for v in torch.randint(0, 37, (15 if i % 4 else 3,), generator=g)))
                    for i in range(12))
    size = model.block(slots)
    loss = qat.group_loss(model, torch.zeros(1), (), tuple(qat.Window(a, l) for a, l in windows), slots, positions,
                          scale)
    want, want_grad = _closed_form_loss(model, windows, size, positions, scale)
    assert float(loss) == pytest.approx(want, rel=1e-5)
    torch.testing.assert_close(model.table.grad.double(), want_grad, rtol=1e-4, atol=1e-6)


def test_group_loss_rejects_what_the_reference_rejects(qat):
    model = _TableDrafter(anchors=4, slots=16, hidden=4, vocab=7)
    with pytest.raises(ValueError, match="an update requires supervised windows"):
        qat.group_loss(model, torch.zeros(1), (), ())
    with pytest.raises(ValueError, match="an update requires supervised windows"):
        qat.group_loss(model, torch.zeros(1), (), (qat.Window(1, ()),))
    with pytest.raises(ValueError, match="an update requires at least one drafted position"):
        qat.group_loss(model, torch.zeros(1), (), (qat.Window(1, (2,)),), slots=1)
    with torch.no_grad():
        model.vocabulary[3] = float("inf")
    with pytest.raises(ValueError, match="nonfinite loss"):
        qat.group_loss(model, torch.zeros(1), (), (qat.Window(1, (2, 3)),), slots=4)
