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


def test_schedule_multiplier(qat):
    assert qat.Schedule().multiplier(0) == 1.0
    warm = qat.Schedule(warmup_updates=4)
    assert [warm.multiplier(u) for u in range(6)] == [0.25, 0.5, 0.75, 1.0, 1.0, 1.0]
    cos = qat.Schedule(decay="cosine", warmup_updates=2, start_update=1, final_update=11)
    assert cos.multiplier(1) == 0.5 and cos.multiplier(2) == 1.0
    assert cos.multiplier(3) == pytest.approx(1.0)
    assert cos.multiplier(7) == pytest.approx(0.5 * (1 + math.cos(math.pi * 4 / 8)))
    with pytest.raises(ValueError, match="update precedes the schedule start"):
        cos.multiplier(0)
    with pytest.raises(ValueError, match="at or beyond the schedule's final update"):
        cos.multiplier(11)
    with pytest.raises(ValueError, match="constant or cosine"):
        qat.Schedule(decay="linear")
    with pytest.raises(ValueError, match="a constant schedule has no final update"):
        qat.Schedule(final_update=3)
    with pytest.raises(ValueError, match="cosine decay requires a final update"):
        qat.Schedule(decay="cosine", warmup_updates=3, final_update=3)


def test_optimization_validation(qat):
    assert qat.Optimization().step_sizes == {"sign": 1e-3, "scale": 1e-5, "midpoint": 1e-5, "gain": 1e-5,
                                             "clip": 1e-5, "norm": 1e-5}
    with pytest.raises(ValueError, match="positive finite step sizes"):
        qat.Optimization(step_sizes={"sign": 1e-3})
    with pytest.raises(ValueError, match="positive finite step sizes"):
        qat.Optimization(step_sizes={**qat.default_step_sizes(), "sign": 0.0})
    with pytest.raises(ValueError, match="bounded latent scale requires"):
        qat.Optimization(latent_multiple=-1.0)


def test_label_weights(qat):
    w = qat.label_weights((3, 1))
    first = torch.exp(-torch.arange(3) / 7)
    torch.testing.assert_close(w[:3], first / first.sum() / 2)
    assert w[3].item() == pytest.approx(0.5)
    assert w.sum().item() == pytest.approx(1.0)
    p = qat.label_weights((2,), (1.0, 3.0, 5.0))
    torch.testing.assert_close(p, torch.tensor([0.25, 0.75]))


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


def test_average_gradients_without_process_group_is_a_no_op(qat):
    p = nn.Parameter(torch.zeros(3))
    p.grad = torch.ones(3)
    qat.average_gradients([p])
    assert torch.equal(p.grad, torch.ones(3))
