"""Data-parallel QAT over NCCL on two GPUs (skipped with fewer): the overlapped
bucketed gradient exchange equals the mean of the ranks' own gradients (also with
the latent gradients deferred to ``LatentGradients``), and one ``qat.update``
leaves every rank with the same parameters."""

from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import package, submodule

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _windows(qat, rank):
    if rank == 0:
        return (qat.Window(3, (4, 5, 6)), qat.Window(10, (11, 12, 13, 14, 15)))
    return (qat.Window(5, (6, 7, 8, 9)), qat.Window(12, (13, 14)))


def _rank_main(rank: int, world: int, port: int, out) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=dev)
    try:
        from test_gpu_model import tiny_model

        bd = package()
        qat = submodule("qat")
        f, model = tiny_model(bd, 4096)
        model = model.to(dev)
        features = torch.from_numpy(f["features"]).to(dev)
        tokens = tuple(range(20))
        windows = _windows(qat, rank)
        params = [p for p in model.parameters() if p.requires_grad]

        # the rank's own gradients
        qat.group_loss(model, features, tokens, windows, 6)
        own = [p.grad.clone() for p in params]
        model.zero_grad()
        # the same backward with the overlapped exchange armed (small buckets: several all-reduces)
        exchange = qat.GradientExchange(params, bucket_bytes=256)
        exchange.armed = True
        qat.group_loss(model, features, tokens, windows, 6)
        exchange.finish()
        exchanged = [p.grad.clone() for p in params]
        exchange.remove()
        # the same with the latent gradients written by one product at the end of the
        # block (LatentGradients) and handed to the exchange as they are written
        model.zero_grad()
        exchange = qat.GradientExchange(params, bucket_bytes=256)
        exchange.armed = True
        with bd.LatentGradients(model, 64, on_ready=exchange.ready):
            qat.group_loss(model, features, tokens, windows, 6)
        exchange.finish()
        deferred = max(float((d.grad - e).abs().max() / e.abs().max().clamp_min(1e-30))
                       for d, e in zip(params, exchanged))
        exchange.remove()
        gathered = []
        for g in own:
            parts = [torch.empty_like(g) for _ in range(world)]
            dist.all_gather(parts, g)
            gathered.append(sum(parts) / world)
        worst = max(float((e - m).abs().max() / m.abs().max().clamp_min(1e-30)) for e, m in zip(exchanged, gathered))

        # one whole update (averaged gradients, clip, AdamW, re-pack) on every rank
        opt = qat.BitAdamW(model)
        loss, norm = qat.update(model, opt, features, tokens, windows, slots=6)
        flat = torch.cat([p.detach().reshape(-1) for p in model.parameters()])
        copies = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(copies, flat)
        same = all(torch.equal(c, copies[0]) for c in copies)
        out[rank] = (worst, exchange.buckets, same, loss, norm, deferred)
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_qat_gradient_exchange_two_nccl_ranks():
    package()  # the extension must load before ranks start
    port = _free_port()
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_rank_main, args=(2, port, out), nprocs=2, join=True)
    for rank in range(2):
        worst, buckets, same, loss, norm, deferred = out[rank]
        assert buckets >= 2, buckets
        assert deferred <= 1e-6, (rank, deferred)
        assert worst <= 1e-6, (rank, worst)  # the kernels reduce in fixed order: same sums, same rounding
        assert same, rank
        assert torch.isfinite(torch.tensor([loss, norm])).all()
