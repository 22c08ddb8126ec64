#!/usr/bin/env python
"""Drafted tokens/s of the 4-layer block-16 HE4 drafter on B200.

One step = one serving draft round on a resident 4096-position context:
ingest 16 new context rows (fusion + per-layer context K/V into the fp16
cache), then the 4-layer block forward over 4096 + 16 keys, the tied LM head
and the per-slot argmax -> 15 drafted tokens.  Geometry of the headline
workload: hidden 2560, FFN inner 9728 (one-bit SwiGLU, HE4 A4/A8 codes), 32 q /
8 kv heads of 128, RoPE theta 1e6, window 4096, taps 4, vocabulary 151936,
batch 1 per GPU.  Weights are random N(0, 0.02) (bf16-representable), features
N(0, 1); there is no network for checkpoints.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Multi-GPU (torchrun, one process per GPU): every rank serves its own request
(data parallel by request, no collective on the data path) -> weak scaling;
time = max over ranks of the device-timed region.
"""

from __future__ import annotations

import argparse
import datetime
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "drafted tokens/s/GPU (block-16 HE4 drafter)"
UNIT = "drafted tokens/s"
GEOMETRY = dict(hidden=2560, intermediate=9728, heads=32, kv_heads=8, head_dim=128, layers=4, slots=16, taps=4,
                window=4096, epsilon=1e-6, theta=1e6)
VOCAB = 151936
CONTEXT = 4096
SLOTS = 16
INGEST = 16
PEAKS = ROOT / "MEASURED_PEAKS.json"


def workload_config() -> dict:
    return {
        "workload": "HE4 block drafter round: ingest 16 context rows + 4-layer block-16 forward over 4096+16 keys "
                    "+ tied LM head argmax (15 drafted tokens), batch 1 per GPU",
        "hidden": 2560, "ffn_inner": 9728, "layers": 4, "heads": 32, "kv_heads": 8, "head_dim": 128, "taps": 4,
        "vocab": VOCAB, "context": CONTEXT, "slots": SLOTS, "ingest_rows": INGEST, "theta": 1e6, "window": 4096,
        "ffn": "one-bit signs, HE4 A4 gate/up + A8 down codes",
        "l2": "inputs larger than L2: every step streams ~1.17 GB of weights (L2 126 MB)",
    }


def make_tensors(seed: int = 0):
    """Random-init drafter tensors keyed by the reference's GGUF names (CPU, fp32, bf16-exact)."""
    cfg = GEOMETRY
    H, F, d = cfg["hidden"], cfg["intermediate"], cfg["head_dim"]
    g = torch.Generator().manual_seed(seed)

    def w(*shape):
        return (torch.randn(shape, generator=g) * 0.02).to(torch.bfloat16).float()

    tensors = {"fc.weight": w(H, cfg["taps"] * H), "enc.output_norm.weight": torch.ones(H),
               "output_norm.weight": torch.ones(H)}
    for i in range(cfg["layers"]):
        p = f"blk.{i}."
        tensors.update({
            p + "attn_norm.weight": torch.ones(H), p + "attn_q_norm.weight": torch.ones(d),
            p + "attn_k_norm.weight": torch.ones(d), p + "ffn_norm.weight": torch.ones(H),
            p + "attn_q.weight": w(cfg["heads"] * d, H), p + "attn_k.weight": w(cfg["kv_heads"] * d, H),
            p + "attn_v.weight": w(cfg["kv_heads"] * d, H), p + "attn_output.weight": w(H, cfg["heads"] * d),
            p + "ffn_gate.weight": w(F, H), p + "ffn_up.weight": w(F, H), p + "ffn_down.weight": w(H, F),
        })
    vocabulary = w(VOCAB, H)
    features = torch.randn((CONTEXT + SLOTS, cfg["taps"] * H), generator=g).to(torch.bfloat16)
    tokens = torch.randint(0, VOCAB, (CONTEXT + SLOTS,), generator=g)
    return tensors, vocabulary, features, tokens


def peaks() -> tuple[float, str]:
    try:
        return float(json.loads(PEAKS.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# --------------------------------------------------------------------------- CPU (oracle) arm


def cpu_round_rate(tensors, vocabulary, features, tokens, steps: int, budget_s: float = 30.0):
    """The CPU restatement of the same draft round (cached context), drafted tokens/s."""
    from oracle import drafter as od

    cfg = od.Geometry(**GEOMETRY)
    t = {k: v.numpy() for k, v in tensors.items()}
    for i in range(cfg.layers):
        p = f"blk.{i}."
        for name in ("ffn_gate", "ffn_up", "ffn_down"):
            t[p + name + ".scale"] = np.abs(t[p + name + ".weight"]).mean(-1, dtype=np.float32)
            t[p + name + ".midpoint"] = np.zeros(t[p + name + ".weight"].shape[0], np.float32)
        t[p + "ffn_gate_up.gain"] = np.ones(cfg.hidden, np.float32)
        t[p + "ffn_gate_up.bound"] = np.float32(1.0)
        t[p + "ffn_down.gain"] = np.ones(cfg.intermediate, np.float32)
        t[p + "ffn_down.bound"] = np.float32(1.0)
    vocab = vocabulary.numpy()
    feats = features.float().numpy()
    tok = tuple(int(v) for v in tokens)
    anchor = CONTEXT
    # context K/V of positions [0, anchor - INGEST): set-up, not timed
    enc = od.encode_context(t, feats, anchor - INGEST, cfg)
    contexts = [od.layer_context(t, i, enc, np.arange(anchor - INGEST), cfg) for i in range(cfg.layers)]
    times = []
    for _ in range(max(1, steps)):
        start = time.perf_counter()
        # ingest INGEST rows: fusion + per-layer context K/V of the new rows
        new = od.encode_context(t, feats[anchor - INGEST:anchor], INGEST, cfg)
        full = []
        for i in range(cfg.layers):
            k, v = od.layer_context(t, i, new, np.arange(anchor - INGEST, anchor), cfg)
            full.append((np.concatenate((contexts[i][0], k)), np.concatenate((contexts[i][1], v))))
        logits = od.he4_forward(t, vocab, VOCAB - 1, feats, tok, anchor, cfg, contexts=full)
        np.argmax(logits[1:], -1)
        times.append(time.perf_counter() - start)
        if sum(times) > budget_s:
            break
    per_step = statistics.median(times)
    return (SLOTS - 1) / per_step, per_step, len(times)


def reference_arm(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    torch.set_num_threads(os.cpu_count() or 1)
    tensors, vocabulary, features, tokens = make_tensors()
    steps = max(1, min(args.steps, 3))
    cpu_round_rate(tensors, vocabulary, features, tokens, 1, budget_s=10.0)  # warm-up (one step)
    rate, per_step, n = cpu_round_rate(tensors, vocabulary, features, tokens, steps)
    cores = os.cpu_count() or 1
    line = {
        "impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT, "n_gpus": world, "steps": n,
        "warmup": 1, "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (random-init weights, N(0,1) features)",
        "config": workload_config(),
        "cpu_baseline": {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{n} draft round(s) of the workload on the numpy restatement of HE4.forward "
                                   "(oracle/drafter.py) with the same cached-context semantics"},
        "e2e": {"value": rate, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU arm


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.rows: list[tuple[float, list[str]]] = []
        self.window = (0.0, 0.0)

    def start(self):
        """Begin sampling (before the warm-up, so short timed regions still see samples)."""
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True, bufsize=1)
        except OSError:
            self.proc = None
        if self.proc is not None:
            import threading

            def reader():
                for line in self.proc.stdout:
                    if line.strip():
                        self.rows.append((time.time(), [v.strip() for v in line.split(",")]))

            self.thread = threading.Thread(target=reader, daemon=True)
            self.thread.start()
        return self

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=5)

    def summary(self) -> dict:
        """Samples taken during the timed window; if it was shorter than the sampling
        interval, the samples of the warm-up right before it (same workload)."""
        t0, t1 = self.window
        inside = [f for t, f in self.rows if t0 <= t <= t1]
        scope = "timed"
        if not inside:
            inside = [f for t, f in self.rows if t <= t1][-5:]
            scope = "warm-up and timed (timed region shorter than the 50 ms sampling interval)"
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for f in inside:
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for name, flag in zip(names, f[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm), "scope": scope}


def gpu_arm(args, rank: int, world: int, local_rank: int) -> None:
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    pkg = importlib.import_module("binary-eagle-decoding_b200")
    from importlib import import_module

    drafter = import_module("binary-eagle-decoding_b200.drafter")
    lib = pkg._lib
    lib.load()
    dist = None
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    tensors, vocabulary, features, tokens = make_tensors(seed=rank)
    geom = importlib.import_module("binary-eagle-decoding_b200.model").Geometry(**GEOMETRY)
    engine = drafter.DraftEngine(tensors, vocabulary, VOCAB - 1, geom, device=device)
    feats_dev = features.to(device)
    engine.prefill(feats_dev, CONTEXT - INGEST)
    rnd = drafter.DraftRound(engine, CONTEXT, SLOTS, INGEST)
    rnd.host_rows.copy_(features[CONTEXT - INGEST:CONTEXT])
    rnd.host_first[0] = int(tokens[CONTEXT])
    rnd()  # the real rows and anchor token in place
    engine.check()

    stream = rnd.stream
    clocks = ClockSampler(local_rank).start()
    for _ in range(args.warmup):
        rnd.replay()
    stream.synchronize()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    before = lib.launches
    wall0 = time.time()
    with torch.cuda.stream(stream):
        start.record(stream)
        for _ in range(args.steps):
            rnd.replay()
        end.record(stream)
    end.synchronize()
    clocks.window = (wall0, time.time())
    clocks.stop()
    ms = start.elapsed_time(end)
    torch.cuda.synchronize()
    if dist:
        t = torch.tensor([ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    ms_per_step = ms / args.steps
    value = world * (SLOTS - 1) * args.steps / (ms / 1e3)

    # launches of this library's kernels in one captured round
    lib.launches = 0
    engine.ingest(feats_dev[CONTEXT - INGEST:CONTEXT], CONTEXT - INGEST)
    engine.draft(CONTEXT, SLOTS)
    per_round = lib.launches
    lib.launches = before
    torch.cuda.synchronize()
    engine.check()

    # end to end through the serving entry point: pinned H2D, round, D2H
    e2e_times = []
    for _ in range(max(3, args.steps)):
        t0 = time.perf_counter()
        rnd()
        e2e_times.append(time.perf_counter() - t0)
    e2e_ms = statistics.median(e2e_times) * 1e3
    if dist:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * (SLOTS - 1) / (e2e_ms / 1e3)

    # roofline of the dominant kernel: the tied LM head (vocab x hidden bf16 GEMV + argmax)
    H = GEOMETRY["hidden"]
    engine._pack(engine.state, SLOTS, H, H, engine.out_norm)
    reps = 50
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        for _ in range(5):
            engine._gemv(engine.head.data_ptr(), VOCAB, H, SLOTS, None, VOCAB, keys=engine.keys)
        s2.record(stream)
        for _ in range(reps):
            engine._gemv(engine.head.data_ptr(), VOCAB, H, SLOTS, None, VOCAB, keys=engine.keys)
        e2.record(stream)
    e2.synchronize()
    engine.keys.zero_()
    head_us = s2.elapsed_time(e2) * 1e3 / reps
    head_bytes = VOCAB * H * 2 + int(lib.load().bd_x16_bytes(SLOTS, H))
    peak, peak_kind = peaks()
    achieved = head_bytes / (head_us * 1e-6) / 1e9

    if dist:
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (random-init N(0,0.02) bf16 weights, N(0,1) bf16 features)",
        "config": workload_config(),
        "roofline": {"bound": "hbm", "kernel": "gemv_kernel (tied LM head, 151936x2560 bf16, 16 tokens, fused argmax)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} HBM copy bandwidth", "traffic": None,
                     "algorithmic_bytes_per_launch": head_bytes, "launch_us": head_us},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": rnd.h2d_bytes,
                "d2h_bytes_per_step": rnd.d2h_bytes, "ms_per_step": e2e_ms},
        "gpu_launches": per_round * args.steps,
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu:
        torch.set_num_threads(os.cpu_count() or 1)
        rate, per_step, n = cpu_round_rate(tensors, vocabulary, features, tokens, 2, budget_s=25.0)
        line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": os.cpu_count() or 1, "kind": "port",
                                "sample": f"{n} draft round(s) of the workload on the numpy restatement "
                                          "(oracle/drafter.py), cached context"}
    print(json.dumps(line), flush=True)


def profile_round() -> None:
    """One draft round between cudaProfilerStart/Stop (for ncu --profile-from-start off)."""
    device = torch.device("cuda", 0)
    drafter = importlib.import_module("binary-eagle-decoding_b200.drafter")
    geom = importlib.import_module("binary-eagle-decoding_b200.model").Geometry(**GEOMETRY)
    tensors, vocabulary, features, tokens = make_tensors()
    engine = drafter.DraftEngine(tensors, vocabulary, VOCAB - 1, geom, device=device)
    feats = features.to(device)
    engine.prefill(feats, CONTEXT - INGEST)
    for _ in range(3):  # the round of the last warm-up is the profiled one
        engine.ingest(feats[CONTEXT - INGEST:CONTEXT], CONTEXT - INGEST)
        engine.set_tokens(int(tokens[CONTEXT]), SLOTS)
        engine.draft(CONTEXT, SLOTS)
        torch.cuda.synchronize()
        if _ == 1:
            torch.cuda.cudart().cudaProfilerStart()
    torch.cuda.cudart().cudaProfilerStop()
    engine.check()
    print("profiled one draft round")


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=2000)
    parser.add_argument("--warmup", type=int, default=50)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    parser.add_argument("--profile-round", action="store_true",
                        help="run one draft round between cudaProfilerStart/Stop and exit")
    args = parser.parse_args()
    if args.profile_round:
        profile_round()
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus if args.gpus == 1 else 1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args, rank, world)
    else:
        gpu_arm(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
