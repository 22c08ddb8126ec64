#!/usr/bin/env python
"""Drafted tokens/s of the 4-layer block-16 HE4 drafter on B200.

One draft round on a resident 4096-position context: ingest 16 new context
rows (fusion + per-layer context K/V into the fp16 cache), then the 4-layer
block forward over 4096 + 16 keys, the tied LM head and the per-slot argmax ->
15 drafted tokens.  One timed step = 128 consecutive rounds (--rounds-per-step).  Geometry of the headline
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

METRIC = "drafted tokens/s (block-16 HE4 drafter, summed over GPUs)"
UNIT = "drafted tokens/s"
# DRAM bytes of one LM-head GEMV launch, from one ncu capture of that launch
# (read 778.10 MB + write 3.31 MB); a constant, not re-measured by this script
LM_HEAD_DRAM_BYTES = 781_410_000
# One step = this many consecutive draft rounds of the request (graph replays),
# so that the default 20 timed steps span about a second of device time and the
# clock sampler sees the timed region.
ROUNDS_PER_STEP = 128
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


def bf16_peak() -> tuple[float, str]:
    """Dense bf16 burst TFLOP/s (cuBLAS), for a GEMM timed alone."""
    try:
        return float(json.loads(PEAKS.read_text())["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


# --------------------------------------------------------------------------- CPU (oracle) arm


def cpu_round_rate(tensors, vocabulary, features, tokens, steps: int, budget_s: float = 30.0, warmup: int = 0):
    """The CPU restatement of the same draft round (cached context), drafted tokens/s.

    ``warmup`` untimed rounds run first, on the same set-up; then up to ``steps``
    timed rounds, stopping once ``budget_s`` seconds of rounds have been timed.
    Returns (rate, median seconds per round, timed rounds).
    """
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
    def round_once():
        # ingest INGEST rows: fusion + per-layer context K/V of the new rows
        new = od.encode_context(t, feats[anchor - INGEST:anchor], INGEST, cfg)
        full = []
        for i in range(cfg.layers):
            k, v = od.layer_context(t, i, new, np.arange(anchor - INGEST, anchor), cfg)
            full.append((np.concatenate((contexts[i][0], k)), np.concatenate((contexts[i][1], v))))
        logits = od.he4_forward(t, vocab, VOCAB - 1, feats, tok, anchor, cfg, contexts=full)
        return np.argmax(logits[1:], -1)

    for _ in range(warmup):
        round_once()
    times = []
    for _ in range(max(1, steps)):
        start = time.perf_counter()
        round_once()
        times.append(time.perf_counter() - start)
        if sum(times) > budget_s:
            break
    per_step = statistics.median(times)
    return (SLOTS - 1) / per_step, per_step, len(times)


def host_threads() -> int:
    """Use every host core for the CPU legs (torchrun sets OMP_NUM_THREADS=1 for
    its ranks): torch's intra-op pool and numpy's BLAS pool.  Returns the BLAS
    thread count actually in effect."""
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    try:
        from threadpoolctl import threadpool_info, threadpool_limits

        threadpool_limits(cores)
        counts = [int(p.get("num_threads", 1)) for p in threadpool_info() if p.get("user_api") == "blas"]
        return max(counts) if counts else 1
    except Exception:
        return 1


def reference_arm(args, rank: int, world: int) -> None:
    if rank != 0:
        return
    cores = host_threads()
    tensors, vocabulary, features, tokens = make_tensors()
    # a bounded sample: at most 3 timed rounds (~3 s each on 16 cores) after 3 untimed ones
    steps = max(1, min(args.steps, 3))
    warmup = 3
    rate, per_step, n = cpu_round_rate(tensors, vocabulary, features, tokens, steps, warmup=warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": rate, "unit": UNIT, "n_gpus": world, "steps": n,
        "warmup": warmup, "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (random-init weights, N(0,1) features)",
        "config": workload_config(),
        "cpu_baseline": {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
                         "sample": f"{n} draft round(s) of the workload on the numpy restatement of HE4.forward "
                                   "(oracle/drafter.py) with the same cached-context semantics; a step here is "
                                   "one round, the value is per round"},
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
    rounds = args.rounds_per_step
    clocks = ClockSampler(local_rank).start()
    for _ in range(args.warmup * rounds):
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
        for _ in range(args.steps * rounds):
            rnd.replay()
        end.record(stream)
    end.synchronize()
    clocks.window = (wall0, time.time())
    clocks.stop()
    ms = start.elapsed_time(end)
    torch.cuda.synchronize()
    rank_ms = [ms]
    if dist:
        t = torch.tensor([ms], device=device)
        gathered = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(gathered, t)
        rank_ms = [float(v.item()) for v in gathered]
        ms = max(rank_ms)
        dist.barrier()
    ms_per_step = ms / args.steps
    value = world * (SLOTS - 1) * rounds * args.steps / (ms / 1e3)

    # launches of this library's kernels in one captured round
    lib.launches = 0
    engine.ingest(feats_dev[CONTEXT - INGEST:CONTEXT], CONTEXT - INGEST)
    engine.draft(CONTEXT, SLOTS)
    per_round = lib.launches
    lib.launches = before
    torch.cuda.synchronize()
    engine.check()

    # end to end through the serving entry point, every round: pinned H2D of the
    # new rows, the round, D2H of the drafted tokens (the call returns them)
    for _ in range(3):
        rnd()
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps * rounds):
        rnd()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / args.steps
    if dist:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * (SLOTS - 1) * rounds / (e2e_ms / 1e3)

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
    config = workload_config()
    config["rounds_per_step"] = rounds
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (random-init N(0,0.02) bf16 weights, N(0,1) bf16 features)",
        "config": config,
        "per_gpu_value": value / world,
        "rank_ms_per_step": [v / args.steps for v in rank_ms],
        "roofline": {"bound": "hbm", "kernel": "gemv_kernel (tied LM head, 151936x2560 bf16, 16 tokens, fused argmax)",
                     "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "peak_source": f"{peak_kind} HBM copy bandwidth (burst; the head is timed alone)",
                     "traffic": LM_HEAD_DRAM_BYTES,
                     "traffic_source": "constant from one earlier ncu capture of this launch "
                                       "(dram__bytes_read.sum + dram__bytes_write.sum), not measured in this run",
                     "algorithmic_bytes_per_launch": head_bytes, "launch_us": head_us},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": rnd.h2d_bytes * rounds,
                "d2h_bytes_per_step": rnd.d2h_bytes * rounds, "ms_per_step": e2e_ms,
                "step": f"{rounds} calls of DraftRound.__call__, each: pinned host rows in, one round, drafted "
                        "tokens out (host wall clock, max over ranks)"},
        "gpu_launches": per_round * rounds * args.steps,
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_sub:
        pkg_ = importlib.import_module("binary-eagle-decoding_b200")
        line["ffn"] = ffn_record(pkg_, device, peak, peak_kind)
        line["accept"] = accept_record(pkg_, device, peak, peak_kind)
        line["w1a1"] = w1a1_record(pkg_, device)
    if world == 1 and not args.no_cpu:
        cores = host_threads()
        rate, per_step, n = cpu_round_rate(tensors, vocabulary, features, tokens, 2, budget_s=25.0)
        line["cpu_baseline"] = {"value": rate, "unit": UNIT, "cores": cores, "kind": "port",
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


# --------------------------------------------------------------------------- other workloads (one GPU)
# The headline is the draft round above; these lines measure the other hot-path
# workloads on their own shapes (single binary FFN block, W1A1 at M = 1024,
# block acceptance, the QAT update) for the kernel summaries.


def _events_us(fn, reps: int) -> float:
    st, en = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    st.record()
    for _ in range(reps):
        fn()
    en.record()
    torch.cuda.synchronize()
    return st.elapsed_time(en) * 1e3 / reps


def _graph_us(fn, calls: int, reps: int) -> float:
    """Capture `calls` invocations of fn(i) in one CUDA graph; time its replays."""
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for i in range(calls):
            fn(i)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    return _events_us(graph.replay, reps) / calls


def _ffn_sets(pkg, device, sets: int, seed: int = 0):
    """`sets` independent config-1 FFN weight sets (W8 sign words + HE4 defaults)."""
    ops = pkg.ops
    H, F = 2560, 9728
    g = torch.Generator(device=device).manual_seed(seed)
    ffns = []
    for _ in range(sets):
        gate, up, down = (torch.randn(s, generator=g, device=device) * 0.02 for s in ((F, H), (F, H), (H, F)))
        f = ops.pack_ffn(gate, up, down)
        del gate, up, down
        f.midpoint_gate, f.midpoint_up = torch.zeros(F, device=device), torch.zeros(F, device=device)
        f.midpoint_down = torch.zeros(H, device=device)
        f.gain_gate_up, f.gain_down = torch.ones(H, device=device), torch.ones(F, device=device)
        f.bound_gate_up, f.bound_down = torch.ones(1, device=device), torch.ones(1, device=device)
        ffns.append(f)
    return ffns


FFN_SETS = 48  # 48 x 9.34 MB of sign words = 448 MB: more than three times the 126 MB L2


def ffn_record(pkg, device, peak: float, peak_kind: str) -> dict:
    """Config 1 (one binary SwiGLU block, 16 tokens, 2560 -> 9728 -> 2560): pure-W1
    (fp32 activations) and HE4 (A4/A8 codes), each timed as a CUDA graph of one
    block per weight set over 48 sets (> 3 x L2), CUDA events on the replay stream."""
    ops = pkg.ops
    H, F, T = 2560, 9728, 16
    ffns = _ffn_sets(pkg, device, FFN_SETS)
    x = torch.randn((T, H), generator=torch.Generator(device=device).manual_seed(1), device=device)
    flags = ops.Flags(device)
    algorithmic = 3 * F * H // 8 + (2 * F + H) * 4 + 2 * T * H * 4
    out = {"workload": "config 1: one binary SwiGLU block, 16 tokens, 2560 -> 9728 -> 2560, fp32 in/out",
           "algorithmic_bytes": algorithmic,
           "timing": f"CUDA graph of {FFN_SETS} blocks over {FFN_SETS} weight sets (448 MB > 3 x L2), CUDA events"}
    for mode, fn in (("w1", lambda i: ops.ffn_w1(x, ffns[i % FFN_SETS], flags=flags)),
                     ("he4", lambda i: ops.ffn_he4(x, ffns[i % FFN_SETS], flags=flags)),
                     ("he4_clusters", lambda i: ops.ffn_he4(x, ffns[i % FFN_SETS], flags=flags, fused=True))):
        us = _graph_us(fn, FFN_SETS, 20)
        gbs = algorithmic / (us * 1e-6) / 1e9
        out[mode] = {"us_per_block": us, "GB/s": gbs, "frac": gbs / peak}
    out["peak"] = peak
    out["peak_source"] = f"{peak_kind} HBM copy bandwidth"
    flags.check()
    del ffns
    torch.cuda.empty_cache()
    return out


def accept_record(pkg, device, peak: float, peak_kind: str) -> dict:
    """Config 4: greedy and rejection block acceptance, 32 requests x 16 drafts,
    vocabulary 151936; bf16 logits of 165 MB / 321 MB (> L2) per call."""
    lines = workload_accept(argparse.Namespace(steps=1000), pkg, device)
    out = {"peak": peak, "peak_source": f"{peak_kind} HBM copy bandwidth"}
    for name, line in zip(("greedy", "rejection"), lines):
        out[name] = {"us_per_call": line["us_per_call"], "GB/s": line["value"], "frac": line["value"] / peak,
                     "algorithmic_bytes": line["algorithmic_bytes"]}
    torch.cuda.empty_cache()
    return out


def w1a1_record(pkg, device) -> dict:
    """Config 3: the W1A1 block at M = 1024 on tcgen05 kind::i8."""
    line = workload_w1a1(argparse.Namespace(steps=2000), pkg, device)[0]
    peak, peak_kind = bf16_peak()
    i8_peak = 2 * peak
    torch.cuda.empty_cache()
    return {"us_per_block": line["us_per_ffn"], "TOP/s": line["value"], "frac": line["value"] / i8_peak,
            "peak": i8_peak, "peak_source": f"twice the {peak_kind} dense bf16 burst (no int8 peak is measured; "
                                            "kind::i8 issues at twice the kind::f16 rate)"}


def workload_ffn(args, pkg, device) -> list[dict]:
    """Config 1: one binary SwiGLU block, 16 tokens, 2560 -> 9728 -> 2560 (HE4, pure-W1, W1A1)."""
    ops = pkg.ops
    H, F, T = 2560, 9728, 16
    sets = 16  # 16 x 9.34 MB of sign tiles rotate through the graph: more than L2
    g = torch.Generator(device=device).manual_seed(0)
    ffns = []
    for _ in range(sets):
        gate, up, down = (torch.randn(s, generator=g, device=device) * 0.02 for s in ((F, H), (F, H), (H, F)))
        f = ops.pack_ffn(gate, up, down)
        f.midpoint_gate, f.midpoint_up = torch.zeros(F, device=device), torch.zeros(F, device=device)
        f.midpoint_down = torch.zeros(H, device=device)
        f.gain_gate_up, f.gain_down = torch.ones(H, device=device), torch.ones(F, device=device)
        f.bound_gate_up, f.bound_down = torch.ones(1, device=device), torch.ones(1, device=device)
        ffns.append(f)
    x = torch.randn((T, H), generator=g, device=device)
    flags = ops.Flags(device)
    algorithmic = 3 * F * H // 8 + (2 * F + H) * 4 + 2 * T * H * 4
    lines = []
    for mode, fn in (("he4", lambda i: ops.ffn_he4(x, ffns[i % sets], flags=flags)),
                     ("he4_clusters", lambda i: ops.ffn_he4(x, ffns[i % sets], flags=flags, fused=True)),
                     ("w1", lambda i: ops.ffn_w1(x, ffns[i % sets], flags=flags)),
                     ("w1a1", lambda i: ops.ffn_w1a1(x, ffns[i % sets], flags=flags))):
        us = _graph_us(fn, sets, max(args.steps // 40, 20))
        lines.append({"workload": f"binary SwiGLU FFN block ({mode}), 16 tokens, 2560x9728x2560",
                      "metric": "packed-FFN HBM GB/s", "value": algorithmic / (us * 1e-6) / 1e9, "unit": "GB/s",
                      "us_per_ffn": us, "algorithmic_bytes": algorithmic, "timing": "CUDA graph of 16 blocks over "
                      "16 weight sets (150 MB > L2), CUDA events"})
    flags.check()
    return lines


def workload_w1a1(args, pkg, device, world: int = 1) -> list[dict]:
    """Config 3: W1A1 SwiGLU block at M = 1024 (64 requests x 16 draft tokens) per GPU;
    under torchrun every rank serves its own 64 requests (data parallel by
    request, no collective on the data path), time = max over ranks."""
    ops = pkg.ops
    H, F, M = 2560, 9728, 1024
    g = torch.Generator(device=device).manual_seed(4)
    gate, up, down = (torch.randn(s, generator=g, device=device) * 0.02 for s in ((F, H), (F, H), (H, F)))
    ffn = ops.pack_ffn(gate, up, down, large=True)
    x = torch.randn((M, H), generator=torch.Generator(device=device).manual_seed(40 + (device.index or 0)),
                    device=device)
    flags = ops.Flags(device)
    for _ in range(3):
        ops.ffn_w1a1(x, ffn, flags=flags)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    us = _events_us(lambda: ops.ffn_w1a1(x, ffn, flags=flags), max(args.steps // 200, 5))
    flags.check()
    if world > 1:
        t = torch.tensor([us], device=device)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        us = float(t.item())
    macs = 3 * M * F * H
    return [{"workload": f"W1A1 SwiGLU block, M = 1024 per GPU (64 requests x 16 tokens), 2560x9728x2560, "
                         f"{world} GPU(s)", "metric": "+-1 TOP/s (MAC = 2 ops), summed over GPUs",
             "value": world * 2 * macs / (us * 1e-6) / 1e12, "unit": "TOP/s", "us_per_ffn": us, "n_gpus": world,
             "requests_per_s": world * 64 / (us * 1e-6)}]


def workload_accept(args, pkg, device) -> list[dict]:
    """Config 4: block acceptance of 32 requests x 16 drafts over a 151936 vocabulary."""
    ops = pkg.ops
    B, n, V = 32, 16, 151936
    g = torch.Generator(device=device).manual_seed(5)
    target = (torch.randn((B, n + 1, V), generator=g, device=device) * 3).to(torch.bfloat16)
    draft = (torch.randn((B, n, V), generator=g, device=device) * 3).to(torch.bfloat16)
    drafts = torch.randint(0, V, (B, n), generator=g, device=device, dtype=torch.int32)
    flags = ops.Flags(device)
    reps = max(args.steps // 200, 5)
    # CUDA graphs of 8 calls each (the logits, 165 MB and 321 MB, exceed L2)
    greedy = _graph_us(lambda i: ops.accept_greedy(target, drafts, flags=flags), 8, reps)
    rej = _graph_us(lambda i: ops.accept_rejection(target, draft, drafts, seed=8 + i, flags=flags), 8, reps)
    flags.check()
    gb, rb = target.numel() * 2 + drafts.numel() * 4, (target.numel() + draft.numel()) * 2 + drafts.numel() * 4
    return [{"workload": "greedy block acceptance, logits bf16 [32, 17, 151936]", "metric": "HBM GB/s",
             "value": gb / (greedy * 1e-6) / 1e9, "unit": "GB/s", "us_per_call": greedy, "algorithmic_bytes": gb},
            {"workload": "rejection sampling, target [32, 17, 151936] + draft [32, 16, 151936] bf16",
             "metric": "HBM GB/s (single-pass bytes)", "value": rb / (rej * 1e-6) / 1e9, "unit": "GB/s",
             "us_per_call": rej, "algorithmic_bytes": rb}]


def workload_ingest(args, pkg, device) -> list[dict]:
    """Teacher-feature ingestion of config-5 captures: per sequence 4 taps x 2048 rows x 2560
    fp16, tap-major -> token-major fp16 features with the finiteness scan."""
    ops = pkg.ops
    taps, rows, hidden, seqs = 4, 2048, 2560, 8
    g = torch.Generator(device=device).manual_seed(9)
    caps = [torch.randn((taps, rows, hidden), generator=g, device=device).half() for _ in range(seqs)]
    flags = ops.Flags(device)
    us = _graph_us(lambda i: ops.ingest_taps(caps[i % seqs], torch.float16, flags=flags), seqs,
                   max(args.steps // 100, 10))
    nbytes = 2 * taps * rows * hidden * 2  # read + write
    host = caps[0].cpu().pin_memory()
    for _ in range(3):
        ops.ingest_taps(host, torch.float16, device=device, flags=flags)
    torch.cuda.synchronize()
    e2e = _events_us(lambda: ops.ingest_taps(host, torch.float16, device=device, flags=flags), 10)
    flags.check()
    return [{"workload": "teacher-feature ingestion, 4 taps x 2048 rows x 2560 fp16 per sequence",
             "metric": "HBM GB/s (read + write)", "value": nbytes / (us * 1e-6) / 1e9, "unit": "GB/s",
             "us_per_sequence": us, "e2e_us_per_sequence_from_pinned_host": e2e,
             "h2d_bytes_per_sequence": nbytes // 2}]


def workload_fusion(args, pkg, device) -> list[dict]:
    """Context fusion of a 4096-row prefill: features [4096, 4 x 2560] bf16 x fc [2560, 10240]^T
    on the tensor cores (tcgen05 kind::f16), with torch's cuBLAS GEMM timed beside it."""
    ops = pkg.ops
    m, n, k = 4096, 2560, 10240
    g = torch.Generator(device=device).manual_seed(10)
    a = torch.randn((m, k), generator=g, device=device).to(torch.bfloat16)
    b = (torch.randn((n, k), generator=g, device=device) * 0.02).to(torch.bfloat16)
    out = torch.empty((m, n), dtype=torch.float32, device=device)
    reps = max(args.steps // 100, 10)
    us = _graph_us(lambda i: ops.gemm_bf16(a, b, out), 4, reps)
    lib_us = _graph_us(lambda i: torch.mm(a, b.t(), out_dtype=torch.float32), 4, reps)
    flops = 2 * m * n * k
    achieved = flops / (us * 1e-6) / 1e12
    peak, peak_kind = bf16_peak()
    return [{"workload": "context fusion GEMM of a 4096-row prefill, 4096 x 2560 x 10240 bf16 -> fp32",
             "metric": "TFLOP/s", "value": achieved, "unit": "TFLOP/s", "us_per_gemm": us,
             "cublas_tflops_same_shape": flops / (lib_us * 1e-6) / 1e12,
             "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                          "frac": achieved / peak, "peak_source": f"{peak_kind} bf16 burst GEMM throughput"}}]


def workload_ste(args, pkg, device) -> list[dict]:
    """Config-5 latent update of the drafter's binary FFN projections (gate, up, down of
    each layer, 9728 x 2560 fp32 latents): the straight-through sign backward
    (``bd_ste_sign_backward``: two fp32 gradient halves, the clip-window mask, the
    HE4 step scale) and the fused AdamW + clamp + W8 re-pack (``bd_adamw_latent``)."""
    lib = pkg._lib
    ops = pkg.ops
    rows, cols, count = 9728, 2560, args.ste_projections
    n = rows * cols
    g = torch.Generator(device=device).manual_seed(11)
    mats = []
    for _ in range(count):
        latent = (torch.randn((rows, cols), generator=g, device=device) * 0.02).clamp_(-1, 1)
        mats.append({"latent": latent, "g1": torch.randn((rows, cols), generator=g, device=device) * 1e-3,
                     "g2": torch.randn((rows, cols), generator=g, device=device) * 1e-6,
                     "out": torch.empty((rows, cols), device=device), "m": torch.zeros((rows, cols), device=device),
                     "v": torch.zeros((rows, cols), device=device),
                     "w8": torch.zeros(ops.w8_words(rows, cols), dtype=torch.int32, device=device)})
    bound = torch.full((1,), 0.05, device=device)
    flags = ops.Flags(device)
    stream = torch.cuda.current_stream(device).cuda_stream

    def sign_backward():
        for t in mats:
            lib.call("bd_ste_sign_backward", t["g1"].data_ptr(), t["g2"].data_ptr(), t["latent"].data_ptr(), n, 1.0,
                     bound.data_ptr(), 8, t["out"].data_ptr(), None, stream)

    def adamw():
        for t in mats:
            lib.call("bd_adamw_latent", t["latent"].data_ptr(), t["out"].data_ptr(), t["m"].data_ptr(),
                     t["v"].data_ptr(), rows, cols, 1e-5, 0.9, 0.999, 1e-8, 1, None, 1, t["w8"].data_ptr(), 1, 0,
                     flags.ptr, stream)

    reps = max(args.steps // 200, 5)
    for _ in range(3):
        sign_backward()
        adamw()
    torch.cuda.synchronize()
    ste_us = _events_us(sign_backward, reps) / count
    adam_us = _events_us(adamw, reps) / count
    flags.check()
    ste_bytes = 16 * n  # read two gradient halves + latent, write the masked gradient
    adam_bytes = 28 * n + 4 * ops.w8_words(rows, cols)  # read p, g, m, v; write p, m, v and the sign words
    peak, peak_kind = peaks()
    lines = []
    for name, us, nbytes in (("straight-through sign backward", ste_us, ste_bytes),
                             ("latent AdamW + clamp + W8 sign re-pack", adam_us, adam_bytes)):
        gbs = nbytes / (us * 1e-6) / 1e9
        lines.append({"workload": f"{name}, {count} x 9728 x 2560 fp32 latents (arrays larger than L2)",
                      "metric": "HBM GB/s (algorithmic)", "value": gbs, "unit": "GB/s", "us_per_projection": us,
                      "bytes_per_projection": nbytes, "frac_of_hbm": gbs / peak, "peak": f"{peak:.1f} GB/s ({peak_kind})"})
    return lines


def workload_qat(args, pkg, device, rank: int, world: int) -> list[dict]:
    """Config 5: QAT update of the 4-layer drafter, per GPU 8 sequences x 2048 positions,
    32 windows of 16 slots each; data parallel (NCCL all-reduce) under torchrun."""
    qat = importlib.import_module("binary-eagle-decoding_b200.qat")
    cfg = pkg.Geometry(**GEOMETRY)
    tensors, vocabulary, _, _ = make_tensors()
    # the straight-through window is a learned clip |w| <= alpha, alpha = 0.05 at the start
    model = pkg.HE4(tensors, vocabulary, VOCAB - 1, cfg, window=0.05, learned_window=True).to(device)
    del tensors, vocabulary
    opt = qat.BitAdamW(model)
    g = torch.Generator().manual_seed(100 + rank)
    seqs, length, windows_per = args.qat_sequences, 2048, 32
    samples = []
    for _ in range(seqs):
        feats = torch.randn((length, 4 * cfg.hidden), generator=g).half().to(device)
        tokens = tuple(torch.randint(0, VOCAB, (length,), generator=g).tolist())
        anchors = [16 + (length - 32) * i // windows_per for i in range(windows_per)]
        samples.append((feats, tokens, tuple(qat.Window(a, tuple(tokens[a + 1:a + 16])) for a in anchors)))
    params = [p for ps in opt.groups.values() for _, p in ps]
    # the gradient all-reduce runs in buckets during the last sequence's backward pass
    exchange = qat.GradientExchange(params)

    model_mod = importlib.import_module("binary-eagle-decoding_b200.model")
    # the latent gradients of all sequences as one product per projection, each handed
    # to the exchange as soon as it is written
    latent_grads = pkg.LatentGradients(model, seqs * windows_per * 16, on_ready=exchange.ready)

    def step(u):
        opt.zero_grad()
        # the device error checks of all sequences read once, before the norm and the update
        with model_mod.deferred_checks(device):
            with latent_grads:
                for i, (feats, tokens, windows) in enumerate(samples):
                    exchange.armed = i == len(samples) - 1
                    qat.group_loss(model, feats, tokens, windows, scale=1.0 / seqs)
            exchange.finish()
        _, coef = qat.clip_grad_norm(params, 1.0)
        opt.step(coef)

    for u in range(2):
        step(u)
    torch.cuda.synchronize()
    reps = 3
    us = _events_us(lambda: step(0), reps)
    t = torch.tensor([us], device=device)
    allreduce_ms = None
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        # the same payload reduced on its own, for the breakdown
        flat = torch.cat([p.grad.reshape(-1) for p in params])
        for _ in range(2):
            torch.distributed.all_reduce(flat)
        torch.cuda.synchronize()
        ar = torch.tensor([_events_us(lambda: torch.distributed.all_reduce(flat), 3) / 1e3], device=device)
        torch.distributed.all_reduce(ar, op=torch.distributed.ReduceOp.MAX)
        allreduce_ms = ar.item()
        del flat
    rows = seqs * windows_per * 16 * world
    n_params = sum(p.numel() for p in params)
    return [{"workload": f"QAT update, {seqs} sequences x 2048 positions x 32 windows of 16 slots per GPU, "
                         f"4-layer drafter, learned straight-through window (alpha 0.05 at the start), {world} GPU(s)",
             "metric": "slot rows / s", "value": rows / (t.item() * 1e-6),
             "unit": "rows/s", "ms_per_step": t.item() / 1e3, "n_gpus": world,
             "gradient_bytes": 4 * n_params, "allreduce_buckets_per_step": exchange.buckets // (reps + 2),
             "allreduce_ms_standalone": allreduce_ms}]


def workload_qat_kernels(args, pkg, device) -> list[dict]:
    """The kernels of the QAT update at config-5 sizes: one binary projection (9728 x
    2560, 4096 slot rows: the forward kind::i8 GEMM with the HE4 epilogue, the input
    gradient and the latent gradient with the straight-through mask, both split bf16),
    the fused cross-entropy head (480 labelled rows x 151936 x 2560, bf16 vocabulary)
    and one layer's window attention (32 windows of 16 slots, 32 / 8 heads of 128,
    2048 context keys, each window seeing the context before its anchor) forward and
    backward."""
    from torch import nn

    qat = importlib.import_module("binary-eagle-decoding_b200.qat")
    T, K, O = 4096, 2560, 9728
    g = torch.Generator().manual_seed(12)
    layer = pkg.Projection(torch.randn((O, K), generator=g) * 0.02, 4, nn.Parameter(torch.zeros(K)),
                           nn.Parameter(torch.tensor(0.0)), window=0.05, learned_window=True).to(device)
    x = torch.randn((T, K), generator=g).to(device).requires_grad_()
    upstream = torch.randn((T, O), generator=g).to(device)

    def projection():
        layer.zero_grad()
        x.grad = None
        (layer(x) * upstream).sum().backward()

    for _ in range(3):
        projection()
    torch.cuda.synchronize()
    reps = max(args.steps // 4, 5)
    us = _events_us(projection, reps)
    flop = 2 * T * O * K * 5  # forward (one int8 product), input and latent gradients (two bf16 halves each)
    R, H, V = 480, 2560, VOCAB

    class Head(nn.Module):
        def __init__(self):
            super().__init__()
            self.register_buffer("vocabulary", (torch.randn((V, H), generator=g) * 0.02).to(torch.bfloat16)
                                 .float().to(device))

    head_owner = Head()
    head = torch.randn((R, H), generator=g).to(device)
    labels = torch.randint(0, V, (R,), generator=g).to(device)
    weights = torch.full((R,), 1.0 / R, device=device)
    for _ in range(3):
        qat.loss_head(head, head_owner, labels, weights)
    torch.cuda.synchronize()
    head_us = _events_us(lambda: qat.loss_head(head, head_owner, labels, weights), reps)
    head_flop = 2 * R * V * H * 2 * 3  # logits twice and the gradient product, two halves each
    peak, kind = bf16_peak()
    lines = []
    for name, t, f in (("binary projection 9728 x 2560, 4096 rows: forward + input and latent gradients", us, flop),
                       ("fused cross-entropy head, 480 rows x 151936 x 2560", head_us, head_flop)):
        tf = f / (t * 1e-6) / 1e12
        lines.append({"workload": name, "metric": "tensor TFLOP/s (bf16-equivalent products)", "value": tf,
                      "unit": "TFLOP/s", "us_per_call": t, "frac_of_bf16_peak": tf / peak,
                      "peak": f"{peak:.1f} TFLOP/s ({kind} bf16 burst)"})
    lines.append(train_attention_record(pkg, device, reps))
    return lines


def train_attention_record(pkg, device, reps: int) -> dict:
    """One layer's window attention of the QAT update on the training-attention kernels."""
    model = importlib.import_module("binary-eagle-decoding_b200.model")
    W, k, kvh, g, d, L = 32, 16, 8, 4, 128, 2048
    gen = torch.Generator().manual_seed(13)
    query = torch.randn((W, k, kvh, g, d), generator=gen).to(device).requires_grad_()
    ctx_k, ctx_v = (torch.randn((L, kvh, d), generator=gen).half().float().to(device).requires_grad_()
                    for _ in range(2))
    slot_k, slot_v = (torch.randn((W, k, kvh, d), generator=gen).half().float().to(device).requires_grad_()
                      for _ in range(2))
    anchors = torch.tensor([16 + (L - 32) * i // W for i in range(W)], device=device)
    allowed = torch.arange(L, device=device)[None, None, :] < anchors[:, None, None]
    upstream = torch.randn((W, k, kvh, g, d), generator=gen).to(device)
    inputs = (query, ctx_k, ctx_v, slot_k, slot_v)

    def forward():
        return model.train_attention(*inputs, allowed, None)

    def both():
        for t in inputs:
            t.grad = None
        (forward() * upstream).sum().backward()

    for _ in range(3):
        both()
    torch.cuda.synchronize()
    with torch.no_grad():
        fwd_us = _events_us(forward, reps)
    both_us = _events_us(both, reps)
    # query-key pairs the mask allows (context before each anchor, plus the 16 slots), x 32 heads
    pairs = int(((anchors + k) * k).sum()) * kvh * g
    flop = pairs * d * 2 * 2  # S = q k and O = p v, 2 flops per multiply-add
    return {"workload": "window attention of one layer, 32 windows x 16 slots, 32 / 8 heads of 128, 2048 context "
                        "keys: forward, forward + backward", "metric": "us per call", "value": both_us, "unit": "us",
            "forward_us": fwd_us, "forward_backward_us": both_us, "visible_pairs": pairs,
            "forward_TFLOP/s": flop / (fwd_us * 1e-6) / 1e12,
            "note": "fp32-precision products as fp16 hi + lo mma.sync pairs: 2 MMAs per product forward"}


def run_workload(args, rank: int, world: int, local_rank: int) -> None:
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    pkg = importlib.import_module("binary-eagle-decoding_b200")
    lib = pkg._lib
    lib.load()
    before = lib.launches
    if args.workload == "ffn":
        lines = workload_ffn(args, pkg, device)
    elif args.workload == "w1a1":
        lines = workload_w1a1(args, pkg, device, world)
    elif args.workload == "accept":
        lines = workload_accept(args, pkg, device)
    elif args.workload == "ingest":
        lines = workload_ingest(args, pkg, device)
    elif args.workload == "fusion":
        lines = workload_fusion(args, pkg, device)
    elif args.workload == "ste":
        lines = workload_ste(args, pkg, device)
    elif args.workload == "qat_kernels":
        lines = workload_qat_kernels(args, pkg, device)
    else:
        lines = workload_qat(args, pkg, device, rank, world)
    if world > 1:
        torch.distributed.destroy_process_group()
    if rank == 0:
        for line in lines:
            line["kernel_launches_issued"] = lib.launches - before
            print(json.dumps(line), flush=True)


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    parser.add_argument("--no-sub", action="store_true", help="skip the per-config sub-records (ffn, accept, w1a1)")
    parser.add_argument("--rounds-per-step", type=int, default=ROUNDS_PER_STEP,
                        help="consecutive draft rounds in one timed step")
    parser.add_argument("--profile-round", action="store_true",
                        help="run one draft round between cudaProfilerStart/Stop and exit")
    parser.add_argument("--workload", choices=("round", "ffn", "w1a1", "accept", "ingest", "fusion", "ste", "qat",
                                               "qat_kernels"), default="round",
                        help="round: the headline draft round; the others measure one hot-path workload each")
    parser.add_argument("--qat-sequences", type=int, default=8)
    parser.add_argument("--ste-projections", type=int, default=12)
    args = parser.parse_args()
    if args.profile_round:
        profile_round()
        return
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus if args.gpus == 1 else 1)))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload != "round":
        run_workload(args, rank, world, local_rank)
        return
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args, rank, world)
    else:
        gpu_arm(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
