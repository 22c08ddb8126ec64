"""Generate the golden fixtures in this folder from the reference implementation.

Run in a checkout that has the reference (philippesic/binary-eagle-decoding)
available read-only; it imports ``w1a1_eagle`` and ``benchmarks`` from there
and writes small ``.npz``/``.json`` fixtures next to this script:

    python tests/golden/make_golden.py /path/to/reference

The fixtures pin the CPU oracle (``oracle/``) to the reference's own outputs
on seeded inputs; the GPU parity tests then compare the CUDA path with the
oracle.  Nothing on the GPU side reads the reference.
"""

from __future__ import annotations

import json
import math
import sys
from pathlib import Path

import numpy as np
import torch
from torch import nn

HERE = Path(__file__).resolve().parent
if len(sys.argv) != 2:
    raise SystemExit("usage: python tests/golden/make_golden.py /path/to/reference-checkout")
REFERENCE = Path(sys.argv[1])
sys.path.insert(0, str(REFERENCE))

from benchmarks.acceptance import reduce_rounds  # noqa: E402
from benchmarks.verifier import reduce_verifier_trace  # noqa: E402
from w1a1_eagle.contracts import argmax as reference_argmax  # noqa: E402
from w1a1_eagle.model import HE4, Geometry, Layer, Projection, bound_latents, hard_sign  # noqa: E402
from w1a1_eagle.numerical.export import packed_signs  # noqa: E402

torch.set_num_threads(1)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().float().numpy().astype(np.float32)


def signs_fixture() -> None:
    one = torch.tensor(1.0)
    edges = torch.tensor([-2.0, -1.0, -0.5, -0.0, 0.0, 0.5, 1.0, 2.0])
    edges = torch.cat((
        edges,
        torch.nextafter(one, torch.tensor(2.0)).reshape(1),
        torch.nextafter(one, torch.tensor(0.0)).reshape(1),
        -torch.nextafter(one, torch.tensor(2.0)).reshape(1),
        -torch.nextafter(one, torch.tensor(0.0)).reshape(1),
        torch.randn(4096, generator=torch.Generator().manual_seed(3)) * 1.5,
    ))
    upstream = torch.randn(edges.shape, generator=torch.Generator().manual_seed(4))
    source = edges.clone().requires_grad_()
    out = hard_sign(source)
    (out * upstream).sum().backward()
    np.savez(HERE / "signs.npz", value=f32(edges), upstream=f32(upstream), sign=f32(out), grad=f32(source.grad))


def packing_fixture() -> None:
    arrays = {}
    kat = torch.full((1, 33), -1.0)
    kat[0, 0] = -0.0
    kat[0, 31] = 1
    kat[0, 32] = 1
    arrays["kat_value"] = f32(kat)
    arrays["kat_words"] = packed_signs(kat)
    for columns in (1, 7, 8, 31, 32, 33, 65, 300):
        values = torch.randn(3 if columns < 300 else 37, columns, generator=torch.Generator().manual_seed(columns))
        values[0, 0] = -0.0
        arrays[f"value_{columns}"] = f32(values)
        arrays[f"words_{columns}"] = packed_signs(values)
    np.savez(HERE / "packing.npz", **arrays)


def projection_cases():
    cases = []
    for index, (bits, tokens, inner, outer) in enumerate(
        [(4, 3, 37, 11), (8, 5, 70, 9), (4, 16, 64, 48), (8, 2, 33, 40), (4, 1, 256, 16)]
    ):
        g = torch.Generator().manual_seed(100 + index)
        weight = torch.randn(outer, inner, generator=g) * 0.6
        weight[0, :3] = torch.tensor([-0.0, 1.0, -1.0])
        gain = nn.Parameter(torch.randn(inner, generator=g) * 0.3)
        clip = nn.Parameter(torch.tensor(float(torch.randn((), generator=g) * 0.5)))
        layer = Projection(weight, bits, gain, clip)
        with torch.no_grad():
            layer.midpoint.copy_(torch.randn(outer, generator=g) * 0.05)
            layer.scale.mul_(1 + 0.1 * torch.randn(outer, generator=g))
            layer.scale[0] = -0.01
        value = (torch.randn(tokens, inner, generator=g) * 1.3).requires_grad_()
        upstream = torch.randn(tokens, outer, generator=g)
        out = layer.forward(value)
        (out * upstream).sum().backward()
        case = {
            "bits": np.int64(bits),
            "value": f32(value),
            "latent": f32(layer.latent_sign),
            "scale": f32(layer.scale),
            "midpoint": f32(layer.midpoint),
            "log_gain": f32(layer.log_gain),
            "log_clip": f32(layer.log_clip),
            "gain": f32(layer.log_gain.exp()),
            "bound": f32(layer.log_clip.exp()),
            "upstream": f32(upstream),
            "output": f32(out),
            "grad_input": f32(value.grad),
        }
        for name, parameter in layer.named_parameters():
            case["grad_" + name] = f32(parameter.grad)
        cases.append(case)
    return cases


def projection_fixture() -> None:
    arrays = {}
    for index, case in enumerate(projection_cases()):
        for key, value in case.items():
            arrays[f"{index}_{key}"] = value
    arrays["count"] = np.int64(index + 1)
    np.savez(HERE / "projection.npz", **arrays)


def he4_ffn_fixture() -> None:
    g = torch.Generator().manual_seed(7)
    hidden, inner, tokens = 64, 96, 5
    cfg = Geometry(hidden=hidden, intermediate=inner, heads=2, kv_heads=1, head_dim=2)
    tensors = {
        "blk.0.attn_norm.weight": torch.ones(hidden),
        "blk.0.attn_q_norm.weight": torch.ones(2),
        "blk.0.attn_k_norm.weight": torch.ones(2),
        "blk.0.ffn_norm.weight": 1 + 0.1 * torch.randn(hidden, generator=g),
        "blk.0.attn_q.weight": torch.zeros(4, hidden),
        "blk.0.attn_k.weight": torch.zeros(2, hidden),
        "blk.0.attn_v.weight": torch.zeros(2, hidden),
        "blk.0.attn_output.weight": torch.zeros(hidden, 4),
        "blk.0.ffn_gate.weight": torch.randn(inner, hidden, generator=g) * 0.02,
        "blk.0.ffn_up.weight": torch.randn(inner, hidden, generator=g) * 0.02,
        "blk.0.ffn_down.weight": torch.randn(hidden, inner, generator=g) * 0.02,
    }
    layer = Layer(tensors, "blk.0.", cfg)
    with torch.no_grad():
        layer.gate.log_gain.copy_(0.2 * torch.randn(hidden, generator=g))
        layer.gate.log_clip.fill_(0.4)
        layer.down.log_gain.copy_(0.2 * torch.randn(inner, generator=g))
        layer.down.log_clip.fill_(-0.3)
        for p in (layer.gate, layer.up, layer.down):
            p.midpoint.copy_(0.01 * torch.randn(p.midpoint.shape, generator=g))
    residual = torch.randn(tokens, hidden, generator=g)
    from w1a1_eagle.model import rms

    with torch.no_grad():
        norm = rms(residual, layer.ffn_norm, cfg.epsilon)
        gate = layer.gate.forward(norm)
        up = layer.up.forward(norm)
        h = torch.nn.functional.silu(gate) * up
        down = layer.down.forward(h)
        out = residual + down
    arrays = {"residual": f32(residual), "norm": f32(norm), "gate_out": f32(gate), "up_out": f32(up),
              "hidden": f32(h), "down_out": f32(down), "output": f32(out), "epsilon": np.float32(cfg.epsilon)}
    arrays["ffn_norm"] = f32(layer.ffn_norm)
    for name, p in (("gate", layer.gate), ("up", layer.up), ("down", layer.down)):
        arrays[name + "_latent"] = f32(p.latent_sign)
        arrays[name + "_scale"] = f32(p.scale)
        arrays[name + "_midpoint"] = f32(p.midpoint)
        arrays[name + "_gain"] = f32(p.log_gain.exp())
        arrays[name + "_bound"] = f32(p.log_clip.exp())
    np.savez(HERE / "he4_ffn.npz", **arrays)


def w1_fixture() -> None:
    """Pure-W1 SwiGLU from the reference's parts (hard_sign, linear, mean|W| scale)."""
    g = torch.Generator().manual_seed(11)
    tokens, hidden, inner = 4, 80, 96
    x = torch.randn(tokens, hidden, generator=g)
    wg = torch.randn(inner, hidden, generator=g) * 0.02
    wu = torch.randn(inner, hidden, generator=g) * 0.02
    wd = torch.randn(hidden, inner, generator=g) * 0.02

    def project(v, w):
        return torch.nn.functional.linear(v, hard_sign(w)) * w.abs().mean(-1)

    with torch.no_grad():
        y = project(torch.nn.functional.silu(project(x, wg)) * project(x, wu), wd)
    np.savez(HERE / "w1_ffn.npz", x=f32(x), w_gate=f32(wg), w_up=f32(wu), w_down=f32(wd), y=f32(y))


def w1a1_fixture() -> None:
    """W1A1 SwiGLU from the reference's parts: ``hard_sign`` for weights and
    activations (x >= 0 -> +1, -0.0 -> +1), ``packed_signs`` for the bit words,
    torch ``linear`` of the +-1 operands for the dots, the ``Projection.scale``
    initialiser ``mean|W|`` per row and a per-token ``mean|x|`` scale; the
    intermediate ``silu(gate) * up`` is re-binarised before the down projection."""
    g = torch.Generator().manual_seed(12)
    tokens, hidden, inner = 5, 96, 160
    x = torch.randn(tokens, hidden, generator=g)
    x[0, 0] = -0.0
    x[1, 5] = 0.0
    wg = torch.randn(inner, hidden, generator=g) * 0.02
    wu = torch.randn(inner, hidden, generator=g) * 0.02
    wd = torch.randn(hidden, inner, generator=g) * 0.02
    wg[0, 0] = -0.0
    arrays = {"x": f32(x), "w_gate": f32(wg), "w_up": f32(wu), "w_down": f32(wd)}

    def project(v, w, tag):
        with torch.no_grad():
            signs_v, signs_w = hard_sign(v), hard_sign(w)
            dot = torch.nn.functional.linear(signs_v, signs_w)
            mean = v.abs().mean(-1)
            out = (dot * w.abs().mean(-1)) * mean[:, None]
        arrays[tag + "_words_in"] = packed_signs(v)
        arrays[tag + "_words_w"] = packed_signs(w)
        arrays[tag + "_dot"] = dot.numpy().astype(np.int64)
        arrays[tag + "_mean"] = f32(mean)
        arrays[tag + "_out"] = f32(out)
        return out

    gate = project(x, wg, "gate")
    up = project(x, wu, "up")
    with torch.no_grad():
        h = torch.nn.functional.silu(gate) * up
    arrays["hidden"] = f32(h)
    arrays["y"] = f32(project(h, wd, "down"))
    np.savez(HERE / "w1a1_ffn.npz", **arrays)


def tiny_he4_fixture() -> None:
    """The reference's tiny six-layer HE4 (``tests/numerical/test_model.py:56-86``), perturbed quantizers."""
    arrays = {}
    for window in (4096, 5):
        cfg = Geometry(hidden=4, intermediate=8, heads=2, kv_heads=1, head_dim=2, window=window)
        generator = torch.Generator().manual_seed(17)
        tensors = {
            "fc.weight": torch.randn((4, 32), generator=generator) * 0.1,
            "enc.output_norm.weight": torch.ones(4),
            "output_norm.weight": torch.ones(4),
        }
        shapes = {
            "attn_norm": (4,), "attn_q_norm": (2,), "attn_k_norm": (2,), "ffn_norm": (4,),
            "attn_q": (4, 4), "attn_k": (2, 4), "attn_v": (2, 4), "attn_output": (4, 4),
            "ffn_gate": (8, 4), "ffn_up": (8, 4), "ffn_down": (4, 8),
        }
        for index in range(6):
            for name, shape in shapes.items():
                tensors[f"blk.{index}.{name}.weight"] = (
                    torch.ones(shape) if len(shape) == 1 else torch.randn(shape, generator=generator) * 0.1
                )
        vocabulary = torch.randn((20, 4), generator=generator)
        model = HE4(tensors, vocabulary, 19, cfg)
        features = torch.randn((20, 32), generator=generator)
        perturb = torch.Generator().manual_seed(23)
        with torch.no_grad():
            for block in model.blocks:
                block.gate.log_gain.copy_(0.3 * torch.randn(4, generator=perturb))
                block.gate.log_clip.fill_(float(0.3 * torch.randn((), generator=perturb)))
                block.down.log_gain.copy_(0.3 * torch.randn(8, generator=perturb))
                block.down.log_clip.fill_(float(0.3 * torch.randn((), generator=perturb)))
                for p in (block.gate, block.up, block.down):
                    p.midpoint.copy_(0.05 * torch.randn(p.midpoint.shape, generator=perturb))
        tag = f"w{window}"
        if window == 4096:
            for name, value in tensors.items():
                arrays["t_" + name] = f32(value)
            arrays["vocabulary"] = f32(vocabulary)
            arrays["features"] = f32(features)
        for index, block in enumerate(model.blocks):
            for name, p in (("ffn_gate", block.gate), ("ffn_up", block.up), ("ffn_down", block.down)):
                arrays[f"{tag}_q_blk.{index}.{name}.scale"] = f32(p.scale)
                arrays[f"{tag}_q_blk.{index}.{name}.midpoint"] = f32(p.midpoint)
            arrays[f"{tag}_q_blk.{index}.ffn_gate_up.gain"] = f32(block.gate.log_gain.exp())
            arrays[f"{tag}_q_blk.{index}.ffn_gate_up.bound"] = f32(block.gate.log_clip.exp())
            arrays[f"{tag}_q_blk.{index}.ffn_down.gain"] = f32(block.down.log_gain.exp())
            arrays[f"{tag}_q_blk.{index}.ffn_down.bound"] = f32(block.down.log_clip.exp())
        with torch.no_grad():
            for anchor in (2, 7, 19):
                arrays[f"{tag}_logits_{anchor}"] = f32(model.forward(features, tuple(range(20)), anchor))
            arrays[f"{tag}_logits_7_s3"] = f32(model.forward(features, tuple(range(20)), 7, 3))
    np.savez(HERE / "tiny_he4.npz", **arrays)


def export_fixture() -> None:
    """The FFN payloads ``prepare`` (``w1a1_eagle/numerical/export.py:174-193``) exports for the
    tiny six-layer HE4 with perturbed quantizers: packed signs, clamped scales, midpoints,
    gains, and the per-projection bits / clip metadata."""
    cfg = Geometry(hidden=4, intermediate=8, heads=2, kv_heads=1, head_dim=2, window=4096)
    f = np.load(HERE / "tiny_he4.npz")
    tensors = {k[2:]: torch.from_numpy(f[k]) for k in f.files if k.startswith("t_")}
    model = HE4(tensors, torch.from_numpy(f["vocabulary"]), 19, cfg)
    perturb = torch.Generator().manual_seed(29)
    arrays = {}
    with torch.no_grad():
        for block in model.blocks:
            block.gate.log_gain.copy_(0.3 * torch.randn(4, generator=perturb))
            block.gate.log_clip.fill_(float(0.3 * torch.randn((), generator=perturb)))
            block.down.log_gain.copy_(0.3 * torch.randn(8, generator=perturb))
            block.down.log_clip.fill_(float(0.3 * torch.randn((), generator=perturb)))
            for q in (block.gate, block.up, block.down):
                q.midpoint.copy_(0.05 * torch.randn(q.midpoint.shape, generator=perturb))
                q.scale.copy_(q.scale - 0.07)  # some scales below zero: the export clamps them
                q.latent_sign.copy_(q.latent_sign + 0.05 * torch.randn(q.latent_sign.shape, generator=perturb))
    for index, block in enumerate(model.blocks):
        for name, q in (("gate", block.gate), ("up", block.up), ("down", block.down)):
            base = f"blk.{index}.ffn_{name}"
            arrays[base + ".latent"] = f32(q.latent_sign)
            arrays[base + ".scale_param"] = f32(q.scale)
            arrays[base + ".midpoint_param"] = f32(q.midpoint)
            arrays[base + ".log_gain_param"] = f32(q.log_gain)
            arrays[base + ".log_clip_param"] = f32(q.log_clip)
            arrays[base + ".w1a1_packed"] = packed_signs(q.latent_sign)
            arrays[base + ".w1a1_scale"] = f32(q.scale.clamp_min(0))
            arrays[base + ".w1ax_midpoint"] = f32(q.midpoint)
            if name != "up":
                arrays[base + ".w1ax_gain"] = f32(q.log_gain.detach().float().cpu().exp())
            arrays[base + ".w1ax.bits"] = np.array(q.bits, dtype=np.uint32)
            arrays[base + ".w1ax.clip"] = np.array(float(q.log_clip.detach().float().cpu().exp()), dtype=np.float32)
    np.savez(HERE / "export_ffn.npz", **arrays)


def layer_fixture() -> None:
    """Inputs of the reference's cache-layer golden case (``test_model.py:555-581``)."""
    arrays = {}
    shapes = {
        "attn_norm": (4,), "attn_q_norm": (2,), "attn_k_norm": (2,), "ffn_norm": (4,),
        "attn_q": (4, 4), "attn_k": (2, 4), "attn_v": (2, 4), "attn_output": (4, 4),
        "ffn_gate": (8, 4), "ffn_up": (8, 4), "ffn_down": (4, 8),
    }
    for name, shape in shapes.items():
        value = torch.ones(shape) if len(shape) == 1 else (
            torch.sin(torch.arange(int(np.prod(shape)), dtype=torch.float32) * 0.37).reshape(shape) * 0.1
        )
        arrays["t_blk.0." + name + ".weight"] = f32(value)
    arrays["encoded"] = f32(torch.cos(torch.arange(12, dtype=torch.float32) * 0.23).reshape(3, 4) * 0.1)
    arrays["state"] = f32(torch.sin(torch.arange(64, dtype=torch.float32) * 0.13).reshape(16, 4) * 0.1)
    golden = json.loads((REFERENCE / "results/he4-checkpoint-migration/cache-layer-reference.json").read_text())
    arrays["output"] = np.asarray(golden["layer"]["output"], dtype=np.float32)
    np.savez(HERE / "layer.npz", **arrays)


def arithmetic_fixture() -> None:
    """The reference's retained projection arithmetic (``evidence/arithmetic-reference.json``)."""
    captured = json.loads((REFERENCE / "evidence/arithmetic-reference.json").read_text())
    projection = captured["projection"]
    out = {
        "weights": [[0.2, -0.4, -1.0], [1.0, 1.4, -0.0]],
        "inputs": [[0.1, 0.7, -0.2], [-0.3, 0.5, 1.2]],
        "gain": [0.1, -0.2, 0.3],
        "clip": 0.7,
        "midpoint": [0.05, -0.03],
        "output": projection["output"],
        "input_grad": projection["input_grad"],
        "gradients": projection["gradients"],
        "updated": projection["updated"],
    }
    (HERE / "arithmetic.json").write_text(json.dumps(out, indent=1))


def greedy_fixture() -> None:
    """Random greedy rounds whose emitted tokens the reference oracle accepts."""
    rng = np.random.default_rng(5)
    cases = []
    for index in range(200):
        n = int(rng.integers(1, 17))
        vocab = int(rng.integers(3, 40))
        targets = rng.integers(0, vocab, size=n + 1)
        drafts = targets[:n].copy()
        cut = int(rng.integers(0, n + 1))
        if cut < n:
            drafts[cut] = (targets[cut] + 1 + int(rng.integers(0, vocab - 1))) % vocab
        eog = [int(v) for v in rng.choice(vocab, size=2, replace=False)] if index % 3 == 0 else [vocab + 5]
        emitted = []
        for i, token in enumerate(drafts.tolist()):
            emitted.append(int(targets[i]))
            if targets[i] != token or (targets[i] in eog and i + 1 < n):
                break
        else:
            emitted.append(int(targets[-1]))
        raw = {"proposed": drafts.tolist(), "target_argmax": targets.tolist(), "accepted_tokens": emitted,
               "eog_ids": eog, "replay": False, "committed": True, "rejection": False}
        reduce_verifier_trace(["BINARY_VERIFIER_TRACE " + json.dumps(raw)])
        accepted = len(emitted) - 1
        reduce_rounds([{"proposed": drafts.tolist(), "accepted": accepted, "target_tokens": [emitted[-1]],
                        "emitted": drafts.tolist()[:accepted] + [emitted[-1]]}])
        cases.append({"targets": targets.tolist(), "drafts": drafts.tolist(), "eog": eog,
                      "accepted": accepted, "next": emitted[-1]})
    ties = []
    for index in range(50):
        row = rng.integers(-3, 3, size=int(rng.integers(1, 30))).astype(float).tolist()
        ties.append({"row": row, "argmax": reference_argmax(row)})
    (HERE / "greedy.json").write_text(json.dumps({"rounds": cases, "ties": ties}))


def adamw_fixture() -> None:
    g = torch.Generator().manual_seed(31)
    param = nn.Parameter(torch.randn(7, 13, generator=g))
    optimizer = torch.optim.AdamW([param], lr=1e-3, weight_decay=0, foreach=False)
    arrays = {"param0": f32(param)}
    for step in range(3):
        grad = torch.randn(7, 13, generator=g) * (0.1 + step)
        param.grad = grad
        optimizer.step()
        arrays[f"grad{step}"] = f32(grad)
        arrays[f"param{step + 1}"] = f32(param)
        state = optimizer.state[param]
        arrays[f"exp_avg{step + 1}"] = f32(state["exp_avg"])
        arrays[f"exp_avg_sq{step + 1}"] = f32(state["exp_avg_sq"])
    np.savez(HERE / "adamw.npz", **arrays)


def bound_fixture() -> None:
    g = torch.Generator().manual_seed(41)
    value = torch.randn(9, 21, generator=g)
    value[2] = 0.0
    projection = Projection(value, 4, nn.Parameter(torch.zeros(21)), nn.Parameter(torch.tensor(0.0)))
    bound_latents(projection, 3.0)
    kat = Projection(torch.tensor([[0.0, -0.0, 2.0, -14.0], [0.0, 0.0, 0.0, 0.0]]), 4,
                     nn.Parameter(torch.zeros(4)), nn.Parameter(torch.tensor(0.0)))
    bound_latents(kat, 2.0)
    np.savez(HERE / "bound.npz", value=f32(value), bounded=f32(projection.latent_sign), kat=f32(kat.latent_sign))


def group_loss_fixture() -> None:
    """The reference's own ``TensorWorker.group_loss`` (``worker.py:315-363``) on the tiny HE4
    (window 4096, the quantizer perturbation of ``tiny_he4_fixture``): the weighted loss
    and every parameter gradient, for exponential label weights (one head chunk) and
    per-position ("reach") weights over 132 label rows (two 128-row head chunks)."""
    from types import SimpleNamespace

    from w1a1_eagle.numerical.worker import TensorWorker

    f = np.load(HERE / "tiny_he4.npz")
    cfg = Geometry(hidden=4, intermediate=8, heads=2, kv_heads=1, head_dim=2, window=4096)
    tensors = {k[2:]: torch.from_numpy(f[k]) for k in f.files if k.startswith("t_")}
    model = HE4(tensors, torch.from_numpy(f["vocabulary"]), 19, cfg)
    perturb = torch.Generator().manual_seed(23)  # the draw order of tiny_he4_fixture
    with torch.no_grad():
        for block in model.blocks:
            block.gate.log_gain.copy_(0.3 * torch.randn(4, generator=perturb))
            block.gate.log_clip.fill_(float(0.3 * torch.randn((), generator=perturb)))
            block.down.log_gain.copy_(0.3 * torch.randn(8, generator=perturb))
            block.down.log_clip.fill_(float(0.3 * torch.randn((), generator=perturb)))
            for p in (block.gate, block.up, block.down):
                p.midpoint.copy_(0.05 * torch.randn(p.midpoint.shape, generator=perturb))
    capture = SimpleNamespace(features=torch.from_numpy(f["features"]), tokens=tuple(range(20)))
    g = torch.Generator().manual_seed(47)
    reach_windows = []
    for index, anchor in enumerate(range(1, 20, 2)):
        count = 6 if index in (3, 7) else 15
        reach_windows.append((anchor, tuple(int(v) for v in torch.randint(0, 20, (count,), generator=g))))
    reach = tuple(float(v) for v in (0.95 ** torch.arange(15, dtype=torch.float64)))
    cases = {
        "exp": (((3, (4, 5, 6)), (10, (11, 12, 13, 14, 15))), 6, "uniform", None),
        "reach": (tuple(reach_windows), None, "reach", reach),
    }
    arrays = {}
    for tag, (windows, slots, kind, positions) in cases.items():
        worker = SimpleNamespace(model=model, blocks=SimpleNamespace(position_weights=kind),
                                 position_weights=positions)
        supervision = tuple(SimpleNamespace(anchor=a, labels=labels) for a, labels in windows)
        model.zero_grad(set_to_none=True)
        loss = TensorWorker.group_loss(worker, capture, supervision, slots)
        arrays[f"{tag}_loss"] = f32(loss)
        arrays[f"{tag}_anchors"] = np.array([a for a, _ in windows], np.int64)
        arrays[f"{tag}_labels"] = np.array([l for _, labels in windows for l in labels], np.int64)
        arrays[f"{tag}_lengths"] = np.array([len(labels) for _, labels in windows], np.int64)
        arrays[f"{tag}_slots"] = np.int64(slots if slots is not None else -1)
        if positions is not None:
            arrays[f"{tag}_positions"] = np.array(positions, np.float64)
        for name, parameter in model.named_parameters():
            if parameter.grad is not None:
                arrays[f"{tag}_grad_{name}"] = f32(parameter.grad)
    np.savez(HERE / "group_loss.npz", **arrays)


def main() -> None:
    signs_fixture()
    packing_fixture()
    projection_fixture()
    he4_ffn_fixture()
    w1_fixture()
    w1a1_fixture()
    tiny_he4_fixture()
    export_fixture()
    layer_fixture()
    arithmetic_fixture()
    greedy_fixture()
    adamw_fixture()
    bound_fixture()
    group_loss_fixture()
    meta = {"reference": "philippesic/binary-eagle-decoding", "torch": torch.__version__, "numpy": np.__version__,
            "generator": "tests/golden/make_golden.py", "math": {"pi": math.pi}}
    (HERE / "meta.json").write_text(json.dumps(meta, indent=1))


if __name__ == "__main__":
    main()
