"""The CPU oracle against the reference's golden vectors and known-answer tests (no GPU)."""

from __future__ import annotations

import json
import struct

import numpy as np
import pytest

from conftest import GOLDEN, group_loss_case
from oracle import acceptance, core, drafter, optim


def load(name):
    return np.load(GOLDEN / name)


# ------------------------------------------------------------------ signs / packing


def test_sign_kat_and_ste():
    # tests/numerical/test_model.py:451-457 of the reference
    src = np.array([-2.0, -1.0, -0.0, 0.0, 1.0, 2.0], dtype=np.float32)
    assert core.hard_sign(src).tolist() == [-1, -1, 1, 1, 1, 1]
    assert core.sign_backward(np.ones(6, np.float32), src).tolist() == [0, 1, 1, 1, 1, 0]
    with pytest.raises(ValueError, match="F32"):
        core.hard_sign(src.astype(np.float64))


def test_sign_matches_reference_values_and_gradients():
    f = load("signs.npz")
    assert np.array_equal(core.hard_sign(f["value"]), f["sign"])
    assert np.array_equal(core.sign_backward(f["upstream"], f["value"]), f["grad"])


def test_packing_kat_and_widths():
    f = load("packing.npz")
    words = core.packed_signs(f["kat_value"])
    assert words.tobytes() == struct.pack("<II", 0x80000001, 1)
    assert np.array_equal(words, f["kat_words"])
    for columns in (1, 7, 8, 31, 32, 33, 65, 300):
        assert np.array_equal(core.packed_signs(f[f"value_{columns}"]), f[f"words_{columns}"]), columns
    with pytest.raises(ValueError, match="finite"):
        core.packed_signs(np.array([[np.nan]], dtype=np.float32))
    with pytest.raises(ValueError, match="finite"):
        core.packed_signs(np.zeros(3, dtype=np.float32))


@pytest.mark.parametrize("shape", [(1, 1), (16, 256), (17, 257), (37, 300), (48, 700)])
def test_t16_roundtrip(shape):
    rng = np.random.default_rng(sum(shape))
    latent = rng.standard_normal(shape).astype(np.float32)
    latent[0, 0] = -0.0
    words = core.tile_signs_t16(latent)
    nrb, ncp = core.t16_shape(*shape)
    assert words.shape == (nrb * ncp * 128,)
    assert np.array_equal(core.untile_signs_t16(words, *shape), latent >= 0)


# ------------------------------------------------------------------ projections


def projection_cases():
    f = load("projection.npz")
    for i in range(int(f["count"])):
        yield {k.split("_", 1)[1]: f[k] for k in f.files if k.startswith(f"{i}_")}


def test_projection_forward_bit_exact_against_reference():
    for c in projection_cases():
        out = core.projection_forward(c["value"], c["latent"], c["scale"], c["midpoint"], c["gain"], c["bound"], int(c["bits"]))
        assert np.array_equal(out, c["output"]), int(c["bits"])


def test_projection_backward_against_reference():
    for c in projection_cases():
        grads = optim.projection_backward(c["upstream"], c["value"], c["latent"], c["scale"], c["midpoint"],
                                          c["log_gain"], c["log_clip"], int(c["bits"]))
        np.testing.assert_allclose(grads["input"], c["grad_input"], rtol=1e-5, atol=1e-6)
        for name in ("latent_sign", "scale", "midpoint", "log_gain", "log_clip"):
            np.testing.assert_allclose(grads[name], c["grad_" + name], rtol=1e-4, atol=1e-5, err_msg=name)


def test_projection_scalar_oracle():
    # tests/numerical/test_model.py:437-449 of the reference
    out = core.projection_forward(np.array([[0.1, 0.7]], np.float32), np.array([[0.2, -0.4]], np.float32),
                                  np.array([0.3], np.float32), np.zeros(1, np.float32), np.ones(2, np.float32),
                                  np.float32(1.0), 4)
    assert abs(float(out[0, 0]) - (1 - 5) * 0.3 / 7) < 1e-6
    grads = optim.projection_backward(np.ones((1, 1), np.float32), np.array([[0.1, 0.7]], np.float32),
                                      np.array([[0.2, -0.4]], np.float32), np.array([0.3], np.float32),
                                      np.zeros(1, np.float32), np.zeros(2, np.float32), np.float32(0.0), 4)
    np.testing.assert_allclose(grads["midpoint"], [6 / 7], rtol=1e-6)
    np.testing.assert_allclose(grads["latent_sign"], [[0.3 / 7, 1.5 / 7]], rtol=1e-6)


def test_historical_arithmetic():
    # evidence/arithmetic-reference.json of the reference
    g = json.loads((GOLDEN / "arithmetic.json").read_text())
    w = np.array(g["weights"], np.float32)
    w[1, 2] = -0.0
    x = np.array(g["inputs"], np.float32)
    log_gain = np.array(g["gain"], np.float32)
    log_clip = np.float32(np.log(np.float32(g["clip"])))
    scale = np.abs(w).mean(-1, dtype=np.float32)
    mid = np.array(g["midpoint"], np.float32)
    gain = np.exp(log_gain).astype(np.float32)
    bound = np.exp(log_clip).astype(np.float32)
    out = core.projection_forward(x, w, scale, mid, gain, bound, 4)
    np.testing.assert_allclose(out, np.array(g["output"], np.float32), atol=1e-7, rtol=1e-6)
    grads = optim.projection_backward(np.ones_like(out), x, w, scale, mid, log_gain, log_clip, 4)
    np.testing.assert_allclose(grads["input"], np.array(g["input_grad"], np.float32), atol=1e-7, rtol=1e-6)
    for name, value in g["gradients"].items():
        np.testing.assert_allclose(grads[name], np.array(value, np.float32), atol=1e-7, rtol=1e-6, err_msg=name)
    params = {"latent_sign": w, "scale": scale, "midpoint": mid, "log_gain": log_gain, "log_clip": log_clip}
    for name, value in g["updated"].items():
        p, _, _ = optim.adamw_step(params[name], grads[name], np.zeros_like(params[name]),
                                   np.zeros_like(params[name]), 1, 1e-4)
        np.testing.assert_allclose(p, np.array(value, np.float32), atol=1e-7, rtol=1e-6, err_msg=name)


def test_he4_ffn_against_reference():
    f = load("he4_ffn.npz")
    norm = core.rms(f["residual"], f["ffn_norm"], float(f["epsilon"]))
    np.testing.assert_allclose(norm, f["norm"], rtol=1e-6, atol=1e-7)

    def params(name):
        return {k: f[f"{name}_{k}"] for k in ("latent", "scale", "midpoint", "gain", "bound")}

    gate, up, down = params("gate"), params("up"), params("down")
    # projections bit-exact given identical inputs
    assert np.array_equal(core.projection_forward(f["norm"], gate["latent"], gate["scale"], gate["midpoint"],
                                                  gate["gain"], gate["bound"], 4), f["gate_out"])
    assert np.array_equal(core.projection_forward(f["hidden"], down["latent"], down["scale"], down["midpoint"],
                                                  down["gain"], down["bound"], 8), f["down_out"])
    out = core.he4_ffn(f["norm"], f["residual"], gate, up, down)
    np.testing.assert_allclose(out, f["output"], rtol=1e-5, atol=1e-6)


def test_w1_ffn_against_reference_parts():
    f = load("w1_ffn.npz")
    y = core.w1_ffn(f["x"], f["w_gate"], f["w_up"], f["w_down"])
    np.testing.assert_allclose(y, f["y"], rtol=1e-5, atol=1e-6)


def test_w1a1_ffn_against_reference_parts():
    """Words, popcount dots, per-token means and outputs of the W1A1 block against
    the fixture built from the reference's hard_sign / packed_signs / linear."""
    f = load("w1a1_ffn.npz")
    x = f["x"]
    y, dots = core.w1a1_ffn(x, f["w_gate"], f["w_up"], f["w_down"])
    for tag, v, w in (("gate", x, f["w_gate"]), ("up", x, f["w_up"]), ("down", f["hidden"], f["w_down"])):
        assert np.array_equal(core.pack_bits_rows(v).view(np.int32), f[tag + "_words_in"]), tag
        assert np.array_equal(core.pack_bits_rows(w).view(np.int32), f[tag + "_words_w"]), tag
        words_dot = core.popcount_dot(core.pack_bits_rows(v), core.pack_bits_rows(w), v.shape[1])
        assert np.array_equal(words_dot, f[tag + "_dot"]), tag
        # torch's mean and the kernel's fixed-order mean may differ in the last bit
        np.testing.assert_allclose(core.fixed_mean_abs(v), f[tag + "_mean"], rtol=2e-7, atol=0)
    assert np.array_equal(dots["gate"], f["gate_dot"]) and np.array_equal(dots["up"], f["up_dot"])
    assert np.array_equal(dots["down"], f["down_dot"])
    np.testing.assert_allclose(dots["hidden"], f["hidden"], rtol=1e-6, atol=1e-9)
    np.testing.assert_allclose(y, f["y"], rtol=1e-6, atol=1e-9)


def test_w1a1_popcount_equals_pm_dot():
    rng = np.random.default_rng(3)
    for t, k, o in ((1, 1, 1), (5, 33, 7), (16, 2560, 40), (3, 97, 65)):
        x = rng.standard_normal((t, k)).astype(np.float32)
        w = rng.standard_normal((o, k)).astype(np.float32)
        x[0, 0] = -0.0
        _, dot, s = core.w1a1_projection(x, w, np.ones(o, np.float32))
        pop = core.popcount_dot(core.pack_bits_rows(x), core.pack_bits_rows(w), k)
        assert np.array_equal(dot, pop)
        np.testing.assert_allclose(s, np.abs(x).mean(-1), rtol=1e-5)


# ------------------------------------------------------------------ drafter forward


def tiny_tensors(f, window):
    tensors = {k[2:]: f[k] for k in f.files if k.startswith("t_")}
    tag = f"w{window}_q_"
    tensors.update({k[len(tag):]: f[k] for k in f.files if k.startswith(tag)})
    return tensors


@pytest.mark.parametrize("window", [4096, 5])
def test_tiny_he4_forward_against_reference(window):
    f = load("tiny_he4.npz")
    cfg = drafter.Geometry(hidden=4, intermediate=8, heads=2, kv_heads=1, head_dim=2, window=window)
    tensors = tiny_tensors(f, window)
    tokens = tuple(range(20))
    for anchor in (2, 7, 19):
        logits = drafter.he4_forward(tensors, f["vocabulary"], 19, f["features"], tokens, anchor, cfg)
        np.testing.assert_allclose(logits, f[f"w{window}_logits_{anchor}"], rtol=1e-4, atol=1e-5)
    logits = drafter.he4_forward(tensors, f["vocabulary"], 19, f["features"], tokens, 7, cfg, slots=3)
    np.testing.assert_allclose(logits, f[f"w{window}_logits_7_s3"], rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("case", ["exp", "reach"])
def test_group_loss_against_reference(case):
    # the reference's own TensorWorker.group_loss on the tiny HE4 (worker.py:315-363)
    f, g = load("tiny_he4.npz"), load("group_loss.npz")
    cfg = drafter.Geometry(hidden=4, intermediate=8, heads=2, kv_heads=1, head_dim=2, window=4096)
    windows, slots, positions = group_loss_case(g, case)
    loss = optim.group_loss(tiny_tensors(f, 4096), f["vocabulary"], 19, f["features"], tuple(range(20)), windows,
                            cfg, slots, positions)
    assert loss == pytest.approx(float(g[f"{case}_loss"]), rel=1e-5)


def test_label_weights_rule():
    # worker.py:41-50: exp(-i/7) per window (or the given weights), each window summing to 1/len
    w = optim.label_weights((3, 1, 2))
    assert w.dtype == np.float32 and w.shape == (6,)
    np.testing.assert_allclose([w[:3].sum(), w[3:4].sum(), w[4:].sum()], [1 / 3] * 3, rtol=1e-6)
    np.testing.assert_allclose(w[1] / w[0], np.exp(-1 / 7), rtol=1e-6)
    p = optim.label_weights((2, 3), positions=(4.0, 2.0, 1.0))
    np.testing.assert_allclose(p, [2 / 6, 1 / 6, 4 / 14, 2 / 14, 1 / 14], rtol=1e-6)


def test_cache_layer_golden():
    f = load("layer.npz")
    tensors = {k[2:]: f[k] for k in f.files if k.startswith("t_")}
    ones4 = np.ones(4, np.float32)
    tensors.update({
        "blk.0.ffn_gate.scale": np.abs(tensors["blk.0.ffn_gate.weight"]).mean(-1, dtype=np.float32),
        "blk.0.ffn_up.scale": np.abs(tensors["blk.0.ffn_up.weight"]).mean(-1, dtype=np.float32),
        "blk.0.ffn_down.scale": np.abs(tensors["blk.0.ffn_down.weight"]).mean(-1, dtype=np.float32),
        "blk.0.ffn_gate.midpoint": np.zeros(8, np.float32), "blk.0.ffn_up.midpoint": np.zeros(8, np.float32),
        "blk.0.ffn_down.midpoint": np.zeros(4, np.float32),
        "blk.0.ffn_gate_up.gain": ones4, "blk.0.ffn_gate_up.bound": np.float32(1.0),
        "blk.0.ffn_down.gain": np.ones(8, np.float32), "blk.0.ffn_down.bound": np.float32(1.0),
    })
    cfg = drafter.Geometry(hidden=4, intermediate=8, heads=2, kv_heads=1, head_dim=2)
    context = drafter.layer_context(tensors, 0, f["encoded"], np.arange(3), cfg)
    out = drafter.layer_forward(tensors, 0, f["state"], context, np.arange(3, 19), np.ones((16, 19), bool), cfg)
    np.testing.assert_allclose(out, f["output"], atol=1e-6, rtol=1e-5)


def test_rope_identity_and_rms():
    value = np.array([[[3.0, 4.0]]], np.float32)
    assert np.array_equal(drafter.rope(value, np.array([0]), 1e7), value)
    np.testing.assert_allclose(core.rms(value, np.ones(2, np.float32), 1e-6), value / np.sqrt(12.5 + 1e-6), rtol=1e-6)


def test_cache_storage_rounding_and_overflow():
    v = np.array([0.1234567, -1.234567], np.float32)
    assert np.array_equal(drafter.cache_storage(v), v.astype(np.float16).astype(np.float32))
    with pytest.raises(ValueError, match="overflow"):
        drafter.cache_storage(np.array([70000.0], np.float32))


# ------------------------------------------------------------------ acceptance


def test_greedy_rounds_validated_by_reference_oracle():
    g = json.loads((GOLDEN / "greedy.json").read_text())
    for case in g["rounds"]:
        acc, nxt = acceptance.greedy_prefix(case["targets"], case["drafts"], case["eog"])
        assert (acc, nxt) == (case["accepted"], case["next"]), case
    for case in g["ties"]:
        assert int(acceptance.argmax_rows(np.array(case["row"], np.float32))) == case["argmax"]


def test_greedy_reference_unit_cases():
    # tests/test_verifier.py:28-43 of the reference, as logits
    eog = [99]

    def logits_for(targets, vocab=128):
        rows = np.full((1, len(targets), vocab), -5.0, np.float32)
        for i, t in enumerate(targets):
            rows[0, i, t] = 3.0
        return rows

    acc, nxt, _ = acceptance.accept_greedy(logits_for([5, 9, 10]), np.array([[5, 6]]), eog)
    assert (acc[0], nxt[0]) == (1, 9)
    acc, nxt, _ = acceptance.accept_greedy(logits_for([5, 9, 1]), np.array([[5, 9]]), eog)
    assert (acc[0], nxt[0]) == (2, 1)
    acc, nxt, _ = acceptance.accept_greedy(logits_for([99, 7, 1]), np.array([[99, 7]]), eog)
    assert (acc[0], nxt[0]) == (0, 99)
    bad = logits_for([1, 2])
    bad[0, 1, 3] = np.inf
    with pytest.raises(ValueError, match="nonfinite"):
        acceptance.accept_greedy(bad, np.array([[1]]), eog)


def test_philox_known_answers():
    # Random123 known-answer vectors for Philox4x32-10
    kat = [
        ((0, 0, 0, 0), (0, 0), (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)),
        ((0xFFFFFFFF,) * 4, (0xFFFFFFFF,) * 2, (0x408F276D, 0x41C83B0E, 0xA20BC7C6, 0x6D5451FD)),
        ((0x243F6A88, 0x85A308D3, 0x13198A2E, 0x03707344), (0xA4093822, 0x299F31D0),
         (0xD16CFE09, 0x94FDCCEB, 0x5001E420, 0x24126EA1)),
    ]
    for ctr, key, expected in kat:
        out = acceptance.philox4x32_10(np.array([ctr], dtype=np.uint64), key)
        assert tuple(int(v) for v in out[0]) == expected


def test_exp_fixed_accuracy():
    x = -np.linspace(0, 86, 200001, dtype=np.float32)
    got = acceptance.exp_fixed(x).astype(np.float64)
    want = np.exp(x.astype(np.float64))
    rel = np.abs(got - want) / want
    # one rounding of x log2 e (relative error of the result about |x| 2^-24) plus the polynomial's 2-3 ulp
    assert (rel <= 2e-7 * (1.0 + np.abs(x))).all()
    assert acceptance.exp_fixed(np.float32(0.0)) == 1.0
    floor = acceptance.exp_fixed(np.float32(-86.5))
    assert acceptance.exp_fixed(np.array([-200.0], np.float32))[0] == floor and 0 < floor < 3e-38


def test_fma32_is_correctly_rounded():
    from fractions import Fraction
    rng = np.random.default_rng(12)
    a = rng.standard_normal(3000).astype(np.float32)
    b = rng.standard_normal(3000).astype(np.float32)
    c = (rng.standard_normal(3000) * 10.0 ** rng.integers(-12, 3, 3000)).astype(np.float32)
    got = acceptance.fma32(a, b, c)
    for i in range(a.size):
        exact = Fraction(float(a[i])) * Fraction(float(b[i])) + Fraction(float(c[i]))
        near = np.float32(float(exact))
        cands = (np.nextafter(near, np.float32(-np.inf)), near, np.nextafter(near, np.float32(np.inf)))
        best = min(cands, key=lambda v: (abs(Fraction(float(v)) - exact), int(np.float32(v).view(np.uint32)) & 1))
        assert got[i] == best, i


def test_sample_index_edges():
    w = np.zeros(10000, np.float32)
    w[4097] = 1.0
    for u in (0.0, 0.5, np.float32(1 - 2**-24)):
        assert acceptance.sample_index(w, np.float32(u)) == 4097
    w = np.ones(9000, np.float32)
    assert acceptance.sample_index(w, np.float32(0.0)) == 0
    # the last entry in the contract's order: lane 255, vector 3, item 7
    assert acceptance.sample_index(w, np.float32(1 - 2**-24)) == 8 * (255 + 256 * 3) + 7
    w = np.zeros(40000, np.float32)
    w[[5, 20000, 39999]] = 1.0
    assert acceptance.sample_index(w, np.float32(0.5)) == 20000
    assert acceptance.sample_index(w, np.float32(0.99)) == 39999


def test_chunked_softmax_total():
    rng = np.random.default_rng(3)
    for vocab in (1, 3, 4097, 16384, 40000, 151936):
        row = (rng.standard_normal(vocab) * 3).astype(np.float32)
        m, total = acceptance.row_stats(row)
        assert m == row.max()
        want = np.exp(row.astype(np.float64) - float(m)).sum()
        assert abs(float(total) - want) <= 1e-5 * want


def test_rejection_statistics_match_reference_sampler_check():
    # native/verifier-test.cpp:43-80 of the reference: marginals within 0.035 of p,
    # acceptance within 0.035 of sum(min(p, q)).
    cases = [((0.55, 0.35, 0.10), (0.10, 0.70, 0.20)), ((0.55, 0.35, 0.10), (1.00, 0.00, 0.00)),
             ((0.55, 0.35, 0.10), (0.55, 0.35, 0.10)), ((0.00, 0.60, 0.40), (0.50, 0.50, 0.00))]
    rng = np.random.default_rng(9101)
    trials = 4000
    for p, q in cases:
        p, q = np.array(p), np.array(q)
        lp = np.where(p > 0, np.log(np.maximum(p, 1e-30)), -60.0).astype(np.float32)
        lq = np.where(q > 0, np.log(np.maximum(q, 1e-30)), -60.0).astype(np.float32)
        drafts = rng.choice(3, size=(trials, 1), p=q)
        target = np.broadcast_to(lp, (trials, 2, 3))
        draft = np.broadcast_to(lq, (trials, 1, 3))
        acc, nxt = acceptance.accept_rejection(target, draft, drafts, seed=8101)
        first = np.where(acc == 1, drafts[:, 0], nxt)
        observed = np.bincount(first, minlength=3) / trials
        assert np.abs(observed - p).max() <= 0.035, (p, q, observed)
        assert abs(acc.mean() - np.minimum(p, q).sum()) <= 0.035


def test_rejection_eog_stop():
    # native/verifier-test.cpp:84-97: drafts [eos, eos] under a point mass stop after one token
    lp = np.full((1, 3, 8), -60.0, np.float32)
    lp[..., 2] = 0.0
    lq = lp[:, :2]
    acc, nxt = acceptance.accept_rejection(lp, lq, np.array([[2, 2]]), seed=1, eog=[2])
    assert (int(acc[0]), int(nxt[0])) == (0, 2)


# ------------------------------------------------------------------ optimizer


def test_adamw_against_reference():
    f = load("adamw.npz")
    p, m, v = f["param0"], np.zeros_like(f["param0"]), np.zeros_like(f["param0"])
    for step in range(3):
        p, m, v = optim.adamw_step(p, f[f"grad{step}"], m, v, step + 1, 1e-3)
        np.testing.assert_allclose(m, f[f"exp_avg{step + 1}"], rtol=1e-6, atol=1e-8)
        np.testing.assert_allclose(v, f[f"exp_avg_sq{step + 1}"], rtol=1e-6, atol=1e-10)
        np.testing.assert_allclose(p, f[f"param{step + 1}"], rtol=1e-6, atol=1e-7)


def test_bound_latents_against_reference():
    f = load("bound.npz")
    # the row mean is a float reduction whose order differs from torch's by an ulp
    bounded = optim.bound_latents(f["value"], 3.0)
    np.testing.assert_allclose(bounded, f["bounded"], rtol=4e-7, atol=0)
    assert np.array_equal(bounded >= 0, f["bounded"] >= 0)
    kat = optim.bound_latents(np.array([[0.0, -0.0, 2.0, -14.0], [0.0] * 4], np.float32), 2.0)
    assert np.array_equal(kat, f["kat"])
    assert kat.tolist() == [[0.0, -0.0, 0.25, -1.0], [0.0] * 4]


@pytest.mark.parametrize("rows,cols", [(1, 1), (8, 256), (13, 777), (32, 2560)])
def test_f8_layout_is_a_permutation(rows, cols):
    off = core.f8_offsets(rows, cols)
    assert off.min() >= 0 and off.max() < core.f8_bytes(rows, cols)
    assert np.unique(off).size == rows * cols
    codes = np.random.default_rng(rows).integers(-127, 128, size=(rows, cols))
    assert np.array_equal(core.untile_codes_f8(core.tile_codes_f8(codes), rows, cols), codes.astype(np.int8))


@pytest.mark.parametrize("rows,cols", [(1, 1), (16, 256), (7, 300), (32, 2560)])
def test_c16_layout_is_a_permutation(rows, cols):
    mt = (rows + 15) // 16
    off = core.c16_offsets(rows, cols, mt).reshape(-1)
    assert len(np.unique(off)) == off.size and off.max() < core.codes_ld(cols) // 32 * mt * 512
    codes = np.random.default_rng(rows * cols).integers(-127, 128, size=(rows, cols))
    buf = core.tile_codes_c16(codes)
    assert np.array_equal(buf[core.c16_offsets(rows, cols, mt)], codes)


def test_w8_layout_bits():
    rng = np.random.default_rng(5)
    latent = rng.standard_normal((13, 300)).astype(np.float32)
    words = core.tile_signs_w8(latent).reshape(2, 1, 32, 4)  # 3 words -> one group of 4
    for row, col in [(0, 0), (7, 299), (12, 129), (8, 17), (3, 255)]:
        n, g, w = row // 8, row % 8, col // 128
        c = col % 128
        ks, r, t, j = c // 32, (c % 32) // 16, (c % 16) // 4, c % 4
        bit = (int(words[n, w // 4, 4 * g + t, w % 4]) >> (8 * j + 2 * ks + r)) & 1
        assert bit == int(latent[row, col] >= 0)
    assert words[1, :, 4 * 5:].sum() == 0  # rows 13..15 are padding
    assert words[:, :, :, 3].sum() == 0    # the fourth word is past column 383
    inter = core.tile_signs_w8(latent, 2, 1).reshape(4, 1, 32, 4)
    assert np.array_equal(inter[1::2], words) and not inter[0::2].any()
