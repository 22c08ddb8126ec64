"""The drop-in model API on the GPU against the reference's own outputs
(golden fixtures generated from w1a1_eagle.model) and against the oracle."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch
from torch import nn

from conftest import GOLDEN, group_loss_case, package, submodule
from oracle import core, optim

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def bd():
    return package()


def load(name):
    return np.load(GOLDEN / name)


def t(a):
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(DEV)


def projection_from_case(bd, f, i):
    latent = f[f"{i}_latent"]
    gain = nn.Parameter(t(f[f"{i}_log_gain"]))
    clip = nn.Parameter(t(f[f"{i}_log_clip"]))
    layer = bd.Projection(torch.from_numpy(latent), int(f[f"{i}_bits"]), gain, clip).to(DEV)
    with torch.no_grad():
        layer.scale.copy_(t(f[f"{i}_scale"]))
        layer.midpoint.copy_(t(f[f"{i}_midpoint"]))
    return layer


def test_projection_forward_and_gradients_match_reference(bd):
    f = load("projection.npz")
    for i in range(int(f["count"])):
        layer = projection_from_case(bd, f, i)
        value = t(f[f"{i}_value"]).requires_grad_()
        out = layer(value)
        # forward: integer dot and epilogue in the reference's operation order; bit-exact
        # whenever this GPU's exp(log_gain) equals the reference host's
        same_gain = np.array_equal(layer.log_gain.detach().exp().cpu().numpy(), f[f"{i}_gain"]) and \
            np.array_equal(layer.log_clip.detach().exp().cpu().numpy(), f[f"{i}_bound"])
        if same_gain:
            assert np.array_equal(out.detach().cpu().numpy(), f[f"{i}_output"]), i
        else:
            np.testing.assert_allclose(out.detach().cpu().numpy(), f[f"{i}_output"], rtol=1e-5, atol=1e-6)
        (out * t(f[f"{i}_upstream"])).sum().backward()
        grads = {"input": value.grad, "latent_sign": layer.latent_sign.grad, "scale": layer.scale.grad,
                 "midpoint": layer.midpoint.grad, "log_gain": layer.log_gain.grad, "log_clip": layer.log_clip.grad}
        # gradients: the GEMMs see dL as two bf16 halves (~16 significant bits), the
        # reference multiplies in fp32; the bound is far inside 1e-2 relative
        for name, g in grads.items():
            want = np.asarray(f[f"{i}_grad_{name}"], np.float64)
            got = g.detach().cpu().numpy().astype(np.float64)
            scale = max(np.abs(want).max(), 1e-30)
            np.testing.assert_allclose(got, want, rtol=0, atol=1e-4 * scale, err_msg=f"case {i} {name}")
            assert np.linalg.norm(got - want) <= 1e-4 * max(np.linalg.norm(want), 1e-30), (i, name)


@pytest.mark.parametrize("tokens", [40, 300])
def test_projection_large_shapes_against_oracle(bd, tokens):
    g = torch.Generator().manual_seed(tokens)
    inner, outer = 2560, 9728
    latent = torch.randn((outer, inner), generator=g) * 0.02
    log_gain = torch.randn(inner, generator=g) * 0.2
    log_clip = torch.tensor(0.3)
    layer = bd.Projection(latent, 4, nn.Parameter(log_gain.clone()), nn.Parameter(log_clip.clone())).to(DEV)
    with torch.no_grad():
        layer.midpoint.copy_(torch.randn(outer, generator=g) * 0.05)
    value = (torch.randn((tokens, inner), generator=g) * 1.5)
    x = value.to(DEV).requires_grad_()
    out = layer(x)
    gain_dev = layer.log_gain.detach().exp().cpu().numpy()
    bound_dev = layer.log_clip.detach().exp().cpu().numpy()
    want = core.projection_forward(value.numpy(), latent.numpy(), layer.scale.detach().cpu().numpy(),
                                   layer.midpoint.detach().cpu().numpy(), gain_dev, bound_dev, 4)
    assert np.array_equal(out.detach().cpu().numpy(), want)
    upstream = torch.randn((tokens, outer), generator=g)
    (out * upstream.to(DEV)).sum().backward()
    ref = optim.projection_backward(upstream.numpy(), value.numpy(), latent.numpy(),
                                    layer.scale.detach().cpu().numpy(), layer.midpoint.detach().cpu().numpy(),
                                    log_gain.numpy(), np.float32(0.3), 4)
    got = {"input": x.grad, "latent_sign": layer.latent_sign.grad, "scale": layer.scale.grad,
           "midpoint": layer.midpoint.grad, "log_gain": layer.log_gain.grad, "log_clip": layer.log_clip.grad}
    for name, gv in got.items():
        a, b = gv.detach().cpu().numpy().astype(np.float64), np.asarray(ref[name], np.float64)
        err = np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)
        assert err < 1e-3, (name, err)


def test_projection_learned_window_against_oracle(bd):
    """The learned straight-through window |w| <= alpha (alpha = 0.05 initially):
    the latent gradient masked by the window and the gradient of log alpha (the
    sum over latents outside the window of their gradient times sign(w)), both
    from the epilogue of the tcgen05 latent-gradient GEMM, against the oracle."""
    g = torch.Generator().manual_seed(5)
    inner, outer, tokens = 2560, 9728, 256
    latent = torch.randn((outer, inner), generator=g) * 0.02
    log_gain = torch.randn(inner, generator=g) * 0.2
    layer = bd.Projection(latent, 8, nn.Parameter(log_gain.clone()), nn.Parameter(torch.tensor(0.1)), window=0.05,
                          learned_window=True).to(DEV)
    value = torch.randn((tokens, inner), generator=g)
    out = layer(value.to(DEV))
    upstream = torch.randn((tokens, outer), generator=g)
    (out * upstream.to(DEV)).sum().backward()
    alpha = np.float32(layer.log_window.detach().exp().cpu().numpy())  # the device's exp, as the kernel used
    ref = optim.projection_backward(upstream.numpy(), value.numpy(), latent.numpy(),
                                    layer.scale.detach().cpu().numpy(), layer.midpoint.detach().cpu().numpy(),
                                    log_gain.numpy(), np.float32(0.1), 8, window=alpha)
    got = layer.latent_sign.grad.cpu().numpy().astype(np.float64)
    want = np.asarray(ref["latent_sign"], np.float64)
    assert np.linalg.norm(got - want) / np.linalg.norm(want) < 1e-3
    outside = np.abs(latent.numpy()) > alpha
    assert outside.any() and not got[outside].any()  # masked exactly outside the window
    gw, ww = float(layer.log_window.grad.cpu()), float(ref["log_window"])
    assert abs(gw - ww) <= 1e-3 * abs(ww), (gw, ww)


def test_latent_gradients_accumulate_as_one_product(bd):
    """``LatentGradients``: three backward passes (256, 100 and 300 rows; the 100-row
    pass leaves padding columns, and ``rows`` = 400 forces a flush before the third)
    give the latent and window gradients of the same passes accumulated by autograd,
    within the fp32 summation-order difference, and every other gradient unchanged."""
    g = torch.Generator().manual_seed(11)
    inner, outer = 2560, 1536
    latent = torch.randn((outer, inner), generator=g) * 0.02
    log_gain = torch.randn(inner, generator=g) * 0.2
    passes = [(torch.randn((n, inner), generator=g), torch.randn((n, outer), generator=g)) for n in (256, 100, 300)]

    def run(accumulate):
        layer = bd.Projection(latent, 4, nn.Parameter(log_gain.clone()), nn.Parameter(torch.tensor(0.1)),
                              window=0.05, learned_window=True).to(DEV)
        ready = []
        acc = bd.LatentGradients(layer, 400, on_ready=ready.append) if accumulate else None
        if acc is not None:
            acc.__enter__()
        for value, upstream in passes:
            (layer(value.to(DEV)) * upstream.to(DEV)).sum().backward()
            if acc is not None and len(ready) == 0:
                assert layer.latent_sign.grad is None  # deferred to the flush
        if acc is not None:
            acc.__exit__(None, None, None)
            assert [id(p) for p in ready] == [id(layer.latent_sign), id(layer.log_window)] * 2
        torch.cuda.synchronize()
        return {n: p.grad.detach().cpu().double() for n, p in layer.named_parameters()}

    want, got = run(False), run(True)
    assert set(got) == set(want)
    for name in want:
        if name in ("latent_sign", "log_window"):
            err = float((got[name] - want[name]).norm() / want[name].norm())
            assert err < 1e-5, (name, err)
        else:
            assert torch.equal(got[name], want[name]), name
    outside = latent.abs() > 0.05
    assert outside.any() and not got["latent_sign"][outside].any()


def test_hard_sign_forward_backward(bd):
    x = torch.tensor([-2.0, -1.0, -0.0, 0.0, 0.5, 1.0, 1.5], device=DEV, requires_grad=True)
    y = bd.hard_sign(x)
    assert y.tolist() == [-1.0, -1.0, 1.0, 1.0, 1.0, 1.0, 1.0]
    y.backward(torch.arange(1.0, 8.0, device=DEV))
    assert x.grad.tolist() == [0.0, 2.0, 3.0, 4.0, 5.0, 6.0, 0.0]
    with pytest.raises(ValueError, match="latent signs must be F32"):
        bd.hard_sign(x.detach().double())


def tiny_model(bd, window):
    f = load("tiny_he4.npz")
    cfg = bd.Geometry(hidden=4, intermediate=8, heads=2, kv_heads=1, head_dim=2, window=window)
    tensors = {k[2:]: torch.from_numpy(f[k]) for k in f.files if k.startswith("t_")}
    model = bd.HE4(tensors, torch.from_numpy(f["vocabulary"]), 19, cfg).to(DEV)
    perturb = torch.Generator().manual_seed(23)  # the fixture's quantizer perturbation, same draw order
    with torch.no_grad():
        for block in model.blocks:
            block.gate.log_gain.copy_(0.3 * torch.randn(4, generator=perturb))
            block.gate.log_clip.fill_(float(0.3 * torch.randn((), generator=perturb)))
            block.down.log_gain.copy_(0.3 * torch.randn(8, generator=perturb))
            block.down.log_clip.fill_(float(0.3 * torch.randn((), generator=perturb)))
            for p in (block.gate, block.up, block.down):
                p.midpoint.copy_(0.05 * torch.randn(p.midpoint.shape, generator=perturb))
    return f, model


# The frozen projections (q, k, v, o, fc, the tied head) run on bf16 tensor cores
# with split operands (hi + lo, fp32 accumulation): within ~1e-5 of the
# reference's fp32 products, hence the absolute tolerance on the O(1) logits.
LOGITS_ATOL = 3e-5


@pytest.mark.parametrize("window", [4096, 5])
def test_he4_forward_matches_reference_logits(bd, window):
    f, model = tiny_model(bd, window)
    features = torch.from_numpy(f["features"])
    tokens = tuple(range(20))
    with torch.no_grad():
        for anchor in (2, 7, 19):
            logits = model.forward(features, tokens, anchor)
            np.testing.assert_allclose(logits.cpu().numpy(), f[f"w{window}_logits_{anchor}"], rtol=1e-4,
                                       atol=LOGITS_ATOL)
        logits = model.forward(features, tokens, 7, 3)
        np.testing.assert_allclose(logits.cpu().numpy(), f[f"w{window}_logits_7_s3"], rtol=1e-4,
                                   atol=LOGITS_ATOL)
    # with gradients enabled the projections take the training path: same logits
    logits = model.forward(features, tokens, 7)
    np.testing.assert_allclose(logits.detach().cpu().numpy(), f[f"w{window}_logits_7"], rtol=1e-4, atol=LOGITS_ATOL)


def test_group_hidden_matches_single_windows(bd):
    f, model = tiny_model(bd, 5)
    features = torch.from_numpy(f["features"])
    tokens = tuple(range(20))
    hidden = model.group_hidden(features, tokens, (3, 9, 15), 6)
    for i, anchor in enumerate((3, 9, 15)):
        single = model.group_hidden(features, tokens, (anchor,), 6)
        torch.testing.assert_close(hidden[i], single[0], rtol=1e-5, atol=1e-6)
    logits = torch.nn.functional.linear(hidden[1], model.vocabulary)
    with torch.no_grad():
        direct = model.forward(features, tokens, 9, 6)
    torch.testing.assert_close(logits, direct, rtol=1e-4, atol=1e-5)


def test_cache_layer_golden(bd):
    f = load("layer.npz")
    tensors = {k[2:]: torch.from_numpy(f[k]) for k in f.files if k.startswith("t_")}
    cfg = bd.Geometry(hidden=4, intermediate=8, heads=2, kv_heads=1, head_dim=2)
    layer = bd.Layer(tensors, "blk.0.", cfg).to(DEV)
    with torch.no_grad():
        context = layer.context(t(f["encoded"]), torch.arange(3, device=DEV))
        out = layer.forward(t(f["state"]), context, torch.arange(3, 19, device=DEV),
                            torch.ones((16, 19), dtype=torch.bool, device=DEV))
    np.testing.assert_allclose(out.cpu().numpy(), f["output"], atol=1e-5, rtol=1e-4)


def test_bound_and_clamp_latents(bd):
    f = load("bound.npz")
    layer = bd.Projection(torch.from_numpy(f["value"]), 4, nn.Parameter(torch.zeros(21)),
                          nn.Parameter(torch.tensor(0.0))).to(DEV)
    bd.bound_latents(layer, 3.0)
    np.testing.assert_allclose(layer.latent_sign.detach().cpu().numpy(), f["bounded"], rtol=4e-7, atol=0)
    kat = bd.Projection(torch.tensor([[0.0, -0.0, 2.0, -14.0], [0.0] * 4]), 4, nn.Parameter(torch.zeros(4)),
                        nn.Parameter(torch.tensor(0.0))).to(DEV)
    bd.bound_latents(kat, 2.0)
    assert np.array_equal(kat.latent_sign.detach().cpu().numpy(), f["kat"])
    tiny = bd.Projection(torch.tensor([[1.0, -1e-38, 1.0, 1.0]]), 4, nn.Parameter(torch.zeros(4)),
                         nn.Parameter(torch.tensor(0.0))).to(DEV)
    with pytest.raises(ValueError, match="bounded latent scale changed a sign"):
        bd.bound_latents(tiny, 1e30)
    assert tiny.latent_sign[0, 1].item() == pytest.approx(-1e-38)  # refused before writing
    wide = bd.Projection(torch.tensor([[3.0, -2.0, 0.5]]), 4, nn.Parameter(torch.zeros(3)),
                         nn.Parameter(torch.tensor(0.0))).to(DEV)
    bd.clamp_latents(wide)
    assert wide.latent_sign.tolist() == [[1.0, -1.0, 0.5]]


def test_adamw_latent_matches_reference_and_repacks(bd):
    qat = submodule("qat")
    f = load("adamw.npz")
    layer = bd.Projection(torch.from_numpy(f["param0"]), 4, nn.Parameter(torch.zeros(13)),
                          nn.Parameter(torch.tensor(0.0))).to(DEV)
    for p in layer.parameters():
        p.requires_grad_(p is layer.latent_sign)
    opt = qat.BitAdamW(layer, qat.UpdatePolicy(step_sizes={**qat.REFERENCE_STEP_SIZES, "sign": 1e-3}))
    for step in range(3):
        layer.latent_sign.grad = t(f[f"grad{step}"])
        opt.step()
        st = opt.state[id(layer.latent_sign)]
        np.testing.assert_allclose(st["exp_avg"].cpu().numpy(), f[f"exp_avg{step + 1}"], rtol=1e-6, atol=1e-8)
        np.testing.assert_allclose(st["exp_avg_sq"].cpu().numpy(), f[f"exp_avg_sq{step + 1}"], rtol=1e-6,
                                   atol=1e-10)
        np.testing.assert_allclose(layer.latent_sign.detach().cpu().numpy(), f[f"param{step + 1}"], rtol=1e-6,
                                   atol=1e-7)
        # the fused re-pack equals a fresh tiling of the updated latent
        fresh = bd.ops.tile_w8(layer.latent_sign.detach().contiguous())
        assert torch.equal(layer.signs_w8(), fresh)


def test_grad_norm_and_clip_coefficient(bd):
    qat = submodule("qat")
    g = torch.Generator().manual_seed(3)
    params = [nn.Parameter(torch.zeros(s, device=DEV)) for s in ((300, 70), (5,), (1,), (4096, 33))]
    for p in params:
        p.grad = (torch.randn(p.shape, generator=g) * 0.01).to(DEV)
    total, coef = qat.clip_grad_norm(params, 1.0)
    want = torch.linalg.vector_norm(torch.stack([torch.linalg.vector_norm(p.grad.double()) for p in params]))
    assert abs(total.item() - want.item()) <= 1e-6 * want.item()
    assert coef.item() == pytest.approx(min(1.0, 1.0 / (want.item() + 1e-6)), rel=1e-6)
    params[0].grad[3, 3] = float("nan")
    with pytest.raises(ValueError, match="non-finite total norm"):
        qat.clip_grad_norm(params, 1.0)


def test_qat_update_smoke(bd):
    qat = submodule("qat")
    f, model = tiny_model(bd, 4096)
    features = torch.from_numpy(f["features"]).to(DEV)
    tokens = tuple(range(20))
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    opt = qat.BitAdamW(model)
    windows = (qat.Window(3, (4, 5, 6)), qat.Window(10, (11, 12, 13, 14, 15)))
    loss, norm = qat.update(model, opt, features, tokens, windows, slots=6)
    assert np.isfinite(loss) and np.isfinite(norm) and norm > 0
    changed = [n for n, p in model.named_parameters() if not torch.equal(p.detach(), before[n])]
    assert any(n.endswith("latent_sign") for n in changed)
    assert any(n.endswith("log_gain") for n in changed)
    for block in model.blocks:  # the W8 caches follow the updated latents
        for proj in (block.gate, block.up, block.down):
            assert torch.equal(proj.signs_w8(), bd.ops.tile_w8(proj.latent_sign.detach().contiguous()))


# Tolerances of the loss-head parity against the reference's own group_loss.  The
# 4-bit activation codes and the clip masks are discontinuous: perturbing the
# reference's frozen fp32 weights by a relative 1e-4 (ten times the error of the
# split-bf16 products here) moved its loss by at most 1.1e-4 and its whole gradient
# vector by at most 2.2e-3 in relative norm, while single per-projection scalars
# (log_clip) moved by up to 37 %.  Hence a bound on the loss and on the global
# gradient, with a tenfold margin, rather than one per tensor.
GROUP_LOSS_RTOL = 1e-3
GROUP_GRAD_RTOL = 2e-2


@pytest.mark.parametrize("case", ["exp", "reach"])
def test_group_loss_matches_reference_loss_and_gradients(bd, case):
    """``qat.group_loss`` against the reference's ``TensorWorker.group_loss``
    (``worker.py:315-363``) on the tiny HE4: exponential label weights over one
    head chunk, per-position weights over 132 label rows (two 128-row chunks)."""
    qat = submodule("qat")
    g = load("group_loss.npz")
    f, model = tiny_model(bd, 4096)
    windows, slots, positions = group_loss_case(g, case)
    features = torch.from_numpy(f["features"]).to(DEV)
    model.zero_grad(set_to_none=True)
    loss = qat.group_loss(model, features, tuple(range(20)), tuple(qat.Window(a, l) for a, l in windows), slots,
                          positions)
    assert float(loss) == pytest.approx(float(g[f"{case}_loss"]), rel=GROUP_LOSS_RTOL)
    prefix = f"{case}_grad_"
    want = {k[len(prefix):]: g[k] for k in g.files if k.startswith(prefix)}
    got = {n: p.grad.detach().cpu().numpy() for n, p in model.named_parameters() if p.grad is not None}
    assert set(got) == set(want)
    num = sum(float(np.square(got[n].astype(np.float64) - want[n]).sum()) for n in want)
    den = sum(float(np.square(want[n].astype(np.float64)).sum()) for n in want)
    assert math.sqrt(num / den) <= GROUP_GRAD_RTOL


@pytest.mark.parametrize("vocab_bf16", [False, True])
def test_loss_head_against_fp64(bd, vocab_bf16):
    """The fused cross-entropy head (tcgen05 products of split-bf16 operands, the
    logits never written) against a float64 evaluation of the reference's
    weighted cross_entropy(linear(head, vocabulary)) and its gradient."""
    qat = submodule("qat")
    g = torch.Generator().manual_seed(21)
    rows, hidden, vocab = 300, 2560, 50000
    vocabulary = torch.randn((vocab, hidden), generator=g) * 0.02
    if vocab_bf16:
        vocabulary = vocabulary.to(torch.bfloat16).float()
    head = torch.randn((rows, hidden), generator=g)
    labels = torch.randint(0, vocab, (rows,), generator=g)
    weights = torch.rand(rows, generator=g) / rows

    class Owner(nn.Module):
        def __init__(self):
            super().__init__()
            self.register_buffer("vocabulary", vocabulary.to(DEV))

    owner = Owner()
    loss, d_head = qat.loss_head(head.to(DEV), owner, labels.to(DEV), weights.to(DEV))
    h64, v64 = head.double().to(DEV), vocabulary.double().to(DEV)
    logits = h64 @ v64.T
    lse = torch.logsumexp(logits, -1)
    want = (weights.double().to(DEV) * (lse - logits[torch.arange(rows), labels.to(DEV)])).sum()
    p = torch.softmax(logits, -1)
    p[torch.arange(rows), labels.to(DEV)] -= 1
    want_d = (p * weights.double().to(DEV)[:, None]) @ v64
    assert abs(float(loss) - float(want)) <= 1e-5 * abs(float(want))
    # fp32 accumulation over 2 x 50000 products on the tensor cores: observed 1.5e-4 to 2.5e-4
    err = float((d_head.double() - want_d).norm() / want_d.norm())
    assert err < 1e-3, err
