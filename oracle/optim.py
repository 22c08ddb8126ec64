"""Oracle for the QAT backward and update of the binary projections.

Test infrastructure only (see ``oracle/__init__.py``).
  * :func:`projection_backward` restates the autograd graph of
    ``Projection.forward`` (``w1a1_eagle/model.py:128-150``) with the
    ``SIGN`` straight-through backward (``model.py:71-73``) and torch's tie
    rule for ``minimum``/``maximum`` (the gradient splits 0.5/0.5 on ties);
  * :func:`adamw_step` restates one ``torch.optim.AdamW`` step with
    ``weight_decay=0`` in the single-tensor order used by the reference's
    golden test (``tests/numerical/test_model.py:544-553``) and the fused
    update of ``w1a1_eagle/numerical/worker.py:365-392``;
  * :func:`bound_latents` / :func:`clamp_latents` restate ``model.py:153-169``;
  * :func:`label_weights` and :func:`group_loss` restate the weighted
    cross-entropy of the drafted positions,
    ``w1a1_eagle/numerical/worker.py:41-50, 315-363`` (its value; the gradients
    are pinned by the reference's own fixture).
"""

from __future__ import annotations

import numpy as np

from .core import hard_sign, quantize_codes

F32 = np.float32


def projection_backward(grad_out, value, latent, scale, midpoint, log_gain, log_clip, bits, window=1.0):
    """Gradients of ``sum(grad_out * Projection(value))`` w.r.t. every input.

    Returns a dict with ``input``, ``latent_sign``, ``scale``, ``midpoint``,
    ``log_gain``, ``log_clip`` and ``log_window``.  ``log_gain``/``log_clip`` are
    the raw parameters (exponentiated here with numpy).  ``log_window`` is the
    gradient of a learned straight-through window ``window = exp(log_window)``:
    the clip ``|w| <= window`` passes the sign gradient inside the window, and
    outside it the clip's output moves with the window, by ``sign(w)``
    (the weight-side counterpart of the activation clip of ``model.py:136-139``).
    """
    G = np.asarray(grad_out, dtype=np.float32)
    x = np.asarray(value, dtype=np.float32)
    latent = np.asarray(latent, dtype=np.float32)
    gain = np.exp(np.asarray(log_gain, dtype=np.float32)).astype(np.float32)
    bound = F32(np.exp(F32(log_clip)))
    codes, step = quantize_codes(x, gain, bound, bits)
    maximum = F32((1 << (bits - 1)) - 1)
    signs = hard_sign(latent)
    scale = np.asarray(scale, dtype=np.float32)
    scale_c = np.maximum(scale, F32(0.0))
    midpoint = np.asarray(midpoint, dtype=np.float32)
    gained = x * gain
    ratio = (F32(1.0) / bound) * maximum
    clipped = np.maximum(np.minimum(gained, bound), -bound)
    values = codes * step
    dot = (values @ signs.T).astype(np.float32)
    d_scale_c = (G * dot).sum(0).astype(np.float32)
    dL = (G * scale_c).astype(np.float32)
    d_values = (dL @ signs).astype(np.float32)
    d_signs = (dL.T @ values).astype(np.float32)
    vsum = values.sum(-1, keepdims=True).astype(np.float32)
    d_mid = (G * vsum).sum(0).astype(np.float32)
    d_values = (d_values + (G * midpoint).sum(-1, keepdims=True)).astype(np.float32)
    inside = np.abs(latent) <= F32(window)
    d_latent = (d_signs * inside).astype(np.float32)
    d_window = F32(np.where(inside, 0.0, d_signs * np.where(latent >= 0, 1.0, -1.0)).sum(dtype=np.float64))
    d_log_window = F32(d_window * F32(window))
    d_scale = (d_scale_c * (scale >= 0)).astype(np.float32)
    d_codes = (d_values * step).astype(np.float32)
    d_step = F32((d_values * codes).sum())
    d_bound = F32(d_step / maximum)
    d_norm = d_codes
    d_clipped = (d_norm * ratio).astype(np.float32)
    d_ratio = F32((d_norm * clipped).sum())
    recip = F32(F32(1.0) / bound)
    d_bound = F32(d_bound + F32(d_ratio * maximum) * -(recip * recip))
    mn = np.minimum(gained, bound)
    # maximum(mn, -bound)
    to_mn = np.where(mn > -bound, 1.0, np.where(mn == -bound, 0.5, 0.0)).astype(np.float32)
    d_mn = d_clipped * to_mn
    d_bound = F32(d_bound - (d_clipped * (F32(1.0) - to_mn)).sum())
    # minimum(gained, bound)
    to_g = np.where(gained < bound, 1.0, np.where(gained == bound, 0.5, 0.0)).astype(np.float32)
    d_gained = d_mn * to_g
    d_bound = F32(d_bound + (d_mn * (F32(1.0) - to_g)).sum())
    d_x = (d_gained * gain).astype(np.float32)
    d_gain = (d_gained * x).sum(0).astype(np.float32)
    return {
        "log_window": d_log_window,
        "input": d_x,
        "latent_sign": d_latent,
        "scale": d_scale,
        "midpoint": d_mid,
        "log_gain": (d_gain * gain).astype(np.float32),
        "log_clip": F32(d_bound * bound),
    }


def adamw_step(param, grad, exp_avg, exp_avg_sq, step, lr, beta1=0.9, beta2=0.999, eps=1e-8):
    """One AdamW update with weight decay 0; returns new ``(param, exp_avg, exp_avg_sq)``.

    ``step`` is the 1-based step count after incrementing.
    """
    p = np.asarray(param, dtype=np.float32)
    g = np.asarray(grad, dtype=np.float32)
    m = np.asarray(exp_avg, dtype=np.float32)
    v = np.asarray(exp_avg_sq, dtype=np.float32)
    weight = F32(1.0 - beta1)
    m = (m + weight * (g - m)).astype(np.float32)
    v = (v * F32(beta2) + (F32(1.0 - beta2) * g) * g).astype(np.float32)
    bias1 = 1.0 - beta1**step
    bias2 = 1.0 - beta2**step
    step_size = lr / bias1
    denom = (np.sqrt(v) / F32(bias2**0.5) + F32(eps)).astype(np.float32)
    p = (p + (F32(-step_size) * m) / denom).astype(np.float32)
    return p, m, v


def bound_latents(latent, multiple: float):
    """``clamp(latent / (multiple * mean_row|latent|), -1, 1)``; refuses sign changes."""
    latent = np.asarray(latent, dtype=np.float32)
    mean = np.abs(latent).mean(-1, keepdims=True, dtype=np.float32)
    denom = np.where(mean > 0, mean * F32(multiple), F32(1.0)).astype(np.float32)
    bounded = np.clip(latent / denom, F32(-1.0), F32(1.0)).astype(np.float32)
    if not np.array_equal(bounded >= 0, latent >= 0):
        raise ValueError("bounded latent scale changed a sign")
    return bounded


def clamp_latents(latent):
    return np.clip(np.asarray(latent, dtype=np.float32), F32(-1.0), F32(1.0))


def label_weights(lengths, positions=None) -> np.ndarray:
    """``label_weights`` (``worker.py:41-50``): per window ``exp(-i / 7)`` for its
    ``i``-th label (or the given per-position weights), each window normalised to
    sum ``1 / len(lengths)``; fp32 as in torch."""
    parts = []
    for length in lengths:
        if positions is None:
            weights = np.exp(-np.arange(length).astype(F32) / F32(7)).astype(F32)
        else:
            weights = np.asarray(positions[:length], dtype=F32)
        parts.append((weights / weights.sum(dtype=F32) / F32(len(lengths))).astype(F32))
    return np.concatenate(parts)


def group_loss(tensors, vocabulary, mask, features, tokens, windows, cfg, slots=None, positions=None) -> float:
    """Value of ``TensorWorker.group_loss`` (``worker.py:315-363``).

    ``windows`` is a sequence of ``(anchor, labels)``.  Each window drafts a
    block of ``size`` slots (``HE4.block``, ``model.py:323-327``); its label rows
    are slots ``1 .. min(len(labels), size - 1)`` of that block, whose logits
    equal ``HE4.forward`` at the window's anchor (``group_hidden`` masks each
    window to its own context, ``model.py:329-367``).  The loss is the
    label-weighted sum of the rows' cross-entropies, accumulated here in fp64.
    """
    from .drafter import he4_forward

    size = cfg.slots if slots is None else slots
    if not windows or any(not labels for _, labels in windows):
        raise ValueError("an update requires supervised windows")
    if not 2 <= size <= cfg.slots:
        raise ValueError("an update requires at least one drafted position")
    lengths = tuple(min(len(labels), size - 1) for _, labels in windows)
    weights = label_weights(lengths, positions).astype(np.float64)
    total, row = 0.0, 0
    for (anchor, labels), length in zip(windows, lengths):
        logits = he4_forward(tensors, vocabulary, mask, features, tokens, anchor, cfg, slots=size)
        rows = logits[1:1 + length].astype(np.float64)
        peak = rows.max(-1, keepdims=True)
        lse = peak[:, 0] + np.log(np.exp(rows - peak).sum(-1))
        picked = rows[np.arange(length), np.asarray(labels[:length])]
        total += float((weights[row:row + length] * (lse - picked)).sum())
        row += length
    return total
