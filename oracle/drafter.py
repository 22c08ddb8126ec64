"""Oracle for the HE4 block-drafter forward (numpy, F32).

Test infrastructure only (see ``oracle/__init__.py``).  Restates
``w1a1_eagle/model.py``: ``rms`` (50-51), ``rope`` (54-63), ``cache_storage``
(98-102), ``Layer.context`` (195-200), ``Layer.forward`` (202-223) and
``HE4.forward`` (369-396).  Weights are passed as a dict keyed by the GGUF
tensor names the reference uses (``fc.weight``, ``blk.{i}.attn_q.weight`` ...),
plus per-layer quantizer parameters (``blk.{i}.ffn_*.{scale,midpoint}``,
``blk.{i}.ffn_gate_up.{gain,bound}``, ``blk.{i}.ffn_down.{gain,bound}``).
"""

from __future__ import annotations

import math

import numpy as np

from .core import he4_ffn, rms

F32 = np.float32


def rope(value: np.ndarray, positions: np.ndarray, theta: float) -> np.ndarray:
    """Rotary embedding over the last axis of ``value [n, heads, d]`` (``model.py:54-63``)."""
    width = value.shape[-1]
    frequency = np.power(F32(theta), -(np.arange(0, width, 2, dtype=np.float32) / F32(width))).astype(np.float32)
    angle = (np.asarray(positions, dtype=np.float32)[:, None] * frequency).astype(np.float32)
    angle = np.concatenate((angle, angle), -1)[:, None, :]
    half = width // 2
    rotated = np.concatenate((-value[..., half:], value[..., :half]), -1)
    return (value * np.cos(angle) + rotated * np.sin(angle)).astype(np.float32)


def cache_storage(value: np.ndarray) -> np.ndarray:
    """Round through F16 and refuse overflow (``model.py:98-102``)."""
    with np.errstate(over="ignore"):
        rounded = np.asarray(value, dtype=np.float32).astype(np.float16).astype(np.float32)
    if not np.isfinite(rounded).all():
        raise ValueError("F16 cache storage overflow")
    return rounded


class Geometry:
    """Plain mirror of ``model.py:11-47`` (validation lives in the product)."""

    def __init__(self, hidden=2560, intermediate=9216, heads=32, kv_heads=8, head_dim=128,
                 layers=6, slots=16, taps=8, window=4096, epsilon=1e-6, theta=1e7):
        self.hidden, self.intermediate = hidden, intermediate
        self.heads, self.kv_heads, self.head_dim = heads, kv_heads, head_dim
        self.layers, self.slots, self.taps, self.window = layers, slots, taps, window
        self.epsilon, self.theta = epsilon, theta


def _linear(value, weight):
    return (np.asarray(value, dtype=np.float32) @ np.asarray(weight, dtype=np.float32).T).astype(np.float32)


def layer_context(tensors, index, encoded, positions, cfg):
    """``Layer.context`` (``model.py:195-200``)."""
    p = f"blk.{index}."
    key = _linear(encoded, tensors[p + "attn_k.weight"]).reshape(-1, cfg.kv_heads, cfg.head_dim)
    value = _linear(encoded, tensors[p + "attn_v.weight"]).reshape(-1, cfg.kv_heads, cfg.head_dim)
    key = rope(rms(key, tensors[p + "attn_k_norm.weight"], cfg.epsilon), positions, cfg.theta)
    return cache_storage(key), cache_storage(value)


def ffn_params(tensors, index):
    p = f"blk.{index}."
    gate = {
        "latent": tensors[p + "ffn_gate.weight"],
        "scale": tensors[p + "ffn_gate.scale"],
        "midpoint": tensors[p + "ffn_gate.midpoint"],
        "gain": tensors[p + "ffn_gate_up.gain"],
        "bound": tensors[p + "ffn_gate_up.bound"],
    }
    up = dict(gate, latent=tensors[p + "ffn_up.weight"], scale=tensors[p + "ffn_up.scale"],
              midpoint=tensors[p + "ffn_up.midpoint"])
    down = {
        "latent": tensors[p + "ffn_down.weight"],
        "scale": tensors[p + "ffn_down.scale"],
        "midpoint": tensors[p + "ffn_down.midpoint"],
        "gain": tensors[p + "ffn_down.gain"],
        "bound": tensors[p + "ffn_down.bound"],
    }
    return gate, up, down


def layer_forward(tensors, index, state, context, positions, allowed, cfg):
    """``Layer.forward`` (``model.py:202-223``)."""
    residual = attention_residual(tensors, index, state, context, positions, allowed, cfg)
    return ffn_residual(tensors, index, residual, cfg)


def ffn_residual(tensors, index, residual, cfg):
    """The feed-forward half of ``Layer.forward`` (``model.py:220-223``)."""
    p = f"blk.{index}."
    norm = rms(residual, tensors[p + "ffn_norm.weight"], cfg.epsilon)
    gate, up, down = ffn_params(tensors, index)
    return he4_ffn(norm, residual, gate, up, down)


def attention_residual(tensors, index, state, context, positions, allowed, cfg):
    """The attention half of ``Layer.forward`` (``model.py:202-219``): ``state + o(attn)``."""
    p = f"blk.{index}."
    norm = rms(state, tensors[p + "attn_norm.weight"], cfg.epsilon)
    query = _linear(norm, tensors[p + "attn_q.weight"]).reshape(-1, cfg.heads, cfg.head_dim)
    key = _linear(norm, tensors[p + "attn_k.weight"]).reshape(-1, cfg.kv_heads, cfg.head_dim)
    value = _linear(norm, tensors[p + "attn_v.weight"]).reshape(-1, cfg.kv_heads, cfg.head_dim)
    query = rope(rms(query, tensors[p + "attn_q_norm.weight"], cfg.epsilon), positions, cfg.theta)
    key = rope(rms(key, tensors[p + "attn_k_norm.weight"], cfg.epsilon), positions, cfg.theta)
    key = np.concatenate((context[0], cache_storage(key)), 0)
    value = np.concatenate((context[1], cache_storage(value)), 0)
    slots = positions.shape[0]
    groups = cfg.heads // cfg.kv_heads
    query = query.reshape(slots, cfg.kv_heads, groups, cfg.head_dim)
    scores = np.einsum("qhgd,khd->hgqk", query, key).astype(np.float32) / F32(math.sqrt(cfg.head_dim))
    scores = np.where(allowed[None, None], scores, F32(-np.inf)).astype(np.float32)
    top = scores.max(-1, keepdims=True)
    weights = np.exp(scores - top).astype(np.float32)
    weights = (weights / weights.sum(-1, keepdims=True)).astype(np.float32)
    attended = np.einsum("hgqk,khd->qhgd", weights, value).astype(np.float32)
    return (state + _linear(attended.reshape(slots, -1), tensors[p + "attn_output.weight"])).astype(np.float32)


def encode_context(tensors, features, anchor, cfg):
    """Fused, normalised context rows ``rms(fc(features[:anchor]))`` (``model.py:382-386``)."""
    return rms(_linear(np.asarray(features[:anchor], dtype=np.float32), tensors["fc.weight"]),
               tensors["enc.output_norm.weight"], cfg.epsilon)


def he4_hidden(tensors, vocabulary, mask, features, tokens, anchor, cfg, slots=None, contexts=None):
    """Final normalised hidden state ``[k, hidden]`` of ``HE4.forward``."""
    size = cfg.slots if slots is None else slots
    positions = np.arange(anchor, anchor + size)
    context_positions = np.arange(anchor)
    identifiers = np.array((tokens[anchor],) + (mask,) * (size - 1))
    state = np.asarray(vocabulary, dtype=np.float32)[identifiers]
    encoded = None if contexts is not None else encode_context(tensors, features, anchor, cfg)
    keys = np.concatenate((context_positions, positions))
    for index in range(cfg.layers):
        allowed = np.ones((size, anchor + size), dtype=bool)
        if index < cfg.layers - 1:
            allowed &= np.abs(positions[:, None] - keys[None, :]) < cfg.window
        context = contexts[index] if contexts is not None else layer_context(tensors, index, encoded, context_positions, cfg)
        state = layer_forward(tensors, index, state, context, positions, allowed, cfg)
    return rms(state, tensors["output_norm.weight"], cfg.epsilon)


def he4_forward(tensors, vocabulary, mask, features, tokens, anchor, cfg, slots=None, contexts=None):
    """Logits ``[k, V]`` of ``HE4.forward`` (``model.py:369-396``)."""
    hidden = he4_hidden(tensors, vocabulary, mask, features, tokens, anchor, cfg, slots, contexts)
    return _linear(hidden, vocabulary)
