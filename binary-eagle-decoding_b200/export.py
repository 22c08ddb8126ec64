"""GGUF export of the binary feed-forward layers, with readback verification.

Mirrors the FFN part of ``w1a1_eagle/numerical/export.py`` (``packed_signs``
79-86, the ``w1ax`` metadata of ``prepare`` 145-160 and the per-projection
tensors 174-193) and the payload check of
``w1a1_eagle/numerical/gguf_readback.py:116-160``.  The sign words are packed
on the GPU (``bd_pack_signs``, bit-identical to the reference's
``np.packbits(..., bitorder="little")`` words); scales, midpoints and gains are
the parameters as the reference writes them (``clamp_min(0)`` and ``exp`` of
the CPU copy, exactly the reference's own expressions, so the bytes agree).
The file is written with the ``gguf`` package the reference pins (0.19.0).

The orchestration around the reference's export (worker state, budget
accounting, artifact store, frozen Q4_0/Q4_K re-quantisation of the attention
and vocabulary tensors) is not part of this module.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch
from torch import Tensor

from . import ops

# File-format constants read by the runtime that loads the drafter
# (w1a1_eagle/numerical/export.py:145-157); kept identical so exported files
# stay loadable by it.
W1AX_VERSION = 2
W1AX_ACTIVATION_BITS = 8
W1AX_STRINGS = {
    "bit_order": "little",
    "sign_rule": "nonnegative_is_one",
    "scale_rule": "f32_learned_nonnegative",
    "arithmetic": "affine_same_quantized_stream_v1",
    "a1": "signed_pm_bound_threshold0_nonnegative_positive_zero_row_scale0",
    "execution": "packed_signs_int8_codes_dp4a",
}
W1AX_MODE = 2
GGUF_KIND_CODES = {"F32": 0, "Q4_0": 2, "Q4_K": 12, "I32": 26}


@dataclass(frozen=True)
class ExportTensor:
    name: str
    data: np.ndarray
    kind_name: str  # "F32" or "I32"


def f32(value: Tensor) -> np.ndarray:
    """A finite parameter as a contiguous F32 host array (export.py:72-76)."""
    if not bool(torch.isfinite(value).all()):
        raise ValueError("nonfinite export operand")
    return value.detach().float().cpu().contiguous().numpy()


def packed_signs(value: Tensor) -> np.ndarray:
    """GGUF sign words ``int32 [rows, ceil(cols / 32)]`` of a latent (export.py:79-86), packed on the GPU."""
    if value.dtype != torch.float32 or value.ndim != 2:
        raise ValueError("finite F32 sign matrix required")
    return ops.pack_signs(value.detach().contiguous()).cpu().numpy()


def projections(model):
    """(layer index, name, Projection) for every gate / up / down projection."""
    for index, block in enumerate(model.blocks):
        for name in ("gate", "up", "down"):
            yield index, name, getattr(block, name)


def ffn_tensors(model) -> tuple[list[ExportTensor], list[tuple[str, object, str]]]:
    """The FFN tensors and per-projection metadata ``prepare`` writes (export.py:174-193).

    Returns ``(tensors, keys)`` with ``keys`` as ``(key, value, type)`` triples,
    type one of ``"uint32"``, ``"float32"``.
    """
    tensors: list[ExportTensor] = []
    keys: list[tuple[str, object, str]] = []
    for index, name, projection in projections(model):
        base = f"blk.{index}.ffn_{name}"
        bound = projection.log_clip.detach().float().cpu().exp()
        if not bool(torch.isfinite(bound)) or float(bound) <= 0:
            raise ValueError("invalid export clipping bound")
        keys.append((base + ".w1ax.bits", int(projection.bits), "uint32"))
        keys.append((base + ".w1ax.mode", W1AX_MODE, "uint32"))
        keys.append((base + ".w1ax.clip", float(bound), "float32"))
        tensors.append(ExportTensor(base + ".w1a1_packed", packed_signs(projection.latent_sign), "I32"))
        tensors.append(ExportTensor(base + ".w1a1_scale", f32(projection.scale.clamp_min(0)), "F32"))
        tensors.append(ExportTensor(base + ".w1ax_midpoint", f32(projection.midpoint), "F32"))
        if name != "up":  # gate and up share one gain (model.py:184-187)
            tensors.append(ExportTensor(base + ".w1ax_gain", f32(projection.log_gain.detach().float().cpu().exp()),
                                        "F32"))
    if len({t.name for t in tensors}) != len(tensors):
        raise ValueError("duplicate export tensor")
    return tensors, keys


def w1ax_keys(model, config_hash: str) -> list[tuple[str, object, str]]:
    """The global ``dflash.w1ax.*`` / ``dflash.component.*`` keys (export.py:145-160)."""
    layers = model.geometry.layers
    keys: list[tuple[str, object, str]] = [
        ("dflash.w1ax.version", W1AX_VERSION, "uint32"),
        ("dflash.w1ax.activation_bits", W1AX_ACTIVATION_BITS, "uint32"),
        ("dflash.w1ax.profile", "ffn" + str(layers * 3), "string"),
    ]
    keys += [("dflash.w1ax." + k, v, "string") for k, v in W1AX_STRINGS.items()]
    keys += [("dflash.w1ax.config_hash", config_hash, "string"),
             ("dflash.w1ax.private_head", True, "bool"),
             ("dflash.component.tied", True, "bool"),
             ("dflash.w1ax.tensors", sorted(f"blk.{i}.ffn_{n}.weight" for i in range(layers)
                                            for n in ("gate", "up", "down")), "array")]
    return keys


def expected_payloads(tensors: list[ExportTensor]) -> dict[str, tuple[str, tuple[int, ...], int, str]]:
    """``name -> (kind, GGUF shape, bytes, sha256)`` as the reference records it (export.py:286-298)."""
    out = {}
    for t in tensors:
        out[t.name] = (t.kind_name, tuple(reversed(t.data.shape)), t.data.nbytes,
                       hashlib.sha256(t.data.tobytes()).hexdigest())
    return out


def write_gguf(path: str | Path, tensors: list[ExportTensor],
               keys: list[tuple[str, object, str]]) -> dict[str, tuple[str, tuple[int, ...], int, str]]:
    """Write ``keys`` and F32 / I32 ``tensors`` as a ``dflash`` GGUF; returns the expected payloads."""
    import gguf

    writer = gguf.GGUFWriter(str(path), "dflash")
    for key, value, kind in keys:
        if kind == "uint32":
            writer.add_uint32(key, value)
        elif kind == "float32":
            writer.add_float32(key, value)
        elif kind == "bool":
            writer.add_bool(key, value)
        elif kind == "string":
            writer.add_string(key, value)
        elif kind == "array":
            writer.add_array(key, value)
        else:
            raise ValueError(f"unsupported metadata type {kind}")
    kinds = gguf.GGMLQuantizationType
    for t in tensors:
        if t.kind_name not in ("F32", "I32"):
            raise ValueError("only F32 and I32 export tensors are written here")
        writer.add_tensor(t.name, t.data, raw_dtype=kinds.I32 if t.kind_name == "I32" else kinds.F32)
    writer.write_header_to_file()
    writer.write_kv_data_to_file()
    writer.write_tensors_to_file()
    writer.close()
    return expected_payloads(tensors)


def write_ffn_gguf(path: str | Path, model, config_hash: str,
                   extra: list[ExportTensor] = ()) -> dict[str, tuple[str, tuple[int, ...], int, str]]:
    """Write the model's FFN export (plus ``extra`` F32/I32 tensors); returns the expected payloads."""
    tensors, proj_keys = ffn_tensors(model)
    return write_gguf(path, tensors + list(extra), w1ax_keys(model, config_hash) + proj_keys)


def verify_gguf(path: str | Path, expected: dict[str, tuple[str, tuple[int, ...], int, str]], recipe: str) -> None:
    """Readback check of a written file (gguf_readback.py:116-160): recipe hash, tensor
    coverage, types, shapes, sizes, alignment, payload digests, no overlaps."""
    import gguf

    path = Path(path)
    reader = gguf.GGUFReader(str(path))
    field = reader.fields.get("dflash.w1ax.config_hash")
    recipe_read = field.contents() if field is not None else None
    if len(reader.tensors) != len(expected) or recipe_read != recipe:
        raise ValueError("GGUF recipe or tensor count differs")
    names = [t.name for t in reader.tensors]
    if len(set(names)) != len(names) or set(names) != set(expected):
        raise ValueError("GGUF tensor coverage differs")
    size = path.stat().st_size
    intervals = []
    for t in reader.tensors:
        kind_name, shape, nbytes, digest = expected[t.name]
        if tuple(int(v) for v in t.shape) != shape or int(t.tensor_type) != GGUF_KIND_CODES[kind_name]:
            raise ValueError("GGUF tensor type or geometry differs")
        start = int(t.data_offset)
        if start % reader.alignment or start + nbytes > size or int(t.n_bytes) != nbytes:
            raise ValueError("GGUF tensor offset exceeds bounds or alignment")
        payload = np.asarray(t.data).tobytes()
        if hashlib.sha256(payload).hexdigest() != digest:
            raise ValueError("GGUF tensor payload differs")
        intervals.append((start, start + nbytes))
    intervals.sort()
    if any(a[1] > b[0] for a, b in zip(intervals, intervals[1:])):
        raise ValueError("GGUF tensor payloads overlap")


def verify_against_device(path: str | Path, model) -> None:
    """Re-pack every projection's live latent on the GPU and compare it with the
    file's ``w1a1_packed`` words bit for bit (and the F32 parameters exactly)."""
    import gguf

    reader = gguf.GGUFReader(str(path))
    stored = {t.name: np.asarray(t.data) for t in reader.tensors}
    tensors, _ = ffn_tensors(model)
    for t in tensors:
        got = stored.get(t.name)
        if got is None or got.shape != t.data.shape or got.tobytes() != t.data.tobytes():
            raise ValueError(f"exported tensor {t.name} differs from the device state")
