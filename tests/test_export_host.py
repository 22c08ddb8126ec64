"""GGUF export host logic (no GPU): the writer and the readback check against
the reference's own export payloads (tests/golden/export_ffn.npz)."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import GOLDEN, package
from oracle import core

export = package().export


class _Geom:
    layers = 6


class _Model:
    geometry = _Geom()


def fixture_tensors():
    f = np.load(GOLDEN / "export_ffn.npz")
    tensors, keys = [], []
    for index in range(6):
        for name in ("gate", "up", "down"):
            base = f"blk.{index}.ffn_{name}"
            keys += [(base + ".w1ax.bits", int(f[base + ".w1ax.bits"]), "uint32"),
                     (base + ".w1ax.mode", 2, "uint32"),
                     (base + ".w1ax.clip", float(f[base + ".w1ax.clip"]), "float32")]
            tensors.append(export.ExportTensor(base + ".w1a1_packed", f[base + ".w1a1_packed"], "I32"))
            tensors.append(export.ExportTensor(base + ".w1a1_scale", f[base + ".w1a1_scale"], "F32"))
            tensors.append(export.ExportTensor(base + ".w1ax_midpoint", f[base + ".w1ax_midpoint"], "F32"))
            if name != "up":
                tensors.append(export.ExportTensor(base + ".w1ax_gain", f[base + ".w1ax_gain"], "F32"))
    return f, tensors, keys


def test_oracle_packing_matches_reference_export():
    f, _, _ = fixture_tensors()
    for index in range(6):
        for name in ("gate", "up", "down"):
            base = f"blk.{index}.ffn_{name}"
            assert np.array_equal(core.packed_signs(f[base + ".latent"]), f[base + ".w1a1_packed"])
            assert np.array_equal(np.maximum(f[base + ".scale_param"], np.float32(0)), f[base + ".w1a1_scale"])


def test_gguf_write_and_readback(tmp_path):
    _, tensors, keys = fixture_tensors()
    path = tmp_path / "ffn.gguf"
    expected = export.write_gguf(path, tensors, export.w1ax_keys(_Model(), "recipe-1") + keys)
    export.verify_gguf(path, expected, "recipe-1")
    import gguf

    reader = gguf.GGUFReader(str(path))
    assert reader.fields["dflash.w1ax.profile"].contents() == "ffn18"
    assert reader.fields["dflash.w1ax.bit_order"].contents() == "little"
    assert reader.fields["blk.0.ffn_down.w1ax.bits"].contents() == 8
    with pytest.raises(ValueError, match="recipe"):
        export.verify_gguf(path, expected, "recipe-2")
    # one flipped payload byte is caught
    data = bytearray(path.read_bytes())
    t = next(t for t in reader.tensors if t.name == "blk.3.ffn_up.w1a1_packed")
    data[int(t.data_offset)] ^= 1
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(bytes(data))
    with pytest.raises(ValueError, match="payload"):
        export.verify_gguf(bad, expected, "recipe-1")
