"""GGUF export from device state (needs a B200): the FFN payloads equal the
reference's own export of the same parameters byte for byte, and the written
file passes the readback checks."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN, package

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda:0")


def tiny_model():
    pkg = package()
    t = np.load(GOLDEN / "tiny_he4.npz")
    f = np.load(GOLDEN / "export_ffn.npz")
    tensors = {k[2:]: torch.from_numpy(t[k]) for k in t.files if k.startswith("t_")}
    cfg = pkg.Geometry(hidden=4, intermediate=8, heads=2, kv_heads=1, head_dim=2, window=4096)
    model = pkg.HE4(tensors, torch.from_numpy(t["vocabulary"]), 19, cfg).to(DEV)
    with torch.no_grad():
        for index, block in enumerate(model.blocks):
            for name in ("gate", "up", "down"):
                q = getattr(block, name)
                base = f"blk.{index}.ffn_{name}"
                q.latent_sign.copy_(torch.from_numpy(f[base + ".latent"]))
                q.scale.copy_(torch.from_numpy(f[base + ".scale_param"]))
                q.midpoint.copy_(torch.from_numpy(f[base + ".midpoint_param"]))
                q.log_gain.copy_(torch.from_numpy(f[base + ".log_gain_param"]))
                q.log_clip.copy_(torch.from_numpy(f[base + ".log_clip_param"]).reshape(q.log_clip.shape))
    return pkg, model, f


def test_ffn_export_matches_reference_payloads():
    pkg, model, f = tiny_model()
    tensors, keys = pkg.export.ffn_tensors(model)
    assert len(tensors) == 6 * 3 * 3 + 6 * 2
    for t in tensors:
        want = f[t.name]
        assert t.data.dtype == want.dtype and t.data.shape == want.shape, t.name
        assert t.data.tobytes() == want.tobytes(), t.name
    values = {k: v for k, v, _ in keys}
    for index in range(6):
        for name in ("gate", "up", "down"):
            base = f"blk.{index}.ffn_{name}"
            assert values[base + ".w1ax.bits"] == int(f[base + ".w1ax.bits"])
            assert values[base + ".w1ax.mode"] == 2
            assert np.float32(values[base + ".w1ax.clip"]) == f[base + ".w1ax.clip"]


def test_gguf_roundtrip_from_device(tmp_path):
    pkg, model, _ = tiny_model()
    path = tmp_path / "drafter_ffn.gguf"
    expected = pkg.export.write_ffn_gguf(path, model, "recipe")
    pkg.export.verify_gguf(path, expected, "recipe")
    pkg.export.verify_against_device(path, model)
    # after an update that flips a sign the file no longer matches the device state
    with torch.no_grad():
        latent = model.blocks[2].down.latent_sign
        latent[1, 3] = -latent[1, 3] if latent[1, 3] != 0 else -1.0
    with pytest.raises(ValueError, match="differs from the device state"):
        pkg.export.verify_against_device(path, model)


def test_full_size_packing_equals_host_packbits():
    pkg = package()
    g = torch.Generator().manual_seed(31)
    latent = torch.randn((2560, 9728), generator=g) * 0.02
    got = pkg.export.packed_signs(latent.to(DEV))
    want = np.packbits(np.pad(latent.numpy() >= 0, ((0, 0), (0, (-9728) % 32))), axis=-1,
                       bitorder="little").view(np.int32)
    assert np.array_equal(got, want)
