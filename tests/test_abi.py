"""The C-ABI library loads and exports every declared symbol (no GPU needed)."""

from __future__ import annotations

import ctypes
import subprocess

import pytest

from conftest import ROOT, submodule


def test_library_exports_every_header_symbol():
    lib = submodule("_lib")
    names = lib.header_symbols()
    assert len(names) >= 15
    handle = lib.load()
    missing = [n for n in names if not hasattr(handle, n)]
    assert not missing, missing
    # every declared symbol has a Python signature and vice versa
    assert set(names) == set(lib.SIGNATURES), set(names) ^ set(lib.SIGNATURES)


def test_integration_table_names_every_entry_point():
    # each declared entry point has a row in the integration guide's table of
    # the reference interfaces they replace
    lib = submodule("_lib")
    text = (ROOT / "INTEGRATION.md").read_text()
    table = "\n".join(line for line in text.splitlines() if line.startswith("| `bd_"))
    missing = [n for n in lib.header_symbols() if f"`{n}`" not in table]
    assert not missing, missing


def test_library_is_sm100a_and_pure_c_abi():
    lib = submodule("_lib")
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib.LIBRARY)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert {n for n in exported if n.startswith("bd_")} == set(lib.header_symbols())


def test_host_only_entry_points():
    lib = submodule("_lib").load()
    assert lib.bd_abi_version() == 1
    assert lib.bd_status_string(0) == b"ok"
    assert lib.bd_t16_words(9728, 2560) == 608 * 10 * 128
    assert lib.bd_t16_words(1, 1) == 128
    assert lib.bd_codes_ld(2560) == 2560 and lib.bd_codes_ld(1) == 256
    assert lib.bd_ffn_workspace_bytes(16, 2560, 9728) > 0
    # host-side validation happens before any device work
    assert lib.bd_pack_signs(None, -1, 4, None, None, None) == 1
    assert lib.bd_quantize_codes(None, 1, 8, 8, None, None, 5, None, None, None, None) == 1
    # the serving submit rejects missing buffers before any CUDA call
    assert lib.bd_round_submit(None, None, None, 0, None, None, None, None, 0, None) == 1
    assert lib.bd_round_submit(8, None, None, 16, None, None, None, None, 0, None) == 1
    assert lib.bd_round_submit(8, None, None, 0, None, None, None, None, -1, None) == 1
    # the allocation-free greedy entry: nothing to do, missing pointers, and sizes beyond
    # its fixed scratch (256 requests, 33 positions) refused before any CUDA call; the
    # stand-in address is never dereferenced
    assert lib.bd_accept_greedy_noalloc(None, 0, 4, 100, None, None, 0, None, None, None, None, None) == 0
    assert lib.bd_accept_greedy_noalloc(None, 1, 4, 100, None, None, 0, None, None, None, None, None) == 1
    addr = 256
    assert lib.bd_accept_greedy_noalloc(addr, 257, 4, 100, addr, None, 0, addr, addr, None, None, None) == 6
    assert lib.bd_accept_greedy_noalloc(addr, 1, 33, 100, addr, None, 0, addr, addr, None, None, None) == 6
    # training entries: sizes outside what the kernels handle are refused on the host
    assert lib.bd_train_attention_forward(*([None] * 8), 0, 16, 8, 4, 128, 2048, 0.1, None, None, None, None) == 1
    assert lib.bd_train_attention_forward(*([None] * 8), 32, 17, 8, 4, 128, 2048, 0.1, None, None, None, None) == 1
    assert lib.bd_train_attention_backward(*([None] * 14), 32, 16, 8, 5, 128, 2048, 0.1, *([None] * 7)) == 1
    assert lib.bd_train_attention_pack(*([None] * 6), 0, 0, 0, None, 0, 0, 32, 16, 8, 4, 129, 2048,
                                       *([None] * 9), None) == 1
    assert lib.bd_train_attention_pack_grad(None, None, 32, 16, 8, 4, 0, None, None, None, None, None) == 1
    assert lib.bd_rms_forward(None, 0, 2560, None, 1e-6, None, None, None) == 0  # nothing to do
    assert lib.bd_rms_forward(None, -1, 2560, None, 1e-6, None, None, None) == 1
    assert lib.bd_head_post(addr, 3, 4, 1, 3, None, 1e-6, None, None, 0, addr, None, None, None) == 1  # odd head_dim
    assert lib.bd_rms_partials(17, 4) == 2 * 4 + 17 and lib.bd_head_post_partials(512, 32) > 0
    # split-K workspaces: a 480-row product over a 151936-long K is split, a 4096-row one is not
    assert lib.bd_gemm_split_workspace_bytes(480, 2560, 151936, 3) > 0
    assert lib.bd_gemm_split_workspace_bytes(4096, 2560, 2560, 2) == 0


def test_missing_library_fails_loudly(monkeypatch, tmp_path):
    lib = submodule("_lib")
    monkeypatch.setattr(lib, "_lib", None)
    monkeypatch.setattr(lib, "LIBRARY", tmp_path / "libbitdraft.so")
    with pytest.raises(RuntimeError, match="not built"):
        lib.load()
