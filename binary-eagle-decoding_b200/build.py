"""Build ``libbitdraft.so`` (sm_100a) in-tree with nvcc.

Every ``csrc/*.cu`` file is compiled to an object in ``_build/`` (in parallel,
only when it or a header changed) and linked into ``libbitdraft.so`` next to
this file, so the library travels with the source tree.  No JIT cache, no
torch extension machinery: the library exports a plain C ABI
(``include/bitdraft.h``).
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
OBJ = HERE / "_build"
LIBRARY = HERE / "libbitdraft.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the bitdraft CUDA library cannot be built")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _compile(source: Path, verbose: bool) -> Path:
    obj = OBJ / (source.stem + ".o")
    newest = max(p.stat().st_mtime for p in [source, *_headers()])
    if obj.exists() and obj.stat().st_mtime >= newest:
        return obj
    cmd = [nvcc(), *ARCH, *FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(source), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed for {source.name}:\n{result.stderr}")
    if verbose and result.stderr:
        print(result.stderr)
    return obj


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile and link the library; returns its path."""
    OBJ.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    if force:
        for obj in OBJ.glob("*.o"):
            obj.unlink()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(sources))) as pool:
        objects = list(pool.map(lambda s: _compile(s, verbose), sources))
    newest = max(o.stat().st_mtime for o in objects)
    if LIBRARY.exists() and LIBRARY.stat().st_mtime >= newest and not force:
        return LIBRARY
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objects), "-lcudart"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stderr}")
    tmp.replace(LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    import sys

    print(build(verbose="-v" in sys.argv, force="--force" in sys.argv))
