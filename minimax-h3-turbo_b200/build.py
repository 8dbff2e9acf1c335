"""Build libh3b.so in-tree for sm_100a (B200) with nvcc.

`python minimax-h3-turbo_b200/build.py [--force] [-v]` or `build()` from Python.  The library is one translation unit
(csrc/libh3b.cu includes every kernel) linked against the static CUDA runtime; it needs no -lcuda (the TMA descriptor
encoder is fetched through cudaGetDriverEntryPoint).  Rebuilds only when a source is newer than the library.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libh3b.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"),
                 shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set CUDA_HOME or NVCC")


def _sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "h3b.h"]


def up_to_date(lib: Path = LIB) -> bool:
    if not lib.exists():
        return False
    t = lib.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _sources())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc_path(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "--shared", "-Xcompiler", "-fPIC,-O3",
           "-I", str(ROOT / "include"), "-o", str(tmp), str(CSRC / "libh3b.cu")]
    if ptxas_info:
        cmd[1:1] = ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        tmp.unlink(missing_ok=True)
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr[-20000:]}")
    if verbose or ptxas_info:
        sys.stdout.write(res.stderr)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    out = build(force="--force" in sys.argv, verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    print(out)
