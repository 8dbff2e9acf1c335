"""Build libh3b.so in-tree for sm_100a (B200) with nvcc.

`python minimax-h3-turbo_b200/build.py [--force] [-v] [--ptxas]` or `build()` from Python.  Each translation unit
(csrc/*.cu: the C ABI and one unit per kernel family, see csrc/launch.h) compiles to an object under `_build/` in
parallel; the objects link into one shared library against the static CUDA runtime (no -lcuda: the TMA descriptor
encoder is fetched through cudaGetDriverEntryPoint; no relocatable device code: every unit is self-contained).
An object is rebuilt when its source or any header is newer than it; the library when any object is.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB = PKG / "libh3b.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc"),
                 shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: set CUDA_HOME or NVCC")


def units():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [ROOT / "include" / "h3b.h"]


def _obj(cu: Path) -> Path:
    return OBJ / (cu.stem + ".o")


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(p.stat().st_mtime > t for p in deps)


def up_to_date(lib: Path = LIB) -> bool:
    hdr = _headers()
    objs = [_obj(cu) for cu in units()]
    if any(_stale(_obj(cu), [cu, *hdr]) for cu in units()):
        return False
    return not _stale(lib, objs)


def _compile(cu: Path, force: bool, ptxas_info: bool, verbose: bool):
    out = _obj(cu)
    if not force and not _stale(out, [cu, *_headers()]):
        return cu, None, ""
    tmp = out.with_suffix(f".o.tmp{os.getpid()}")
    cmd = [nvcc_path(), *ARCH, *FLAGS, "-I", str(ROOT / "include"), "-c", "-o", str(tmp), str(cu)]
    if ptxas_info:
        cmd[1:1] = ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        tmp.unlink(missing_ok=True)
        return cu, f"nvcc failed on {cu.name} ({res.returncode}):\n{res.stderr[-20000:]}", res.stderr
    os.replace(tmp, out)
    return cu, None, res.stderr


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    OBJ.mkdir(exist_ok=True)
    cus = units()
    with ThreadPoolExecutor(max_workers=min(len(cus), os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda cu: _compile(cu, force, ptxas_info, verbose), cus))
    errs = [e for _, e, _ in results if e]
    if errs:
        raise RuntimeError("\n".join(errs))
    if verbose or ptxas_info:
        for cu, _, log in results:
            if log:
                sys.stdout.write(f"--- {cu.name}\n{log}")
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc_path(), *ARCH, "--shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, (_obj(cu) for cu in cus))]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        tmp.unlink(missing_ok=True)
        raise RuntimeError(f"link failed ({res.returncode}):\n{res.stderr[-20000:]}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    out = build(force="--force" in sys.argv, verbose="-v" in sys.argv, ptxas_info="--ptxas" in sys.argv)
    print(out)
