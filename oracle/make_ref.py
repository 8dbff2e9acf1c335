"""Stage the reference's own qlinear module under oracle/_ref/ -- TEST AND BASELINE INFRASTRUCTURE, NOT PRODUCT CODE.

The reference path (`h3turbo/h3/qlinear.py` + `h3turbo/h3/types.py` of Alexpoopy1/MiniMax-H3-Turbo) is pure Python on
torch, with no native code to compile.  This recipe copies those two files and the two package markers above them
UNCHANGED from the reference tree into `oracle/_ref/h3turbo/...`, so that `bench.py --impl reference` can time the
reference's own code -- its CPU qlinear and its portable CUDA path (`_TorchRunner`, torch._int_mm) -- on a machine that
has no copy of the reference tree.  `oracle/_ref/` is ignored by git (the reference's source is not part of this
repository's history); it travels with the working tree like a built library.

Usage:  python oracle/make_ref.py [/path/to/reference]        (default: the REF_ROOT environment variable)
`build()` of the repository's entry point runs it when the reference tree is present.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
FILES = ("h3turbo/__init__.py", "h3turbo/h3/__init__.py", "h3turbo/h3/qlinear.py", "h3turbo/h3/types.py")


def stage(ref_root: str) -> Path:
    root = Path(ref_root)
    missing = [f for f in FILES if not (root / f).is_file()]
    if missing:
        raise FileNotFoundError(f"reference tree {root} lacks {missing}")
    tmp = OUT.with_name("_ref.tmp")
    if tmp.exists():
        shutil.rmtree(tmp)
    lines = []
    for f in FILES:
        dst = tmp / f
        dst.parent.mkdir(parents=True, exist_ok=True)
        shutil.copyfile(root / f, dst)
        lines.append(f"{hashlib.sha256(dst.read_bytes()).hexdigest()}  {f}")
    (tmp / "SOURCES.sha256").write_text("\n".join(lines) + "\n")
    if OUT.exists():
        shutil.rmtree(OUT)
    tmp.rename(OUT)
    return OUT


def available() -> bool:
    return all((OUT / f).is_file() for f in FILES)


if __name__ == "__main__":
    ref = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REF_ROOT", "")
    if not ref:
        raise SystemExit("usage: python oracle/make_ref.py /path/to/reference")
    print(stage(ref))
