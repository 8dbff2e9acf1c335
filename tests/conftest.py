"""Shared test setup: the `gpu` marker, import paths, and the golden vectors.

The package directory is `minimax-h3-turbo_b200/` (not a valid Python identifier); it is registered under the import name
`minimax_h3_turbo_b200`, the same way bench.py and __graft_entry__.py load it.
"""
import importlib.util
import os
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
for _p in (ROOT, ROOT / "tests" / "helpers"):  # the repo root (oracle) and the test helpers (torch_ops, ...)
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))
os.environ.setdefault("OMP_NUM_THREADS", "4")


def load_package():
    name = "minimax_h3_turbo_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = ROOT / "minimax-h3-turbo_b200"
    spec = importlib.util.spec_from_file_location(name, pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


load_package()


def _ensure_built():
    """Build libh3b.so if it is missing, lacks a declared entry point, or (on a machine without a GPU, where the sources
    are edited) is older than a source.  nvcc cross-compiles for sm_100a without a GPU."""
    import ctypes

    spec = importlib.util.spec_from_file_location("h3b_build", ROOT / "minimax-h3-turbo_b200" / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    from minimax_h3_turbo_b200 import _lib

    stale = not mod.LIB.exists()
    if not stale:  # probe a copy: loading the real path would pin the old library in this process
        import shutil
        import tempfile

        with tempfile.TemporaryDirectory() as d:
            tmp = Path(d) / "probe.so"
            shutil.copyfile(mod.LIB, tmp)
            probe = ctypes.CDLL(str(tmp))
            stale = any(not hasattr(probe, name) for name in _lib.exported_symbols())
    if not stale and not has_cuda():
        stale = not mod.up_to_date()
    if stale:
        mod.build()



def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (a B200) and the built libh3b.so")


@pytest.fixture(scope="session")
def golden():
    with np.load(ROOT / "tests" / "golden" / "qlinear_golden.npz") as z:
        return {k: z[k] for k in z.files}


def golden_cases(g):
    """Names of the full linear cases in the golden file (those that carry an output)."""
    return sorted({k.split("/")[0] for k in g if k.endswith("/out")})


def has_cuda():
    try:
        import torch

        return torch.cuda.is_available()
    except Exception:
        return False


_ensure_built()
