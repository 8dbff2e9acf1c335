"""The warp-per-row rotate+quantise kernel (bf16, ConvRot 256, M >= 4096, K <= 6144 a multiple of 256) against the
CTA-per-row-group kernel, bit for bit, and against the oracle: both quantiser modes, SwiGLU inputs, half-warp passes,
ragged M and degenerate rows (zeros, a value near the bf16 maximum, subnormals only, an infinity)."""
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def test_row_kernel_equals_the_cta_kernel(tmp_path):
    sys.path.insert(0, str(HERE / "helpers"))
    import rotq_cases

    got = rotq_cases.run()
    for tag, env_add in (("cta", {"H3B_ROTQ_ROW": "0"}),):
        ref_file = tmp_path / f"{tag}.pt"
        subprocess.run([sys.executable, str(HERE / "helpers" / "rotq_cases.py"), str(ref_file)], check=True,
                       env=dict(os.environ, **env_add), timeout=600)
        want = torch.load(ref_file)
        for case, (q, xs), (wq, wxs) in zip(rotq_cases.CASES, got, want):
            assert torch.equal(q.cpu(), wq), (tag, case)
            assert torch.equal(xs.cpu().view(torch.int32), wxs.view(torch.int32)), (tag, case)


def test_row_kernel_against_the_oracle():
    sys.path.insert(0, str(HERE / "helpers"))
    import rotq_cases
    from oracle import qlinear_oracle as orc
    from minimax_h3_turbo_b200.h3 import qlinear as ql

    for i in (0, 1, 3, 5, 7, 8, 9):  # the cases without SwiGLU (the oracle's exp comes from the host libm)
        m, k, mode, _ = rotq_cases.CASES[i]
        x = rotq_cases.case_input(i)
        q, xs = ql._quantize_rows(x, 256, mode)
        xn = x[4:].cpu().view(torch.int16).numpy().view(np.uint16)  # finite rows (the oracle warns on the others)
        codes_o, xs_o = orc.quantize_rows(xn, "bf16", mode=mode)
        qn, xsn = q[4:].cpu().numpy(), xs.reshape(-1)[4:].cpu().numpy()
        mism = int((qn != codes_o).sum())
        print(f"{rotq_cases.CASES[i]}: code mismatches {mism}/{qn.size}, scale rows off {int((xsn != xs_o).sum())}")
        assert mism <= max(1, qn.size // 100000)
        assert np.abs(xsn.astype(np.float64) / xs_o - 1).max() <= 2.0 ** -22


def test_these_shapes_take_the_row_kernel():
    sys.path.insert(0, str(HERE / "helpers"))
    import rotq_cases
    from minimax_h3_turbo_b200.h3 import qlinear as ql

    for i, (m, k, mode, sw) in enumerate(rotq_cases.CASES):
        x = rotq_cases.case_input(i)
        with torch.profiler.profile(activities=[torch.profiler.ProfilerActivity.CUDA]) as prof:
            ql._quantize_rows(x, 256, mode, swiglu=sw)
            torch.cuda.synchronize()
        names = [e.key for e in prof.key_averages()]
        assert any("rotq_row_kernel" in n for n in names), (rotq_cases.CASES[i], names)
