"""The CTA-pair GEMM (tcgen05.mma.cta_group::2, 256 x 256 tiles) against the 1-CTA kernel, bit for bit, on shapes that
take the pair path: int32 accumulators, every epilogue dtype, bias, both quantiser modes, ragged M, N and K."""
import os
import subprocess
import sys
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
HERE = Path(__file__).resolve().parent


def test_pair_kernel_equals_the_one_cta_kernel(tmp_path):
    sys.path.insert(0, str(HERE / "helpers"))
    import gemm_cases

    got = gemm_cases.run()
    ref_file = tmp_path / "one_cta.pt"
    env = dict(os.environ, H3B_GEMM_PAIR="0")
    subprocess.run([sys.executable, str(HERE / "helpers" / "gemm_cases.py"), str(ref_file)], check=True, env=env,
                   timeout=600)
    want = torch.load(ref_file)
    for case, g, w in zip(gemm_cases.CASES, got, want):
        assert torch.equal(g.cpu(), w), case


def test_pair_kernel_int32_is_exact():
    from minimax_h3_turbo_b200.h3 import qlinear as ql

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(7)
    a = torch.randint(-128, 128, (2304, 1040), generator=g, device=dev, dtype=torch.int8)
    b = torch.randint(-127, 128, (4864, 1040), generator=g, device=dev, dtype=torch.int8)
    a[:3] = -128
    b[:5] = -127
    want = (a.double() @ b.double().t()).to(torch.int64)  # exact: |sums| < 2^53
    assert torch.equal(ql._int8_mm(a, b).to(torch.int64), want)
