"""Runs the quantiser cases of tests/test_rotq_row_gpu.py in this process and saves codes and scales (torch.save) to
argv[1].  The test starts it with H3B_ROTQ_ROW=0, so that process uses the CTA-per-row-group kernel for every shape."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
import conftest  # noqa: E402,F401  (registers the package)
import torch  # noqa: E402

from minimax_h3_turbo_b200.h3 import qlinear as ql  # noqa: E402

DEV = torch.device("cuda")
CASES = [  # (M, K, quant mode, SwiGLU input): bf16, ConvRot 256, M >= 4096, K <= 6144 a multiple of 256 (the row kernel)
    (4096, 5120, "ck", False),
    (4133, 3072, "eager", False),   # M not a multiple of the warps of a CTA
    (4096, 2560, "ck", True),       # the last pass of a row is half a warp
    (4500, 512, "ck", False),       # one half-warp pass per row
    (4096, 1536, "eager", True),
    (4096, 3840, "ck", False),      # K = 15 x 256, not a multiple of 512: the upper lane runs off the row end
    (4133, 1280, "eager", True),    # the same with a SwiGLU input
    (4096, 256, "ck", False),       # one ConvRot block: the upper lane has nothing at all
    (4096, 5376, "ck", False),      # the official width: six passes, the last one half a warp
    (4133, 6144, "eager", False),   # the longest row one warp holds
]


def case_input(i):
    m, k, _, sw = CASES[i]
    g = torch.Generator(device=DEV).manual_seed(500 + i)
    x = torch.randn(m, 2 * k if sw else k, generator=g, device=DEV)
    x[:, :: 97] *= 20.0  # outlier channels
    x[0] = 0.0  # degenerate rows: all zero, one huge value, subnormal values only, an infinity
    x[1, 3] = 3.0e38
    x[2] = x[2].sign() * 1e-39
    x[3, 5] = float("inf")
    x[4] = torch.round(x[4] * 4) / 4  # short significands: rotations land on quotient ties more often
    return x.to(torch.bfloat16)


def run():
    outs = []
    for i, (m, k, mode, sw) in enumerate(CASES):
        q, xs = ql._quantize_rows(case_input(i), 256, mode, swiglu=sw)
        outs.append((q, xs.reshape(-1)))
    return outs


if __name__ == "__main__":
    torch.save([(q.cpu(), xs.cpu()) for q, xs in run()], sys.argv[1])
