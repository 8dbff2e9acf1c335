"""Runs the GEMM cases of tests/test_gemm_pair_gpu.py in this process and saves the outputs (torch.save) to argv[1].
The test starts it with H3B_GEMM_PAIR=0, so this process uses the 1-CTA kernel for every shape."""
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
import conftest  # noqa: E402,F401  (registers the package)
import torch  # noqa: E402

from minimax_h3_turbo_b200.h3 import qlinear as ql  # noqa: E402
from minimax_h3_turbo_b200.h3.synth import synthetic_w4a8  # noqa: E402

DEV = torch.device("cuda")
CASES = [  # (M, N, K, out dtype, bias, quant mode): all large enough for 256 x 256 pair tiles
    (4096, 5120, 1024, torch.int32, False, "ck"),
    (4000, 5000, 1040, torch.int32, False, "ck"),
    (8192, 5120, 5120, torch.bfloat16, True, "ck"),
    (3000, 13824, 5120, torch.float32, False, "eager"),
    (2311, 6144, 2048, torch.float16, True, "ck"),
]


def run():
    outs = []
    for i, (m, n, k, dt, bias, mode) in enumerate(CASES):
        g = torch.Generator(device=DEV).manual_seed(100 + i)
        qa = torch.randint(-128, 128, (m, k), generator=g, device=DEV, dtype=torch.int8)
        qa[0, :] = -128  # extremes: every product at its largest magnitude in one row
        xs = torch.rand(m, generator=g, device=DEV) * 0.05 + 1e-3
        w = synthetic_w4a8(n, k, group=16 if k % 256 else 128, convrot=16 if k % 256 else 256, seed=i, device=DEV)
        b = torch.randn(n, generator=g, device=DEV) if bias else None
        outs.append(ql._gemm_codes(qa, xs, w, b, out_dtype=dt, quant_mode=mode))
    return outs


if __name__ == "__main__":
    torch.save([o.cpu() for o in run()], sys.argv[1])
