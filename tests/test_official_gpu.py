"""Parity at the official H3 geometry and weight format, and at both ends of the config-2 sweep, against the CPU oracle.

The official H3 DiT (h3turbo/h3/config.py:12-31) has hidden 5376 = 21 x 256 (not a multiple of 512), 56 heads x 128
(inner 7168) and a SwiGLU FFN of 14336, so its four projections are qkv 5376 -> 21504, out 7168 -> 5376,
fc1 5376 -> 28672 and fc2 14336 -> 5376 (SwiGLU input of 28672 columns).  Real checkpoints store fp8-e4m3 group
scales with group 16 and a 16-level Lloyd-Max codebook (the reference's REAL_CB, read here from the golden vectors the
reference produced); the weights below are generated like the reference's own test fixture (random nibbles, group
scales 20..200 so the decode clamp is exercised, tests/test_h3_qlinear.py:46-53).

Each case runs the whole linear on the GPU at full size and checks a slice against the oracle: 32 rows spread over M
and 768 output channels spread over N (the qlinear is token-wise and every output column depends only on its own
weight row, so a slice is an exact sub-problem).  Counted and printed per case: int8 code mismatches, rows whose
scale differs, output mismatches and the max-rel error; the bars are the north star's (max-rel <= 1e-2, codes within
1 in 10^5, outputs within 1 in 10^3)."""
import numpy as np
import pytest
import torch

from oracle import qlinear_oracle as orc
from minimax_h3_turbo_b200.h3 import qlinear as ql
from minimax_h3_turbo_b200.h3.synth import synthetic_activation, synthetic_w4a8
from minimax_h3_turbo_b200.h3.types import W4A8Weight

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
MAXREL_TOL = 1e-2
ROWS, COLS = 32, 768

HID, INNER, FFN = 5376, 56 * 128, 14336
OFFICIAL = {"qkv": (HID, 3 * INNER, False), "out": (INNER, HID, False), "fc1": (HID, 2 * FFN, False),
            "fc2": (FFN, HID, True)}


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def real_weight(n, k, seed, codebook):
    """An fp8-e4m3 group-16 W4A8 layer with the real codebook, generated like the reference's make_weight."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8)
    s = (torch.rand(n, k // 16, generator=g) * 180 + 20).to(torch.float8_e4m3fn)
    s_ch = torch.rand(n, generator=g) * 0.02 + 0.005
    return W4A8Weight(q, s, s_ch, torch.from_numpy(codebook.astype(np.float32)), 16, 256)


def _slice_check(name, x, w, swiglu, s_kind, group):
    """Full-size linear on the GPU; ROWS x COLS slice against the oracle.  Returns the counts."""
    m, n = x.shape[0], w.q.shape[0]
    y = ql.linear(x, w, input_act="swiglu" if swiglu else None)
    rows = torch.linspace(0, m - 1, min(ROWS, m)).round().long()
    cols = torch.linspace(0, n - 1, min(COLS, n)).round().long()
    xs_rows = x[rows.to(DEV)]
    got = _bits(y[rows.to(DEV)][:, cols.to(DEV)])
    q, s_rel, s_ch = w.q.cpu().numpy(), w.s_rel.cpu(), w.s_ch.cpu().numpy()
    s_np = s_rel.view(torch.uint8).numpy() if s_kind == "fp8" else s_rel.numpy()
    cb = w.codebook.cpu().numpy()
    ci = cols.numpy()
    xn = _bits(xs_rows)
    want = orc.linear(xn, "bf16", q[ci], s_np[ci], s_kind, s_ch[ci], cb, group, input_act="swiglu" if swiglu else None)
    # the activation side alone: codes and scales of the slice's rows
    xq_in = orc.swiglu(xn, "bf16") if swiglu else xn
    codes_o, xsc_o = orc.quantize_rows(xq_in, "bf16")
    gq, gxs = ql._quantize_rows(xs_rows, 256, "ck", swiglu=swiglu)  # the kernel the linear runs (SwiGLU fused)
    code_mism = int((gq.cpu().numpy() != codes_o).sum())
    scale_rows = int((gxs.reshape(-1).cpu().numpy() != xsc_o).sum())
    gf, wf = orc.f32_from_bf16_bits(got).astype(np.float64), orc.f32_from_bf16_bits(want).astype(np.float64)
    maxrel = float(np.abs(gf - wf).max() / max(np.abs(wf).max(), 1e-30))
    out_mism = int((got != want).sum())
    print(f"{name}: M={m} K={w.q.shape[1] * 2} N={n}: code mismatches {code_mism}/{codes_o.size}, scale rows off "
          f"{scale_rows}/{codes_o.shape[0]}, output mismatches {out_mism}/{got.size}, max rel {maxrel:.2e}")
    assert np.isfinite(gf).all()
    assert maxrel <= MAXREL_TOL
    assert code_mism <= max(1, codes_o.size // 100000)
    assert out_mism <= max(2, got.size // 1000)
    # the decode of the slice's weight rows is bit-exact
    grid = ql.decode_int8_grid(W4A8Weight(w.q[cols.to(DEV)], w.s_rel[cols.to(DEV)], w.s_ch[cols.to(DEV)], w.codebook,
                                          w.group_size, w.convrot)).cpu().numpy()
    assert np.array_equal(grid, orc.decode_int8_grid(q[ci], s_np[ci], s_kind, cb, group))
    return code_mism, scale_rows, out_mism, maxrel


@pytest.mark.parametrize("m", [256, 4096])
@pytest.mark.parametrize("proj", list(OFFICIAL))
def test_official_projection_real_format(proj, m, golden):
    k, n, swiglu = OFFICIAL[proj]
    w = real_weight(n, k, seed=list(OFFICIAL).index(proj) + 11, codebook=golden["real16/cb"]).to(DEV)
    x = synthetic_activation(m, 2 * k if swiglu else k, seed=m + k, device=DEV)
    _slice_check(f"official {proj} fp8 g16", x, w, swiglu, "fp8", 16)


@pytest.mark.parametrize("proj", ["qkv", "out", "fc2"])
def test_official_projection_benchmark_format(proj):
    """The same official shapes with the benchmark's int4 group-128 fp16-scale weights."""
    k, n, swiglu = OFFICIAL[proj]
    w = synthetic_w4a8(n, k, seed=7, device=DEV)
    x = synthetic_activation(1024, 2 * k if swiglu else k, seed=k, device=DEV)
    _slice_check(f"official {proj} int4 g128", x, w, swiglu, "fp16", 128)


@pytest.mark.parametrize("m", [256, 65536])
@pytest.mark.parametrize("k,n", [(5120, 5120), (5120, 13824), (13824, 5120)])
def test_config2_sweep_ends_against_the_oracle(k, n, m):
    """The config-2 sweep at its smallest and largest M (the decode-in-GEMM kernel and the CTA-pair kernel)."""
    w = synthetic_w4a8(n, k, seed=k + n, device=DEV)
    x = synthetic_activation(m, k, seed=1000 + k + m, device=DEV)
    _slice_check("config2", x, w, False, "fp16", 128)
