"""GPU parity of the sm_100a kernels against the reference (golden vectors) and the CPU oracle.

The bar (north star): the int4 -> int8 decode and the int32 accumulator are bit-exact; given the reference's own int8
codes and scales, the whole GEMM + epilogue is bit-exact; end to end the outputs agree within max-rel 1e-2 with every
int8 code mismatch counted.  (The only float step that differs is the rotation: fp32 FWHT on the GPU, correctly
rounded fp64 in the reference -- in practice identical codes, and scale mismatches in the last bit of a few rows.)
"""
import numpy as np
import pytest
import torch

from conftest import golden_cases
from oracle import qlinear_oracle as orc
from minimax_h3_turbo_b200 import _lib
from minimax_h3_turbo_b200.h3 import qlinear as ql
from minimax_h3_turbo_b200.h3.types import W4A8Weight

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
MAXREL_TOL = 1e-2  # north-star output tolerance

_NP2T = {np.dtype(np.uint16): torch.bfloat16, np.dtype(np.float16): torch.float16, np.dtype(np.float32): torch.float32}
_T2NAME = {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float32: "fp32"}


def t_act(a: np.ndarray) -> torch.Tensor:
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(DEV)
    return torch.from_numpy(a.copy()).to(DEV)


def n_act(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def f32(a: np.ndarray) -> np.ndarray:
    return orc.f32_from_bf16_bits(a) if a.dtype == np.uint16 else a.astype(np.float32)


def golden_weight(g, name) -> W4A8Weight:
    p = name + "/"
    group, convrot = (int(v) for v in g[p + "meta"])
    s = g[p + "s_rel"]
    if s.dtype == np.uint8:
        st = torch.from_numpy(s.copy()).view(torch.float8_e4m3fn)
    elif s.dtype == np.uint16:
        st = torch.from_numpy(s.view(np.int16).copy()).view(torch.bfloat16)
    else:
        st = torch.from_numpy(s.copy())
    return W4A8Weight(torch.from_numpy(g[p + "q"].copy()), st, torch.from_numpy(g[p + "s_ch"].copy()),
                      torch.from_numpy(g[p + "cb"].copy()), group, convrot).to(DEV)


def maxrel(got: np.ndarray, want: np.ndarray) -> float:
    got, want = f32(got).astype(np.float64), f32(want).astype(np.float64)
    return float(np.abs(got - want).max() / max(np.abs(want).max(), 1e-30))


LINEAR_CASES = ["cfg1s", "real16", "real16_f32", "real16_f16", "real16_outf32", "real16_eager", "swiglu", "intval",
                "k128_g4", "k128_g16", "k128_g32", "k64", "real16_sf32", "real16_sbf16"]


def _call_args(g, name):
    p = name + "/"
    x = t_act(g[p + "x"])
    bias = t_act(g[p + "bias"]) if p + "bias" in g else None
    out_dt = _NP2T[g[p + "out"].dtype]
    return x, bias, out_dt, ("eager" if name.endswith("eager") else "ck"), ("swiglu" if name == "swiglu" else None)


def test_golden_cases_are_covered(golden):
    assert sorted(LINEAR_CASES) == golden_cases(golden)


@pytest.mark.parametrize("name", LINEAR_CASES)
def test_decode_is_bit_exact(golden, name):
    w = golden_weight(golden, name)
    assert np.array_equal(ql.decode_int8_grid(w).cpu().numpy(), golden[name + "/grid"])


def test_decode_ties_and_every_fp8_byte(golden):
    w = W4A8Weight(torch.from_numpy(golden["ties/q"]), torch.from_numpy(golden["ties/s_rel"]).view(torch.float8_e4m3fn),
                   torch.ones(10), torch.from_numpy(golden["ties/cb"]), 16, 16).to(DEV)
    assert np.array_equal(ql.decode_int8_grid(w).cpu().numpy(), golden["ties/grid"])
    w = W4A8Weight(torch.from_numpy(golden["fp8all/q"]), torch.from_numpy(golden["fp8all/s_rel"]).view(torch.float8_e4m3fn),
                   torch.ones(256), torch.from_numpy(golden["real_cb"]), 16, 256).to(DEV)
    assert np.array_equal(ql.decode_int8_grid(w).cpu().numpy(), golden["fp8all/grid"])
    # raw fp8 bytes (uint8 view) are accepted as well
    w2 = W4A8Weight(w.q, w.s_rel.view(torch.uint8), w.s_ch, w.codebook, 16, 256)
    assert np.array_equal(ql.decode_int8_grid(w2).cpu().numpy(), golden["fp8all/grid"])


@pytest.mark.parametrize("name", LINEAR_CASES)
def test_int32_accumulator_is_bit_exact_given_the_reference_codes(golden, name):
    p = name + "/"
    codes = torch.from_numpy(golden[p + "codes"]).to(DEV)
    grid = torch.from_numpy(golden[p + "grid"]).to(DEV)
    assert np.array_equal(ql._int8_mm(codes, grid).cpu().numpy(), golden[p + "acc"])
    # the same accumulator through the W4A8 GEMM entry point (int4 weights decoded on the fly)
    acc = ql._gemm_codes(codes, torch.from_numpy(golden[p + "xs"]).to(DEV), golden_weight(golden, name), out_dtype=torch.int32)
    assert np.array_equal(acc.cpu().numpy(), golden[p + "acc"])


@pytest.mark.parametrize("name", LINEAR_CASES)
def test_gemm_and_epilogue_are_bit_exact_given_the_reference_codes(golden, name):
    p = name + "/"
    x, bias, out_dt, mode, _ = _call_args(golden, name)
    out = ql._gemm_codes(torch.from_numpy(golden[p + "codes"]).to(DEV), torch.from_numpy(golden[p + "xs"]).to(DEV),
                         golden_weight(golden, name), bias, out_dt, mode)
    assert np.array_equal(n_act(out), golden[p + "out"])


@pytest.mark.parametrize("name", LINEAR_CASES)
def test_quantiser_against_the_reference(golden, name):
    p = name + "/"
    x, _, _, mode, act = _call_args(golden, name)
    w = golden_weight(golden, name)
    if act:
        q, xs = ql._quantize_rows(x.reshape(-1, x.shape[-1]), w.convrot, mode, swiglu=True)
    else:
        q, xs = ql.quantize_activation(x, size=w.convrot, quant_mode=mode)
    qn, xsn = q.cpu().numpy(), xs.reshape(-1).cpu().numpy()
    code_mism = int((qn != golden[p + "codes"]).sum())
    rel = np.abs(xsn.astype(np.float64) / golden[p + "xs"] - 1)
    print(f"{name}: code mismatches {code_mism}/{qn.size}, scale rows off {int((rel > 0).sum())}/{xsn.size}, max rel {rel.max():.2e}")
    assert code_mism <= max(1, qn.size // 10000)
    assert rel.max() <= 2.0 ** -22  # at most a last-bit difference of the fp32 scale
    if name == "intval":  # small integers: every rotation is exact, so the codes and scales are identical
        assert code_mism == 0 and rel.max() == 0


@pytest.mark.parametrize("name", LINEAR_CASES)
def test_linear_against_the_reference(golden, name):
    """End to end: rows whose int8 codes and fp32 scale match the reference's are bit-identical (everything after the
    quantiser is exact); the few rows whose scale differs in the last bit stay within the output tolerance."""
    p = name + "/"
    x, bias, out_dt, mode, act = _call_args(golden, name)
    w = golden_weight(golden, name)
    y = ql.linear(x, w, bias, out_dtype=out_dt, quant_mode=mode, input_act=act)
    assert y.dtype == out_dt and tuple(y.shape) == golden[p + "out"].shape
    got, want = n_act(y), golden[p + "out"]
    q, xs = ql._quantize_rows(x.reshape(-1, x.shape[-1]), w.convrot, mode, swiglu=act == "swiglu")
    same = (q.cpu().numpy() == golden[p + "codes"]).all(1) & (xs.reshape(-1).cpu().numpy() == golden[p + "xs"])
    mism = int((got != want).sum())
    print(f"{name}: output mismatches {mism}/{got.size} (rows with a different scale or code: {int((~same).sum())}), "
          f"max rel {maxrel(got, want):.2e}")
    assert np.array_equal(got[same], want[same])
    assert maxrel(got, want) <= MAXREL_TOL
    assert (~same).sum() <= max(1, same.size // 4)
    if name == "intval":
        assert mism == 0


@pytest.mark.parametrize("dt", ["bf16", "fp16", "fp32"])
def test_quantiser_degenerate_rows(golden, dt):
    x = t_act(golden[f"degen_{dt}/x"])
    q, xs = ql.quantize_activation(x)
    assert np.array_equal(q.cpu().numpy(), golden[f"degen_{dt}/codes"])
    assert np.array_equal(xs.reshape(-1).cpu().numpy(), golden[f"degen_{dt}/xs"])


# ------------------------------------------------------------------------------------------------ integer GEMM
@pytest.mark.parametrize("m,n,k", [(1, 8, 16), (7, 40, 512), (129, 264, 1536), (300, 200, 4096), (256, 5120, 5120),
                                   (1000, 1536, 13824), (2, 13824, 256), (517, 96, 1040)])
def test_int8_gemm_exact_including_extreme_magnitudes(m, n, k):
    g = torch.Generator().manual_seed(m * 7 + n + k)
    a = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    a[: max(1, m // 3)] = -128  # worst-case magnitudes: |sum| up to K * 16256
    b[: max(1, n // 3)] = -127
    want = (a.numpy().astype(np.int64) @ b.numpy().astype(np.int64).T).astype(np.int32)
    got = ql._int8_mm(a.to(DEV), b.to(DEV)).cpu().numpy()
    assert np.array_equal(got, want)


# ------------------------------------------------------------------------------------------------ oracle at scale
def _synth(m, k, n, seed=0, outliers=None, dt="bf16"):
    q, s_rel, s_ch, cb = orc.synth_weight_int4_g128(n, k, seed=seed)
    x = orc.synth_activation(m, k, seed=seed, outlier_frac=0.005 if outliers is None else None, n_outliers=outliers, dt=dt)
    w = W4A8Weight(torch.from_numpy(q), torch.from_numpy(s_rel), torch.from_numpy(s_ch), torch.from_numpy(cb), 128, 256).to(DEV)
    return x, (q, s_rel, s_ch, cb), w


def test_config1_full_size_against_the_oracle():
    """Config 1 exactly (M=1024, K=N=1536, int4 g128 fp16 scales, 8 outlier channels x20, bf16 bias, seed 0)."""
    x, (q, s_rel, s_ch, cb), w = _synth(1024, 1536, 1536, seed=0, outliers=8)
    bias = orc.bf16_bits_from_f32(np.random.default_rng(1).standard_normal(1536).astype(np.float32) * np.float32(0.1))
    codes_o, xs_o = orc.quantize_rows(x, "bf16")
    want = orc.linear(x, "bf16", q, s_rel, "fp16", s_ch, cb, 128, bias=bias)
    xt = t_act(x)
    qg, xsg = ql.quantize_activation(xt)
    code_mism = int((qg.cpu().numpy() != codes_o).sum())
    xs_off = int((xsg.reshape(-1).cpu().numpy() != xs_o).sum())
    y = n_act(ql.linear(xt, w, t_act(bias)))
    mism = int((y != want).sum())
    print(f"config1: code mismatches {code_mism}/{codes_o.size}, scale rows off {xs_off}/1024, "
          f"output mismatches {mism}/{y.size}, max rel {maxrel(y, want):.2e}")
    assert code_mism <= codes_o.size // 100000
    assert maxrel(y, want) <= MAXREL_TOL and mism <= y.size // 1000
    # given the oracle's codes, the GEMM + epilogue is bit-exact
    exact = ql._gemm_codes(torch.from_numpy(codes_o).to(DEV), torch.from_numpy(xs_o).to(DEV), w, t_act(bias))
    assert np.array_equal(n_act(exact), want)


@pytest.mark.parametrize("k,n", [(5120, 5120), (5120, 13824), (13824, 5120)])
def test_config2_shapes_against_the_oracle_on_a_row_slice(k, n):
    """Config-2 projections at M=2048 on the GPU; the first 48 rows are checked against the oracle (the path is
    token-wise, so a row slice is an exact sub-problem)."""
    x, (q, s_rel, s_ch, cb), w = _synth(2048, k, n, seed=k + n)
    y = ql.linear(t_act(x), w)
    rows = 48
    want = orc.linear(x[:rows], "bf16", q, s_rel, "fp16", s_ch, cb, 128)
    got = n_act(y[:rows])
    mism = int((got != want).sum())
    print(f"K={k} N={n}: output mismatches {mism}/{got.size}, max rel {maxrel(got, want):.2e}")
    assert maxrel(got, want) <= MAXREL_TOL and mism <= got.size // 1000
    grid = ql.decode_int8_grid(w).cpu().numpy()
    assert np.array_equal(grid, orc.decode_int8_grid(q, s_rel, "fp16", cb, 128))


def test_token_wise_properties_at_full_size():
    """Size-independent checks at the benchmark size: chunking and row permutation never change a row's result."""
    x, _, w = _synth(16384, 5120, 5120, seed=3)
    xt = t_act(x)
    y = ql.linear(xt, w)
    assert torch.equal(ql.linear(xt, w, chunk_tokens=3000), y)
    perm = torch.randperm(xt.shape[0], generator=torch.Generator().manual_seed(0)).to(DEV)
    assert torch.equal(ql.linear(xt[perm], w), y[perm])
    assert torch.equal(ql.linear(xt[:1], w), y[:1])
    assert torch.isfinite(y.float()).all()


# ------------------------------------------------------------------------------------------------ edge cases
def test_shapes_dtypes_and_layouts(golden):
    w = golden_weight(golden, "real16")
    base = torch.randn(37, 512, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(DEV)
    full = ql.linear(base, w)
    for m in (1, 2, 3, 17, 36):
        assert torch.equal(ql.linear(base[:m], w), full[:m])
    assert ql.linear(base[:0], w).shape == (0, 40)
    assert ql.linear(torch.zeros(2, 0, 512, dtype=torch.bfloat16, device=DEV), w).shape == (2, 0, 40)
    y3 = ql.linear(base[:36].reshape(3, 12, 512), w)
    assert y3.shape == (3, 12, 40) and torch.equal(y3.reshape(36, 40), full[:36])
    nc = base.t().contiguous().t()  # non-contiguous view of the same values
    assert not nc.is_contiguous() and torch.equal(ql.linear(nc, w), full)
    y32 = ql.linear(base, w, out_dtype=torch.float32)
    assert y32.dtype == torch.float32 and torch.equal(y32.to(torch.bfloat16), full)
    b = torch.randn(40, generator=torch.Generator().manual_seed(21)).to(DEV)
    assert torch.equal(ql.linear(base, w, b), full + b.to(torch.bfloat16))  # bias after the output rounding
    with pytest.raises(ValueError, match="bias"):
        ql.linear(base, w, b[:-1])
    with pytest.raises(ValueError, match="do not match"):
        ql.linear(base[:, :256], w)


def test_odd_output_widths_and_ragged_tiles():
    for n, m in ((8, 5), (40, 129), (200, 300), (264, 1000)):
        x, (q, s_rel, s_ch, cb), w = _synth(m, 512, n, seed=n)
        want = orc.linear(x, "bf16", q, s_rel, "fp16", s_ch, cb, 128)
        got = n_act(ql.linear(t_act(x), w))
        assert maxrel(got, want) <= MAXREL_TOL and (got != want).sum() <= max(2, got.size // 1000), (n, m)


def test_rotate_and_dequantize(golden):
    x = torch.randn(64, 512, generator=torch.Generator().manual_seed(2)).to(DEV)
    y = ql.rotate(x)
    ref = orc.rot32(x.cpu().numpy())
    assert np.abs(y.cpu().numpy() - ref).max() <= 1e-5 * np.abs(ref).max()
    assert torch.allclose(ql.rotate(y), x, atol=1e-5)  # involution
    xb = x.to(torch.bfloat16)
    yb = n_act(ql.rotate(xb))
    refb = orc.bf16_bits_from_f32(orc.rot32(f32(n_act(xb))))
    assert (yb != refb).mean() < 1e-3
    w = golden_weight(golden, "real16")
    rot = ql.dequantize(w, torch.float32, rotated=True).cpu().numpy()
    want = golden["real16/grid"].astype(np.float32) * golden["real16/s_ch"][:, None]
    assert np.array_equal(rot, want)
    orig = ql.dequantize(w).cpu().numpy()
    ref = (want.astype(np.float64).reshape(40, 2, 256) @ orc.hadamard_regular(256)).reshape(40, 512)
    assert np.abs(orig - ref).max() < 2e-6 * np.abs(ref).max()
    assert torch.equal(ql.dequantize(w, rows=slice(5, 11)), ql.dequantize(w)[5:11])


def test_a16_precision(golden):
    w = golden_weight(golden, "real16")
    x = torch.randn(48, 512, generator=torch.Generator().manual_seed(13)).to(torch.bfloat16).to(DEV)
    y16 = ql.linear(x, w, precision="a16").float().cpu().numpy()
    ref = x.float().cpu().numpy().astype(np.float64) @ ql.dequantize(w, torch.float64).cpu().numpy().T
    y8 = ql.linear(x, w).float().cpu().numpy()
    r16 = np.linalg.norm(y16 - ref) / np.linalg.norm(ref)
    r8 = np.linalg.norm(y8 - ref) / np.linalg.norm(ref)
    assert r16 < 0.004 and r16 < 0.5 * r8


def test_backends_report_b200():
    info = ql.available_backends()
    assert info["b200"]["available"] and info["ck"]["available"]


def test_no_device_error_was_raised():
    assert _lib.lib().h3b_device_error(1) == 0


def test_a_bounded_wait_that_runs_out_reports_and_leaves_the_context_usable():
    """Failure detection without a fault: a wait on a barrier nothing arrives on gives up after 0.2 s, raises the device
    flag, and the next kernels run normally."""
    L = _lib.lib()
    assert L.h3b_device_error(1) == 0
    gave_up = torch.zeros(1, dtype=torch.int32, device=DEV)
    _lib.check(L.h3b_selftest_wait_timeout(0.2, gave_up.data_ptr(), _lib.stream_ptr(DEV)), "selftest")
    assert L.h3b_device_error(1) == 1  # synchronises; then clears the flag
    assert gave_up.item() == 1
    a = torch.randint(-128, 128, (256, 512), device=DEV, dtype=torch.int8)
    b = torch.randint(-127, 128, (384, 512), device=DEV, dtype=torch.int8)
    assert torch.equal(ql._int8_mm(a, b).long(), (a.double() @ b.double().t()).long())
    assert L.h3b_device_error(0) == 0
