"""Pin the CPU oracle to the reference: every golden vector in tests/golden/qlinear_golden.npz was produced by the reference
qlinear itself (tests/golden/make_golden.py); the oracle must reproduce each bit for bit.  CPU only."""
import numpy as np
import pytest

from oracle import qlinear_oracle as orc
from conftest import golden_cases

ACT_DT = {np.dtype(np.uint16): "bf16", np.dtype(np.float16): "fp16", np.dtype(np.float32): "fp32"}
S_KIND = {np.dtype(np.uint8): "fp8", np.dtype(np.uint16): "bf16", np.dtype(np.float16): "fp16", np.dtype(np.float32): "fp32"}


def _case(g, name):
    p = name + "/"
    group, convrot = (int(v) for v in g[p + "meta"])
    return dict(x=g[p + "x"], q=g[p + "q"], s_rel=g[p + "s_rel"], s_ch=g[p + "s_ch"], cb=g[p + "cb"], group=group,
                convrot=convrot, bias=g.get(p + "bias"), out=g[p + "out"], codes=g[p + "codes"], xs=g[p + "xs"],
                grid=g[p + "grid"], acc=g[p + "acc"], rot=g[p + "rot"], act=g.get(p + "act"))


def test_golden_file_has_the_expected_cases(golden):
    names = golden_cases(golden)
    for want in ("cfg1s", "real16", "real16_f32", "real16_f16", "real16_outf32", "real16_eager", "swiglu", "intval",
                 "k128_g4", "k128_g16", "k128_g32", "k64", "real16_sf32", "real16_sbf16"):
        assert want in names


@pytest.mark.parametrize("size", [4, 16, 64, 256])
def test_hadamard(golden, size):
    h = orc.hadamard_regular(size)
    assert np.array_equal(h.astype(np.float32), golden[f"hadamard/{size}"])
    assert np.array_equal(h @ h, np.eye(size))


def test_fp8_table_matches_the_format():
    t = orc.fp8_e4m3fn_table()
    assert np.isnan(t[0x7F]) and np.isnan(t[0xFF]) and np.isnan(t).sum() == 2
    assert t[0x38] == 1.0 and t[0x7E] == 448.0 and t[0x01] == 2.0 ** -9 and t[0xB8] == -1.0


def test_decode_ties_and_symmetric_clamp(golden):
    grid = orc.decode_int8_grid(golden["ties/q"], golden["ties/s_rel"], "fp8", golden["ties/cb"], 16)
    assert np.array_equal(grid, golden["ties/grid"])
    assert grid[:, 0].tolist() == [2, 2, -2, 127, -127, 2, -2, 5, 0, 4]


def test_decode_every_fp8_scale_byte(golden):
    grid = orc.decode_int8_grid(golden["fp8all/q"], golden["fp8all/s_rel"], "fp8", golden["real_cb"], 16)
    assert np.array_equal(grid, golden["fp8all/grid"])


@pytest.mark.parametrize("name", ["cfg1s", "real16", "real16_f32", "real16_f16", "real16_outf32", "real16_eager", "swiglu",
                                  "intval", "k128_g4", "k128_g16", "k128_g32", "k64", "real16_sf32", "real16_sbf16"])
def test_oracle_reproduces_the_reference(golden, name):
    c = _case(golden, name)
    dt = ACT_DT[c["x"].dtype]
    s_kind = S_KIND[c["s_rel"].dtype]
    mode = "eager" if name.endswith("eager") else "ck"
    act = "swiglu" if name == "swiglu" else None
    out_dt = ACT_DT[c["out"].dtype]
    bias_dt = ACT_DT[c["bias"].dtype] if c["bias"] is not None else None
    xin = orc.swiglu(c["x"], dt) if act else c["x"]
    if act:
        assert np.array_equal(xin, c["act"])
    # rotation, quantiser, decode, exact GEMM, epilogue: each stage bit for bit
    assert np.array_equal(orc.rot32(orc.to_f32(xin, dt), c["convrot"]), c["rot"])
    codes, xs = orc.quantize_rows(xin, dt, c["convrot"], mode)
    assert np.array_equal(codes, c["codes"]) and np.array_equal(xs, c["xs"])
    grid = orc.decode_int8_grid(c["q"], c["s_rel"], s_kind, c["cb"], c["group"])
    assert np.array_equal(grid, c["grid"])
    acc = orc.int8_mm(codes, grid)
    assert np.array_equal(acc, c["acc"])
    out = orc.linear(c["x"], dt, c["q"], c["s_rel"], s_kind, c["s_ch"], c["cb"], c["group"], c["convrot"], bias=c["bias"],
                     bias_dt=bias_dt, out_dt=out_dt, input_act=act, mode=mode)
    assert out.dtype == c["out"].dtype and np.array_equal(out, c["out"])


@pytest.mark.parametrize("dt", ["bf16", "fp16", "fp32"])
def test_quantiser_degenerate_rows(golden, dt):
    codes, xs = orc.quantize_rows(golden[f"degen_{dt}/x"], dt)
    assert np.array_equal(codes, golden[f"degen_{dt}/codes"]) and np.array_equal(xs, golden[f"degen_{dt}/xs"])
    assert np.isfinite(xs).all() and (xs > 0).all()


def test_int8_mm_worst_case_magnitudes():
    """|a| <= 128, |w| <= 127 with odd products past 2^24 (tests/test_h3_qlinear.py:226-243): the chunked fp32 GEMM stays exact."""
    for k in (8, 1000, 1032, 4096):
        a = np.full((3, k), 127, np.int8)
        w = np.full((2, k), 127, np.int8)
        assert orc.int8_mm(a, w)[2, 1] == 16129 * k
        a = np.full((3, k), -128, np.int8)
        a[:, 1::2] = -127
        w = np.full((2, k), -127, np.int8)
        assert np.array_equal(orc.int8_mm(a, w), (a.astype(np.int64) @ w.astype(np.int64).T).astype(np.int32))


def test_check_weight_errors():
    q, s_rel, s_ch, cb = orc.synth_weight_int4_g128(8, 512, seed=1)
    orc.check_weight(q, s_rel, s_ch, cb, 128, 256)
    for args, msg in (((q, s_rel[:, :-1], s_ch, cb, 128, 256), "s_rel"), ((q, s_rel, s_ch[:-1], cb, 128, 256), "s_ch"),
                      ((q, s_rel, s_ch, cb[:8], 128, 256), "codebook"), ((q.astype(np.float32), s_rel, s_ch, cb, 128, 256), "int8"),
                      ((q, s_rel, s_ch, cb, 96, 256), "divisible")):
        with pytest.raises(ValueError, match=msg):
            orc.check_weight(*args)


def test_synthetic_weight_uses_the_clamp_edge_and_round_trips():
    """The benchmark's int4-g128 mapping: |codebook * s_rel| reaches ~127 (the reference clamp covers the edge) and the
    dequantised weight approximates the drawn N(0, 0.02) matrix."""
    q, s_rel, s_ch, cb = orc.synth_weight_int4_g128(64, 512, seed=3)
    grid = orc.decode_int8_grid(q, s_rel, "fp16", cb, 128)
    assert np.abs(grid).max() == 127
    w_rot = grid.astype(np.float32) * s_ch[:, None]
    w = (w_rot.astype(np.float64).reshape(64, 2, 256) @ orc.hadamard_regular(256)).reshape(64, 512)
    rng = np.random.default_rng(3)
    w0 = rng.standard_normal((64, 512), dtype=np.float32) * np.float32(0.02)
    assert np.linalg.norm(w - w0) / np.linalg.norm(w0) < 0.2
