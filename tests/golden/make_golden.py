"""Generate the golden vectors that pin the oracle: run the REFERENCE qlinear (h3turbo/h3/qlinear.py, CPU, backend="torch")
on seeded inputs and store its inputs and outputs in tests/golden/qlinear_golden.npz.

This script needs the reference source tree (pass its path as argv[1]); it is run once on a machine that has it, and the
resulting .npz is committed.  Nothing at test time reads the reference.  The reference's own test fixture `make_weight`
and its real Lloyd-Max codebook (tests/test_h3_qlinear.py:10-13, :46-53) are imported from the reference's test file so the
real-format cases use exactly the reference's generator.

Usage:  python tests/golden/make_golden.py /path/to/reference
"""
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))  # repo root, for the oracle's synthetic generators


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def _store_act(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return _bf16_bits(t)
    return t.numpy()


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from h3turbo.h3 import qlinear as ql  # noqa: E402  (the reference)
    from h3turbo.h3.types import W4A8Weight  # noqa: E402

    spec = importlib.util.spec_from_file_location("ref_test_qlinear", Path(ref_root) / "tests" / "test_h3_qlinear.py")
    rt = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(rt)
    from oracle import qlinear_oracle as orc  # only for the synthetic int4-g128 inputs of the benchmark configs

    torch.set_num_threads(8)
    out = {"real_cb": np.array(rt.REAL_CB, dtype=np.float32)}

    def weight_arrays(prefix, w, s_kind):
        out[prefix + "q"] = w.q.numpy()
        if s_kind == "fp8":
            out[prefix + "s_rel"] = w.s_rel.view(torch.uint8).numpy()
        elif s_kind == "bf16":
            out[prefix + "s_rel"] = _bf16_bits(w.s_rel)
        else:
            out[prefix + "s_rel"] = w.s_rel.numpy()
        out[prefix + "s_ch"] = w.s_ch.numpy()
        out[prefix + "cb"] = w.codebook.numpy()
        out[prefix + "meta"] = np.array([w.group_size, w.convrot], dtype=np.int64)

    def case(name, x, w, s_kind, bias=None, out_dtype=None, input_act=None, mode="ck"):
        p = name + "/"
        weight_arrays(p, w, s_kind)
        out[p + "x"] = _store_act(x)
        if bias is not None:
            out[p + "bias"] = _store_act(bias)
        xin = ql._swiglu(x) if input_act == "swiglu" else x
        if input_act == "swiglu":
            out[p + "act"] = _store_act(xin)
        qc, xs = ql.quantize_activation(xin, size=w.convrot, quant_mode=mode)
        grid = ql.decode_int8_grid(w)
        acc = ql._int8_mm(qc, grid)
        y = ql.linear(x, w, bias, out_dtype=out_dtype, backend="torch", input_act=input_act, quant_mode=mode)
        out[p + "codes"] = qc.numpy()
        out[p + "xs"] = xs.reshape(-1).numpy()
        out[p + "grid"] = grid.numpy()
        out[p + "acc"] = acc.numpy()
        out[p + "out"] = _store_act(y)
        out[p + "rot"] = ql._rot32(xin.reshape(-1, xin.shape[-1]), w.convrot).numpy()  # fp32 rotation before any rounding

    # 1. the benchmark's synthetic format (int4 g128, integer codebook, fp16 group scales) at config-1 width, 64 rows
    q, s_rel, s_ch, cb = orc.synth_weight_int4_g128(192, 1536, seed=0)
    w1 = W4A8Weight(torch.from_numpy(q), torch.from_numpy(s_rel), torch.from_numpy(s_ch), torch.from_numpy(cb), group_size=128, convrot=256)
    x1 = torch.from_numpy(orc.f32_from_bf16_bits(orc.synth_activation(64, 1536, seed=0, n_outliers=8))).to(torch.bfloat16)
    b1 = (torch.randn(192, generator=torch.Generator().manual_seed(1)) * 0.1).to(torch.bfloat16)
    case("cfg1s", x1, w1, "fp16", bias=b1)

    # 2. the real checkpoint format (reference make_weight: REAL_CB, fp8 group-16 scales in 20..200), bf16 / fp32 / fp16
    wr = rt.make_weight(40, 512, seed=11)
    xr = torch.randn(33, 512, generator=torch.Generator().manual_seed(99)).to(torch.bfloat16)
    br = torch.randn(40, generator=torch.Generator().manual_seed(21))
    case("real16", xr, wr, "fp8", bias=br)
    case("real16_f32", torch.randn(21, 512, generator=torch.Generator().manual_seed(5)), wr, "fp8", bias=br)
    case("real16_f16", torch.randn(17, 512, generator=torch.Generator().manual_seed(6)).to(torch.float16), wr, "fp8")
    case("real16_outf32", xr, wr, "fp8", bias=br, out_dtype=torch.float32)
    case("real16_eager", torch.randn(19, 512, generator=torch.Generator().manual_seed(7)).to(torch.bfloat16), wr, "fp8", mode="eager")
    # 3. SwiGLU input (fc2): x is [gate | up]
    case("swiglu", torch.randn(9, 1024, generator=torch.Generator().manual_seed(18)).to(torch.bfloat16), wr, "fp8", input_act="swiglu")
    # 4. small integers: any correct rotation is exact (reference test's _int_valued, tests/test_h3_qlinear.py:311-313)
    xi = torch.randint(-9, 10, (33, 512), generator=torch.Generator().manual_seed(5)).float().to(torch.bfloat16)
    case("intval", xi, wr, "fp8")
    # 5. small rotation blocks and other group sizes (make_weight shrinks convrot to 64 for K=128)
    for g in (4, 16, 32):
        wg = rt.make_weight(24, 128, seed=3, group=g)
        case(f"k128_g{g}", torch.randn(7, 128, generator=torch.Generator().manual_seed(g)).to(torch.bfloat16), wg, "fp8")
    wk = rt.make_weight(16, 64, seed=4)  # K=64 -> convrot 64
    case("k64", torch.randn(5, 64, generator=torch.Generator().manual_seed(40)).to(torch.bfloat16), wk, "fp8")
    # 6. generic (non-fp8) group scales take the arithmetic decode path
    wf = W4A8Weight(wr.q, wr.s_rel.float(), wr.s_ch, wr.codebook, 16, wr.convrot)
    case("real16_sf32", xr[:11], wf, "fp32")
    wb = W4A8Weight(wr.q, wr.s_rel.float().to(torch.bfloat16), wr.s_ch, wr.codebook, 16, wr.convrot)
    case("real16_sbf16", xr[:11], wb, "bf16")

    # 7. degenerate rows for the quantiser (tests/test_h3_qlinear.py:291-300): zero, tiny, large, huge
    for dt, name in ((torch.bfloat16, "bf16"), (torch.float16, "fp16"), (torch.float32, "fp32")):
        x = torch.zeros(4, 256, dtype=dt)
        x[1, 3], x[2], x[3, 0] = 1e-3, 3.0, (6e4 if dt == torch.float16 else 1e30)
        qd, sd = ql.quantize_activation(x, quant_mode="ck")
        out[f"degen_{name}/x"] = _store_act(x)
        out[f"degen_{name}/codes"] = qd.numpy()
        out[f"degen_{name}/xs"] = sd.reshape(-1).numpy()

    # 8. decode ties and the symmetric clamp (tests/test_h3_qlinear.py:171-184)
    cbt = torch.tensor([0.5, -0.5, 1.0, -1.0, 0.25, -0.25, 0.75, -0.75, 0.0, 0.5, 0.5, 0.5, 0.5, 0.5, 0.5, 0.5])
    cases = [(0, 3.0), (0, 5.0), (1, 5.0), (2, 448.0), (3, 448.0), (4, 6.0), (5, 6.0), (6, 7.0), (8, 448.0), (0, 7.0)]
    codes = torch.tensor([c[0] for c in cases])
    byte = (codes | (codes << 4)).to(torch.int32)
    qt = ((byte + 128) % 256 - 128).to(torch.int8)[:, None].expand(-1, 8).contiguous()
    st = torch.tensor([[c[1]] for c in cases]).to(torch.float8_e4m3fn)
    wt = W4A8Weight(qt, st, torch.ones(len(cases)), cbt, group_size=16, convrot=16)
    out["ties/q"] = qt.numpy()
    out["ties/s_rel"] = st.view(torch.uint8).numpy()
    out["ties/cb"] = cbt.numpy()
    out["ties/grid"] = ql.decode_int8_grid(wt).numpy()

    # 9. every fp8 byte through the decode table (scale byte s, codebook entry): the whole 256 x 16 level table
    qall = torch.arange(256, dtype=torch.int32)
    qall = ((qall + 128) % 256 - 128).to(torch.int8)
    qfull = qall[None, :].expand(256, -1).contiguous()  # [256 rows (scale byte), 256 bytes]
    sfull = torch.arange(256, dtype=torch.uint8)[:, None].expand(-1, 32).contiguous().view(torch.float8_e4m3fn)
    wfull = W4A8Weight(qfull, sfull, torch.ones(256), torch.tensor(rt.REAL_CB), group_size=16, convrot=256)
    out["fp8all/q"] = qfull.numpy()
    out["fp8all/s_rel"] = sfull.view(torch.uint8).numpy()
    out["fp8all/grid"] = ql.decode_int8_grid(wfull).numpy()

    # 10. the Hadamard matrices
    for size in (4, 16, 64, 256):
        out[f"hadamard/{size}"] = ql.hadamard_regular(size, "cpu", torch.float32).numpy()

    np.savez_compressed(HERE / "qlinear_golden.npz", **out)
    total = sum(v.nbytes for v in out.values())
    print(f"wrote {len(out)} arrays, {total / 1e6:.2f} MB uncompressed -> {HERE / 'qlinear_golden.npz'}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <reference source root>")
    main(sys.argv[1])
