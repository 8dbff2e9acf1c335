"""The allocation-free W4A8 GEMM entry point, h3b_w4a8_gemm_noalloc, called through the C ABI.

It exists for callers that cannot allocate device memory (a plugin host that gives them no device allocator, a C or FFI
caller without a CUDA memory pool, a latency-critical loop that must not call cudaMalloc because it can synchronise the
device): its scratch is a fixed 16 MiB device array inside the library instead of a caller-provided workspace.  These
tests check it against the allocating entry point (h3b_w4a8_gemm) on two different calls in a row -- the second call
reuses the array the first one left behind -- and that too-wide rows are refused.  This file is collected last.
"""
import numpy as np
import pytest
import torch

from minimax_h3_turbo_b200 import _lib
from minimax_h3_turbo_b200.h3 import qlinear as ql
from minimax_h3_turbo_b200.h3.synth import synthetic_activation, synthetic_w4a8

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
MAXREL_TOL = 1e-2  # the output tolerance the parity tests use


def _gemm(entry, qa, xs, w, bias, out_dtype, quant_mode="ck", with_sch=True):
    """One call of h3b_w4a8_gemm_noalloc ("noalloc") or of the allocating h3b_w4a8_gemm ("alloc", with a workspace
    from torch) on the same arguments.  out_dtype torch.int32 asks for the raw accumulator (xs, s_ch, bias unused:
    with_sch=False passes null pointers for them, as a C caller may)."""
    a = ql._WeightArgs(w)
    m = qa.shape[0]
    out = torch.empty(m, a.n, dtype=out_dtype, device=DEV)
    code = _lib.INT32 if out_dtype == torch.int32 else _lib.act_code(out_dtype)
    b = None if bias is None else bias.to(device=DEV, dtype=out_dtype).contiguous()
    xs_p = xs.data_ptr() if with_sch else None
    sch_p = a.s_ch.data_ptr() if with_sch else None
    args = (qa.data_ptr(), qa.stride(0), xs_p, m, a.q.data_ptr(), a.ldq, a.s.data_ptr(), a.s_dtype, a.lds, sch_p,
            a.cb.data_ptr(), a.group, _lib.ptr(b), out.data_ptr(), code, a.n, a.n, a.k, _lib.QMODE[quant_mode])
    L = _lib.lib()
    if entry == "noalloc":
        _lib.check(L.h3b_w4a8_gemm_noalloc(*args, _lib.stream_ptr(DEV)), "h3b_w4a8_gemm_noalloc")
    else:
        nbytes = L.h3b_gemm_workspace_bytes(m, a.n, a.k)
        ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=DEV)
        _lib.check(L.h3b_w4a8_gemm(*args, ws.data_ptr(), ws.numel(), _lib.stream_ptr(DEV)), "h3b_w4a8_gemm")
    return out


def _noalloc(qa, xs, w, bias, out_dtype):
    return _gemm("noalloc", qa, xs, w, bias, out_dtype)


def _case(m, k, n, seed, out_dtype, with_bias):
    w = synthetic_w4a8(n, k, seed=seed, device=DEV)
    qa, xs = ql.quantize_activation(synthetic_activation(m, k, seed=seed, device=DEV))
    bias = torch.randn(n, generator=torch.Generator().manual_seed(seed)).to(DEV) if with_bias else None
    return qa, xs.reshape(-1), w, bias, out_dtype


def _check(qa, xs, w, bias, out_dtype):
    got = _noalloc(qa, xs, w, bias, out_dtype)
    want = ql._gemm_codes(qa, xs, w, bias, out_dtype)  # the allocating entry point, h3b_w4a8_gemm
    torch.cuda.synchronize()
    g, r = got.float().cpu().numpy().astype(np.float64), want.float().cpu().numpy().astype(np.float64)
    maxrel = float(np.abs(g - r).max() / max(np.abs(r).max(), 1e-30))
    assert maxrel <= MAXREL_TOL
    assert torch.equal(got, want)  # the same kernels on the same data: identical, not merely within tolerance


def test_noalloc_matches_the_allocating_entry_point_on_two_calls_in_a_row():
    # call 1: K = 5120, N = 5120 -> two slabs of decoded rows (3264 + 1856), bf16 output with bias
    first = _case(300, 5120, 5120, seed=1, out_dtype=torch.bfloat16, with_bias=True)
    _check(*first)
    # call 2: a different layer (K = 13824: slabs of 1184 rows, N = 1500 -> two slabs), fp32 output, no bias; the array
    # still holds call 1's rows
    _check(*_case(129, 13824, 1500, seed=2, out_dtype=torch.float32, with_bias=False))
    # and call 1 again, after call 2 left its rows behind
    _check(*first)


@pytest.mark.parametrize("quant_mode", ["ck", "eager"])
def test_noalloc_matches_in_both_quant_modes(quant_mode):
    """The eager epilogue (acc * (xs * s_ch)) as well as ck, over three slabs of decoded rows (K = 13824: 1184 rows per
    slab, N = 3000), twice in a row."""
    qa, xs, w, bias, _ = _case(200, 13824, 3000, seed=3, out_dtype=torch.bfloat16, with_bias=True)
    for _ in range(2):
        got = _gemm("noalloc", qa, xs, w, bias, torch.bfloat16, quant_mode)
        want = _gemm("alloc", qa, xs, w, bias, torch.bfloat16, quant_mode)
        torch.cuda.synchronize()
        assert torch.equal(got, want)


def test_noalloc_int32_accumulator_over_several_slabs_without_scales():
    """int32 output (the raw accumulator; no xs, s_ch or bias given) over four slabs (K = 5120: 3264 rows per slab,
    N = 10000), compared with the allocating entry point, twice in a row."""
    qa, xs, w, _, _ = _case(130, 5120, 10000, seed=4, out_dtype=torch.int32, with_bias=False)
    for _ in range(2):
        got = _gemm("noalloc", qa, xs, w, None, torch.int32, with_sch=False)
        want = _gemm("alloc", qa, xs, w, None, torch.int32, with_sch=False)
        torch.cuda.synchronize()
        assert torch.equal(got, want)
        assert int(got.abs().max()) > 0


def test_noalloc_refuses_rows_wider_than_its_scratch():
    k = _lib.NOALLOC_SCRATCH_BYTES // 32 + 256  # 32 decoded rows of this K no longer fit
    q = torch.zeros(4, k // 2, dtype=torch.int8, device=DEV)
    s = torch.ones(4, k // 128, dtype=torch.float16, device=DEV)
    w = ql.W4A8Weight(q, s, torch.ones(4, device=DEV), torch.arange(16, dtype=torch.float32, device=DEV), 128, 256)
    qa = torch.zeros(2, k, dtype=torch.int8, device=DEV)
    xs = torch.ones(2, dtype=torch.float32, device=DEV)
    with pytest.raises(ValueError, match="allocation-free limit"):
        _noalloc(qa, xs, w, None, torch.bfloat16)
