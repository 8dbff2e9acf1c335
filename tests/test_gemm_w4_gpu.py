"""The GEMM that decodes the int4 weight in its producer warps (small M) against the separate decode pass followed by
the int8 GEMM, bit for bit: both scale formats it takes (fp16 group 128, fp8 e4m3 group 16), every output dtype, bias,
both quantiser modes, ragged M, N and K."""
import pytest
import torch

from minimax_h3_turbo_b200 import _lib
from minimax_h3_turbo_b200.h3 import qlinear as ql
from minimax_h3_turbo_b200.h3.synth import synthetic_w4a8
from minimax_h3_turbo_b200.h3.types import W4A8Weight

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _fp8_weight(n, k, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    q = torch.randint(-128, 128, (n, k // 2), generator=g, device=DEV, dtype=torch.int8)
    s_rel = (torch.rand(n, k // 16, generator=g, device=DEV) * 180 + 20).to(torch.float8_e4m3fn)
    s_ch = torch.rand(n, generator=g, device=DEV) * 1e-3 + 1e-4
    cb = torch.linspace(-1.0, 1.0, 16, device=DEV)
    return W4A8Weight(q, s_rel, s_ch, cb, 16, 16 if k % 256 else 256)


def _unfused(qa, xs, w, bias, out_dtype, mode):
    a = ql._WeightArgs(w)
    n, k = a.n, a.k
    grid = torch.empty(n, k, dtype=torch.int8, device=DEV)
    L = _lib.lib()
    _lib.check(L.h3b_decode_grid(a.q.data_ptr(), n, k, a.ldq, a.s.data_ptr(), a.s_dtype, a.lds, a.cb.data_ptr(), a.group,
                                 grid.data_ptr(), k, _lib.stream_ptr(DEV)), "decode")
    out = torch.empty(qa.shape[0], n, dtype=out_dtype, device=DEV)
    code = _lib.INT32 if out_dtype == torch.int32 else _lib.act_code(out_dtype)
    b = None if bias is None or out_dtype == torch.int32 else bias.to(out_dtype).contiguous()
    _lib.check(L.h3b_int8_gemm_epilogue(qa.data_ptr(), k, xs.data_ptr(), qa.shape[0], grid.data_ptr(), k,
                                        a.s_ch.data_ptr(), _lib.ptr(b), out.data_ptr(), code, n, n, k, _lib.QMODE[mode],
                                        _lib.stream_ptr(DEV)), "gemm")
    return out


@pytest.mark.parametrize("m,n,k,fmt,dt,bias,mode", [
    (256, 5120, 5120, "fp16", torch.bfloat16, False, "ck"),
    (256, 13824, 5120, "fp16", torch.bfloat16, True, "ck"),
    (200, 5000, 13824, "fp16", torch.float32, False, "eager"),
    (1024, 1536, 1536, "fp16", torch.bfloat16, True, "ck"),     # config 1
    (77, 3072, 1056, "fp8", torch.bfloat16, False, "ck"),       # K not a multiple of 128
    (300, 4096, 4096, "fp8", torch.float16, True, "eager"),
    (64, 1000, 2048, "fp8", torch.int32, False, "ck"),
])
def test_decode_in_producer_equals_separate_decode(m, n, k, fmt, dt, bias, mode):
    w = synthetic_w4a8(n, k, seed=n + k, device=DEV) if fmt == "fp16" else _fp8_weight(n, k, n + k)
    a = ql._WeightArgs(w)
    assert _lib.lib().h3b_w4a8_gemm_decodes_in_kernel(m, n, k, a.q.data_ptr(), a.ldq, a.s_dtype, a.group) == 1
    g = torch.Generator(device=DEV).manual_seed(m)
    qa = torch.randint(-128, 128, (m, k), generator=g, device=DEV, dtype=torch.int8)
    xs = torch.rand(m, generator=g, device=DEV) * 0.05 + 1e-3
    b = torch.randn(n, generator=g, device=DEV) if bias else None
    fused = ql._gemm_codes(qa, xs, w, b, out_dtype=dt, quant_mode=mode)
    assert torch.equal(fused, _unfused(qa, xs, w, b, dt, mode))


def test_large_m_keeps_the_separate_decode():
    w = synthetic_w4a8(5120, 5120, seed=1, device=DEV)
    a = ql._WeightArgs(w)
    assert _lib.lib().h3b_w4a8_gemm_decodes_in_kernel(16384, 5120, 5120, a.q.data_ptr(), a.ldq, a.s_dtype, a.group) == 0


def _w4a8_gemm(qa, xs, w, bias, out_dtype, mode):
    """h3b_w4a8_gemm with the workspace h3b_gemm_workspace_bytes asks for."""
    a = ql._WeightArgs(w)
    m, n, k = qa.shape[0], a.n, a.k
    L = _lib.lib()
    need = L.h3b_gemm_workspace_bytes(m, n, k)
    ws = torch.empty(max(need, 256), dtype=torch.uint8, device=DEV)
    out = torch.empty(m, n, dtype=out_dtype, device=DEV)
    code = _lib.INT32 if out_dtype == torch.int32 else _lib.act_code(out_dtype)
    b = None if bias is None or out_dtype == torch.int32 else bias.to(out_dtype).contiguous()
    _lib.check(L.h3b_w4a8_gemm(qa.data_ptr(), k, xs.data_ptr(), m, a.q.data_ptr(), a.ldq, a.s.data_ptr(), a.s_dtype, a.lds,
                               a.s_ch.data_ptr(), a.cb.data_ptr(), a.group, _lib.ptr(b), out.data_ptr(), code, n, n, k,
                               _lib.QMODE[mode], ws.data_ptr(), need, _lib.stream_ptr(DEV)), "w4a8 gemm")
    return out


@pytest.mark.parametrize("m,n,k,fmt,dt,bias,mode", [
    (256, 5120, 5120, "fp16", torch.bfloat16, False, "ck"),      # the config-2 M = 256 points
    (256, 13824, 5120, "fp16", torch.bfloat16, False, "ck"),
    (256, 5120, 13824, "fp16", torch.bfloat16, False, "ck"),
    (129, 5376, 5376, "fp8", torch.bfloat16, True, "ck"),        # two subtiles, the second almost empty; official width
    (128, 21504, 5376, "fp8", torch.float16, True, "eager"),     # one subtile; the official qkv projection
    (1, 7168, 1536, "fp16", torch.float32, True, "ck"),          # one token
    (40, 1000, 2048, "fp8", torch.int32, False, "ck"),           # ragged N (not a multiple of the tile), int32 out
    (250, 264, 13824, "fp16", torch.bfloat16, True, "eager"),    # few N tiles: many K splits
    (96, 40, 4096, "fp8", torch.float32, False, "ck"),           # N below one tile
])
def test_small_m_split_k_equals_separate_decode(m, n, k, fmt, dt, bias, mode):
    """The small-M kernel (all M rows per CTA, K split across the CTAs of a cluster, partial sums added up in the
    cluster's shared memory) against decode + GEMM, bit for bit.  The planner picks one split for some of these shapes
    (the epilogue then runs straight from the accumulator) and several for the others."""
    w = synthetic_w4a8(n, k, seed=n + k, device=DEV) if fmt == "fp16" else _fp8_weight(n, k, n + k)
    a = ql._WeightArgs(w)
    assert _lib.lib().h3b_w4a8_gemm_decodes_in_kernel(m, n, k, a.q.data_ptr(), a.ldq, a.s_dtype, a.group) == 1
    g = torch.Generator(device=DEV).manual_seed(m + n)
    qa = torch.randint(-128, 128, (m, k), generator=g, device=DEV, dtype=torch.int8)
    xs = torch.rand(m, generator=g, device=DEV) * 0.05 + 1e-3
    b = torch.randn(n, generator=g, device=DEV) if bias else None
    want = _unfused(qa, xs, w, b, dt, mode)
    got = _w4a8_gemm(qa, xs, w, b, dt, mode)
    torch.cuda.synchronize()
    assert torch.equal(got, want)
    assert _lib.lib().h3b_device_error(0) == 0


def test_small_m_worst_case_accumulators_are_exact():
    """|acc| up to K x 128 x 127 over 13824 columns split across CTAs: the int32 partial sums add up exactly."""
    m, n, k = 200, 512, 13824
    q = torch.full((n, k // 2), 0x00, dtype=torch.int8, device=DEV)  # nibble 0 everywhere: codebook level cb[0] * s
    s_rel = torch.full((n, k // 128), 127.0, dtype=torch.float16, device=DEV)
    cb = torch.full((16,), -1.0, device=DEV)
    w = W4A8Weight(q, s_rel, torch.ones(n, device=DEV), cb, 128, 256)  # every level -127
    qa = torch.full((m, k), -128, dtype=torch.int8, device=DEV)
    xs = torch.ones(m, device=DEV)
    got = _w4a8_gemm(qa, xs, w, None, torch.int32, "ck")
    assert int(got.min()) == int(got.max()) == k * 128 * 127


@pytest.mark.parametrize("plan", ["128,8,1", "128,2,2", "128,3,2", "128,5,2", "128,7,1", "128,1,2", "128,1,1", "128,4,2"])
def test_small_m_every_tile_plan_is_exact(plan, monkeypatch):
    """Forced tile plans (N tile, K splits = cluster size, M subtiles per CTA) on a ragged problem: two M subtiles, the
    second almost empty, N not a multiple of the tile, K splits of unequal length -- bit for bit against decode + GEMM."""
    m, n, k = 131, 1000, 3584
    w = synthetic_w4a8(n, k, seed=7, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(11)
    qa = torch.randint(-128, 128, (m, k), generator=g, device=DEV, dtype=torch.int8)
    xs = torch.rand(m, generator=g, device=DEV) * 0.05 + 1e-3
    b = torch.randn(n, generator=g, device=DEV)
    want = _unfused(qa, xs, w, b, torch.bfloat16, "ck")
    monkeypatch.setenv("H3B_W4S_PLAN", plan)
    got = _w4a8_gemm(qa, xs, w, b, torch.bfloat16, "ck")
    torch.cuda.synchronize()
    assert torch.equal(got, want), plan
    assert _lib.lib().h3b_device_error(0) == 0
