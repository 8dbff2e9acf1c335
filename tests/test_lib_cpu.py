"""CPU checks of the C ABI and the Python host layer: the library loads, exports every symbol include/h3b.h declares, and
rejects bad arguments before touching a device.  No compute runs here (no GPU)."""
import ctypes
import re

import pytest
import torch

from conftest import ROOT, has_cuda
from minimax_h3_turbo_b200 import _lib
from minimax_h3_turbo_b200.h3 import qlinear as ql
from minimax_h3_turbo_b200.h3.types import W4A8Weight


def header_functions():
    text = (ROOT / "include" / "h3b.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(h3b_\w+)\s*\(", text, re.M)))


def test_header_declares_what_the_binding_binds():
    assert sorted(_lib.exported_symbols()) == header_functions()


def test_library_loads_and_exports_every_declared_symbol():
    L = _lib.lib()
    for name in header_functions():
        assert hasattr(L, name), name
    assert L.h3b_version() == _lib.ABI_VERSION


def test_workspace_sizes_are_host_arithmetic():
    L = _lib.lib()
    m, n, k = 1000, 1536, 1536
    r256 = lambda v: (v + 255) // 256 * 256  # noqa: E731
    assert L.h3b_gemm_workspace_bytes(m, n, k) == r256(n * k)
    assert L.h3b_linear_workspace_bytes(m, n, k) == r256(m * k) + r256(m * 4) + r256(n * k)


def _err(rc):
    return rc, _lib.lib().h3b_last_error().decode()


def test_rotq_argument_errors_need_no_device():
    L = _lib.lib()
    buf = ctypes.create_string_buffer(4096)
    p = ctypes.addressof(buf) + (-ctypes.addressof(buf)) % 256
    rc, msg = _err(L.h3b_rotq(p, 7, 4, 256, 256, 256, 0, 0, p, 256, p, None))
    assert rc == _lib.ERR_ARG and "dtype" in msg
    rc, msg = _err(L.h3b_rotq(p, _lib.BF16, 4, 250, 256, 256, 0, 0, p, 256, p, None))
    assert rc == _lib.ERR_ARG and "multiple of the rotation block" in msg
    rc, msg = _err(L.h3b_rotq(p, _lib.BF16, 4, 256, 256, 12, 0, 0, p, 256, p, None))
    assert rc == _lib.ERR_ARG and "power of 4" in msg
    rc, msg = _err(L.h3b_rotq(p, _lib.BF16, 4, 1024, 1024, 1024, 0, 0, p, 1024, p, None))
    assert rc == _lib.ERR_UNSUPPORTED and "1024" in msg
    rc, msg = _err(L.h3b_rotq(p + 2, _lib.BF16, 4, 256, 256, 256, 0, 0, p, 256, p, None))
    assert rc == _lib.ERR_ARG and "aligned" in msg
    rc, msg = _err(L.h3b_rotq(p, _lib.BF16, 4, 256, 256, 256, 0, 5, p, 256, p, None))
    assert rc == _lib.ERR_ARG and "quant_mode" in msg
    rc, msg = _err(L.h3b_rotq(p, _lib.BF16, 4, 256, 256, 256, 1, 0, p, 256, p, None))  # swiglu needs rows of 2K
    assert rc == _lib.ERR_ARG and "ldx" in msg


def test_weight_argument_errors_need_no_device():
    L = _lib.lib()
    buf = ctypes.create_string_buffer(8192)
    p = ctypes.addressof(buf) + (-ctypes.addressof(buf)) % 256
    rc, msg = _err(L.h3b_decode_grid(p, 4, 100, 50, p, _lib.FP8_E4M3, 7, p, 16, p, 112, None))
    assert rc == _lib.ERR_ARG and "divisible" in msg
    rc, msg = _err(L.h3b_decode_grid(p, 4, 256, 128, p, _lib.FP8_E4M3, 16, p, 24, p, 256, None))
    assert rc == _lib.ERR_ARG and "group_size" in msg
    rc, msg = _err(L.h3b_decode_grid(p, 4, 256, 128, p, 9, 16, p, 16, p, 256, None))
    assert rc == _lib.ERR_ARG and "scale dtype" in msg
    rc, msg = _err(L.h3b_w4a8_gemm(p, 256, p, 4, p, 128, p, _lib.FP8_E4M3, 16, p, p, 16, None, p, _lib.BF16, 8, 8, 256, 0,
                                   p, 16, None))
    assert rc == _lib.ERR_ARG and "workspace" in msg
    rc, msg = _err(L.h3b_int8_gemm_s32(p, 256, 4, p, 256, 8, 250, p, 8, None))
    assert rc == _lib.ERR_ARG and "multiple of 16" in msg


def _w(n=8, k=512, group=16):
    g = torch.Generator().manual_seed(0)
    q = torch.randint(-128, 128, (n, k // 2), generator=g, dtype=torch.int8)
    s = (torch.rand(n, k // group, generator=g) * 180 + 20).to(torch.float8_e4m3fn)
    return W4A8Weight(q, s, torch.rand(n, generator=g) * 0.02 + 0.005, torch.linspace(-1, 1, 16), group_size=group)


def test_python_validation_matches_the_reference_messages():
    w = _w()
    x = torch.randn(3, 512)
    for kw, msg in (({"backend": "cuda"}, "backend"), ({"precision": "a4"}, "precision"), ({"quant_mode": "x"}, "quant_mode"),
                    ({"input_act": "gelu"}, "input_act"), ({"chunk_tokens": 0}, "chunk_tokens")):
        with pytest.raises(ValueError, match=msg):
            ql.linear(x, w, **kw)
    with pytest.raises(ValueError, match="floating"):
        ql.linear(torch.zeros(2, 512, dtype=torch.int8), w)
    with pytest.raises(ValueError, match="even"):
        ql.linear(torch.zeros(2, 5), w, input_act="swiglu")
    with pytest.raises(ValueError, match="power of 4"):
        ql.hadamard_regular(12)
    with pytest.raises(ValueError, match="multiple"):
        ql.quantize_activation(torch.zeros(2, 100))
    with pytest.raises(ValueError, match="floating"):
        ql.rotate(torch.zeros(3, 256, dtype=torch.int8))
    bad = [(W4A8Weight(w.q, w.s_rel[:, :-1], w.s_ch, w.codebook), "s_rel"), (W4A8Weight(w.q, w.s_rel, w.s_ch[:-1], w.codebook), "s_ch"),
           (W4A8Weight(w.q, w.s_rel, w.s_ch, w.codebook[:8]), "codebook"), (W4A8Weight(w.q.float(), w.s_rel, w.s_ch, w.codebook), "int8")]
    for weight, msg in bad:
        with pytest.raises(ValueError, match=msg):
            ql._check_weight(weight)


@pytest.mark.skipif(has_cuda(), reason="checks the CPU-tensor refusal")
def test_cpu_tensors_are_refused_not_emulated():
    w = _w()
    with pytest.raises(RuntimeError, match="CUDA"):
        ql.linear(torch.randn(3, 512), w)
    with pytest.raises(RuntimeError, match="CUDA"):
        ql.quantize_activation(torch.randn(3, 512))
    with pytest.raises(RuntimeError, match="CUDA"):
        ql.decode_int8_grid(w)
    info = ql.available_backends()
    assert set(info) == {"b200", "ck"} and info["b200"]["available"] is False and info["b200"]["reason"]


def test_hadamard_matrix():
    for size in (4, 16, 64, 256):
        h = ql.hadamard_regular(size)
        assert torch.equal(h, h.T) and torch.equal(h @ h, torch.eye(size))
        assert ql.hadamard_regular(size) is h
