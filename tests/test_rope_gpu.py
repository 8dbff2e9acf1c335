"""The fused q/k RMSNorm + RoPE kernel against the reference's bit-exact torch form (layout.py:309-356), on GPU."""
import pytest
import torch

import torch_ops as tops
from minimax_h3_turbo_b200.h3 import rope

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _case(s, heads, d, half, dt, tdt, seed, scale=1.0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    qkv = (torch.randn(s, 3 * heads * d, generator=g, device=DEV) * scale).to(dt)
    q, k, _ = (t.view(s, heads, d) for t in qkv.split(heads * d, dim=-1))
    wq = (1 + 0.2 * torch.randn(d, generator=g, device=DEV)).to(dt)
    wk = (1 + 0.2 * torch.randn(d, generator=g, device=DEV)).to(dt)
    ang = torch.rand(s, half, generator=g, device=DEV) * 100
    return qkv, q, k, wq, wk, ang.cos().to(tdt), ang.sin().to(tdt)


@pytest.mark.parametrize("s,heads,d,half,dt,tdt", [
    (777, 40, 128, 48, torch.bfloat16, torch.bfloat16),   # the H3 shape (rope_inv_freq_len 16 x 3 axes)
    (300, 8, 128, 64, torch.bfloat16, torch.float32),
    (129, 6, 64, 16, torch.float16, torch.float16),
    (64, 3, 256, 0, torch.bfloat16, torch.bfloat16),       # norm only
    (50, 2, 32, 16, torch.bfloat16, torch.bfloat16),
])
def test_fused_equals_the_reference_torch_form(s, heads, d, half, dt, tdt):
    for seed, scale in ((0, 1.0), (1, 300.0), (2, 1e-3)):
        qkv, q, k, wq, wk, cos, sin = _case(s, heads, d, half, dt, tdt, seed, scale)
        ref = qkv.clone()
        rq, rk, _ = (t.view(s, heads, d) for t in ref.split(heads * d, dim=-1))
        tops.norm_rope_(rq, rk, wq, wk, 1e-5, cos, sin, impl="torch")
        rope.norm_rope_(q, k, wq, wk, 1e-5, cos, sin, impl="b200")
        assert torch.equal(qkv, ref), (seed, (qkv != ref).sum().item())


def test_one_of_q_k_and_zero_heads():
    qkv, q, k, wq, wk, cos, sin = _case(100, 4, 128, 48, torch.bfloat16, torch.bfloat16, 5)
    q[3].zero_()  # an all-zero token: rsqrt(eps) scaling of zeros stays zero
    ref = qkv.clone()
    rq, rk, _ = (t.view(100, 4, 128) for t in ref.split(512, dim=-1))
    tops.norm_rope_(rq, None, wq, None, 1e-5, cos, sin, impl="torch")
    rope.norm_rope_(q, None, wq, None, 1e-5, cos, sin, impl="b200")
    assert torch.equal(qkv, ref)
    rope.norm_rope_(rq[:0], rk[:0], wq, wk, 1e-5, cos[:0], sin[:0], impl="b200")  # empty sequence


def test_rejects_unsupported_shapes():
    qkv, q, k, wq, wk, cos, sin = _case(10, 2, 128, 48, torch.bfloat16, torch.bfloat16, 6)
    with pytest.raises(RuntimeError):
        rope.norm_rope_(q.float(), k.float(), wq, wk, 1e-5, cos, sin, impl="b200")
    with pytest.raises(ValueError):
        rope.norm_rope_(q, k, wq, wk, 1e-5, cos[:5], sin[:5], impl="b200")
    with pytest.raises(RuntimeError):
        rope.norm_rope_(q, k, wq, wk, 1e-5, cos, sin, impl="eager")  # ComfyUI's portable formula is not built
    with pytest.raises(RuntimeError):
        rope.norm_rope_(q.cpu(), k.cpu(), wq.cpu(), wk.cpu(), 1e-5, cos.cpu(), sin.cpu())  # no CPU path


def test_k_only_with_fp32_weights_and_a_strided_layout():
    qkv, q, k, wq, wk, cos, sin = _case(333, 8, 128, 48, torch.bfloat16, torch.float32, 7)
    ref = qkv.clone()
    rq, rk, _ = (t.view(333, 8, 128) for t in ref.split(1024, dim=-1))
    tops.norm_rope_(None, rk, None, wk.float(), 1e-6, cos, sin, impl="torch")
    rope.norm_rope_(None, k, None, wk.float(), 1e-6, cos, sin, impl="b200")
    assert torch.equal(qkv, ref)
