"""The SwiGLU fused into the rotate+quantise kernel against the reference's own form on the GPU, `F.silu(gate) * up` in
the activation dtype (qlinear.py:376-379), for EVERY bf16 gate value (NaN, infinities and subnormals included) and
every fp16 gate value: the quantiser's codes and scales must be identical whether torch or the kernel applies it."""
import pytest
import torch
import torch.nn.functional as F

from minimax_h3_turbo_b200.h3 import qlinear as ql

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _every_value(dt, k):
    bits = torch.arange(-32768, 32768, dtype=torch.int32).to(torch.int16)
    g = bits.view(dt).to(DEV).reshape(-1, k)  # 65536 / k rows
    gen = torch.Generator(device=DEV).manual_seed(11)
    up = (torch.rand(g.shape, generator=gen, device=DEV) * 4 - 2).to(dt)
    return torch.cat([g, up], dim=1)


@pytest.mark.parametrize("dt,k", [(torch.bfloat16, 4096), (torch.bfloat16, 1024), (torch.float16, 4096)])
@pytest.mark.parametrize("mode", ["ck", "eager"])
def test_fused_swiglu_equals_torch_silu_times_up(dt, k, mode):
    x = _every_value(dt, k)
    gate, up = x[:, :k], x[:, k:]
    h = F.silu(gate) * up  # the reference's _swiglu
    q, xs = ql._quantize_rows(x, 256, mode, swiglu=True)
    wq, wxs = ql._quantize_rows(h, 256, mode)
    assert torch.equal(q, wq)
    assert torch.equal(xs.view(torch.int32), wxs.view(torch.int32))
