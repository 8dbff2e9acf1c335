"""The fused RMSNorm + AdaLN modulation kernel against the reference's torch ops (model.py:64-66, 106-109), on GPU."""
import pytest
import torch

import torch_ops as tops
from minimax_h3_turbo_b200.h3 import block as blk

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _ref(x, w, eps, sh, sc, segs):
    return tops.scale_shift_(tops.rms(x, w, eps), sh, sc, segs)


def _inputs(m, hid, dt, mdt, seed, int_valued=False):
    g = torch.Generator(device=DEV).manual_seed(seed)
    if int_valued:  # every partial sum of squares exact in fp32, whatever the order
        x = torch.randint(-8, 9, (m, hid), generator=g, device=DEV).to(dt)
    else:
        x = (torch.randn(m, hid, generator=g, device=DEV) * 3).to(dt)
    w = (1 + 0.1 * torch.randn(hid, generator=g, device=DEV)).to(dt)
    sh, sc = (torch.randn(3, hid, generator=g, device=DEV).to(mdt) for _ in range(2))
    return x, w, sh, sc


@pytest.mark.parametrize("m,hid,dt,mdt", [(1000, 5120, torch.bfloat16, torch.bfloat16), (257, 5120, torch.bfloat16, torch.float32),
                                          (64, 3072, torch.float16, torch.float16), (33, 8, torch.bfloat16, torch.bfloat16)])
def test_matches_torch_up_to_the_row_sum_order(m, hid, dt, mdt):
    x, w, sh, sc = _inputs(m, hid, dt, mdt, 0)
    segs = [(0, m // 2, 0), (m // 2, m - 3, 2)]  # the last 3 tokens: no modulation
    got = blk.rms_modulate(x, w, 1e-5, sh, sc, segs)
    want = _ref(x, w, 1e-5, sh, sc, segs)
    diff = (got.float() - want.float()).abs()
    assert (diff > 0).float().mean().item() < 1e-4
    assert diff.max().item() <= 0.02 * want.float().abs().max().item()


def test_bit_exact_when_the_row_sum_is_exact():
    x, w, sh, sc = _inputs(512, 4096, torch.bfloat16, torch.bfloat16, 1, int_valued=True)
    segs = [(0, 100, 1), (100, 400, 0), (450, 512, 2)]
    assert torch.equal(blk.rms_modulate(x, w, 1e-5, sh, sc, segs), _ref(x, w, 1e-5, sh, sc, segs))


def test_per_token_rows_equal_segment_rows():
    x, w, sh, sc = _inputs(300, 1024, torch.bfloat16, torch.bfloat16, 2)
    rows = torch.tensor([0, 2, 1] * 100, device=DEV)
    per_token = blk.rms_modulate(x, w, 1e-5, sh, sc, [(0, 300, rows)])
    segs = [(i, i + 1, int(rows[i])) for i in range(300)]  # > 16 segments: also takes the per-token map
    assert torch.equal(per_token, blk.rms_modulate(x, w, 1e-5, sh, sc, segs))
    few = blk.rms_modulate(x[:3], w, 1e-5, sh, sc, [(0, 1, 0), (1, 2, 2), (2, 3, 1)])  # the by-value table
    assert torch.equal(few, per_token[:3])


def test_rejects_bad_segments():
    x, w, sh, sc = _inputs(10, 64, torch.bfloat16, torch.bfloat16, 3)
    with pytest.raises(ValueError):
        blk.rms_modulate(x, w, 1e-5, sh, sc, [(0, 10, 3)])
    with pytest.raises(ValueError):
        blk.rms_modulate(x, w, 1e-5, sh, sc, [(0, 11, 0)])


def _gate_ref(x, gate, other, segs):
    for a, b, row in segs:
        if b > a:
            x[a:b].addcmul_(other[a:b], gate[row].to(x.dtype))
    return x


@pytest.mark.parametrize("dt,mdt", [(torch.bfloat16, torch.bfloat16), (torch.bfloat16, torch.float32), (torch.float16, torch.float16)])
def test_gate_residual_is_bit_identical_to_addcmul(dt, mdt):
    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn(777, 5120, generator=g, device=DEV).to(dt)
    other = torch.randn(777, 5120, generator=g, device=DEV).to(dt)
    gate = torch.randn(2, 5120, generator=g, device=DEV).to(mdt)
    segs = [(0, 700, 0), (700, 770, 1)]  # tokens 770.. untouched
    want = _gate_ref(x.clone(), gate, other, segs)
    got = blk.gate_(x.clone(), gate, other, segs)
    assert torch.equal(got, want)
    rows = torch.tensor([1, 0] * 350 + [0] * 77, device=DEV)
    assert torch.equal(blk.gate_(x.clone(), gate, other, [(0, 777, rows)]),
                       _gate_ref(x.clone(), gate, other, [(i, i + 1, int(rows[i])) for i in range(777)]))
