"""RMSNorm + modulation fused into the rotate+quantise kernel (h3b_rotq_rms_modulate) against the two-kernel chain it
replaces -- h3b_rms_modulate, then h3b_rotq on the materialised h -- bit for bit: codes, scales, and the whole DiT
block's output."""
import pytest
import torch

from minimax_h3_turbo_b200.h3 import block as blk
from minimax_h3_turbo_b200.h3 import qlinear as ql
from minimax_h3_turbo_b200.h3.synth import synthetic_activation, synthetic_w4a8
from minimax_h3_turbo_b200.h3.types import BlockWeights

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")


def _inputs(m, k, mdt, seed, n_rows=3):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = (torch.randn(m, k, generator=g, device=DEV) * 3)
    x[:, ::61] *= 25.0  # outlier channels
    if m > 3:
        x[1] = 0.0  # a zero row: rs = rsqrt(eps)
        x[2] = x[2].sign() * 1e-30  # sums of squares that underflow
    x = x.to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(k, generator=g, device=DEV)).to(torch.bfloat16)
    sh, sc = (torch.randn(n_rows, k, generator=g, device=DEV).to(mdt) for _ in range(2))
    return x, w, sh, sc


def _check(pre, mode="ck"):
    q, xs = blk.prenorm_codes(pre, 256, mode)
    h = pre.materialize()
    wq, wxs = ql._quantize_rows(h, 256, mode)
    assert torch.equal(q, wq)
    assert torch.equal(xs.reshape(-1).view(torch.int32), wxs.reshape(-1).view(torch.int32))


@pytest.mark.parametrize("m,k,mdt,mode", [(4096, 5120, torch.float32, "ck"), (4133, 5120, torch.bfloat16, "eager"),
                                          (37, 5120, torch.float32, "ck"), (1, 1536, torch.bfloat16, "ck"),
                                          (1000, 512, torch.float16, "eager"), (300, 6144, torch.float32, "ck"),
                                          # the official H3 width 5376 = 21 x 256 and other widths that are not
                                          # multiples of 512
                                          (4096, 5376, torch.float32, "ck"), (777, 5376, torch.bfloat16, "eager"),
                                          (2000, 768, torch.bfloat16, "ck"), (129, 256, torch.float32, "ck")])
def test_fused_codes_equal_norm_then_quantise(m, k, mdt, mode):
    x, w, sh, sc = _inputs(m, k, mdt, seed=m + k)
    segs = [(0, m // 2, 0), (m // 2, max(m // 2, m - 3), 2)]  # the last tokens: no modulation
    _check(blk.Prenorm(x, w, 1e-5, sh, sc, segs), mode)


def test_fused_codes_with_per_token_rows_and_without_modulation():
    m, k = 2000, 5120
    x, w, sh, sc = _inputs(m, k, torch.float32, seed=5, n_rows=4)
    rows = torch.randint(0, 4, (m,), generator=torch.Generator().manual_seed(3)).to(DEV)
    _check(blk.Prenorm(x, w, 1e-6, sh, sc, [(0, m, rows)]))  # per-token rows (a device row map)
    _check(blk.Prenorm(x, w, 1e-6, sh, sc, []))  # no segment: every token keeps the plain norm
    x2 = torch.empty(m, k + 512, dtype=torch.bfloat16, device=DEV)[:, 256:256 + k]  # strided rows, 16-byte aligned
    x2.copy_(x)
    _check(blk.Prenorm(x2, w, 1e-6, sh, sc, [(0, 700, 1), (900, m, 3)]))


def test_shapes_outside_the_fused_kernel_fall_back():
    x, w, sh, sc = _inputs(64, 6400, torch.float32, seed=9)
    pre = blk.Prenorm(x, w, 1e-5, sh, sc, [(0, 64, 0)])
    assert blk.prenorm_codes(pre) is None  # K = 6400: wider than the fused kernel's row buffer allows
    wt = synthetic_w4a8(256, 6400, seed=1, device=DEV)
    assert torch.equal(blk.prenorm_linear(pre, wt), ql.linear(pre.materialize(), wt))


def test_block_with_the_fused_norm_equals_the_unfused_block():
    hid, heads, hd, ffn, s = 1024, 8, 128, 2048, 700
    g = torch.Generator(device=DEV).manual_seed(0)
    norm = lambda n: (1 + 0.1 * torch.randn(n, generator=g, device=DEV)).bfloat16()  # noqa: E731
    w = BlockWeights(qkv=synthetic_w4a8(3 * hid, hid, seed=1, device=DEV), out=synthetic_w4a8(hid, hid, seed=2, device=DEV),
                     fc1=synthetic_w4a8(2 * ffn, hid, seed=3, device=DEV), fc2=synthetic_w4a8(hid, ffn, seed=4, device=DEV),
                     norm1=norm(hid), norm2=norm(hid), q_norm=norm(hd), k_norm=norm(hd))
    mod = blk.Modulation(*(torch.randn(2, hid, generator=g, device=DEV) for _ in range(6)))
    x = synthetic_activation(s, hid, seed=0, device=DEV)
    pos = blk.video_audio_positions(10, 6, 10, s - 600, DEV)
    cos, sin = blk.rope_tables(pos, 1.0 / (10000 ** (torch.arange(16, device=DEV) / 16)), torch.bfloat16)
    seg = [(0, 600, 0), (600, s, 1)]
    fused = blk.DiTBlock(heads, hd)(x.clone(), w, mod, seg, cos, sin)
    plain = blk.DiTBlock(heads, hd, fuse_norm=False)(x.clone(), w, mod, seg, cos, sin)
    assert torch.equal(fused, plain)
