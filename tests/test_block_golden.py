"""The DiT block composition against the reference's own block (tests/golden/block_golden.npz), on CPU: our DiTBlock with
the oracle as its linear and the reference's torch operators (tests/helpers/torch_ops.py: F.rms_norm, modulation, the
exact "torch" form of q/k norm + RoPE, SDPA, gating) must match every intermediate and the output bit for bit -- the
block's composition (order of the steps, what each one reads) is the reference's."""
import numpy as np
import torch

import torch_ops as tops
from minimax_h3_turbo_b200.h3 import block as blk
from oracle import qlinear_oracle as orc

import block_golden_util as bg  # noqa: E402


def oracle_linear(x, w, input_act=None):
    bits = x.contiguous().view(torch.int16).numpy().view(np.uint16)
    y = orc.linear(bits, "bf16", w.q.numpy(), w.s_rel.numpy(), "fp16", w.s_ch.numpy(), w.codebook.numpy(), w.group_size,
                   w.convrot, input_act=input_act)
    return bg.bf16(y)


def test_block_equals_the_reference_block_on_cpu():
    w, mod, segs, (hid, heads, hd, ffn), (eps, qk_eps), t = bg.load()
    block = blk.DiTBlock(heads, hd, eps, qk_eps, linear=oracle_linear, ops=tops.TorchOps())
    h1 = tops.rms_modulate(t["x"], w.norm1, eps, mod.shift_a, mod.scale_a, segs)
    assert torch.equal(h1, t["h1"])
    qkv = oracle_linear(t["h1"], w.qkv)
    assert torch.equal(qkv, t["qkv"])
    y = block(t["x"].clone(), w, mod, segs, t["cos"], t["sin"])
    assert torch.equal(y, t["y"])
