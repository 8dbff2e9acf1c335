"""The DiT block on the W4A8 kernels (GPU): against the same block in fp32 on the dequantized weights (the difference is
the int8 activation quantisation noise, ~1 %), exact query chunking, and the block fed by the streaming provider."""
import pytest
import torch

from minimax_h3_turbo_b200.h3 import block as blk
from minimax_h3_turbo_b200.h3 import qlinear as ql
from minimax_h3_turbo_b200.h3.synth import synthetic_activation, synthetic_w4a8
from minimax_h3_turbo_b200.h3.types import BlockWeights

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
HID, HEADS, HD, FFN, S = 512, 4, 128, 1024, 300


def make(seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, device=DEV)  # noqa: E731
    w = BlockWeights(qkv=synthetic_w4a8(3 * HID, HID, seed=seed + 1, device=DEV), out=synthetic_w4a8(HID, HID, seed=seed + 2, device=DEV),
                     fc1=synthetic_w4a8(2 * FFN, HID, seed=seed + 3, device=DEV), fc2=synthetic_w4a8(HID, FFN, seed=seed + 4, device=DEV),
                     norm1=(1 + 0.1 * r(HID)).bfloat16(), norm2=(1 + 0.1 * r(HID)).bfloat16(),
                     q_norm=(1 + 0.1 * r(HD)).bfloat16(), k_norm=(1 + 0.1 * r(HD)).bfloat16())
    mod = blk.Modulation(*(0.1 * r(2, HID) for _ in range(6)))
    x = synthetic_activation(S, HID, seed=seed, device=DEV)
    pos = blk.video_audio_positions(5, 6, 9, S - 270, DEV)
    cos, sin = blk.rope_tables(pos, 1.0 / (10000 ** (torch.arange(16, device=DEV) / 16)), torch.bfloat16)
    return x, w, mod, [(0, 270, 0), (270, S, 1)], cos, sin


def test_block_matches_the_dequantized_fp32_block():
    x, w, mod, seg, cos, sin = make()
    y = blk.DiTBlock(HEADS, HD)(x.clone(), w, mod, seg, cos, sin)
    dense = {k: ql.dequantize(getattr(w, k), torch.float32) for k in ("qkv", "out", "fc1", "fc2")}
    wd = BlockWeights(qkv=dense["qkv"], out=dense["out"], fc1=dense["fc1"], fc2=dense["fc2"], norm1=w.norm1.float(),
                      norm2=w.norm2.float(), q_norm=w.q_norm.float(), k_norm=w.k_norm.float())

    def lin(t, wt, input_act=None):
        if input_act == "swiglu":
            g, u = t.chunk(2, dim=-1)
            t = torch.nn.functional.silu(g) * u
        return t @ wt.t()

    ref = blk.DiTBlock(HEADS, HD, linear=lin)(x.float(), wd, mod, seg, cos.float(), sin.float())
    upd, ref_upd = (y.float() - x.float()), (ref - x.float())
    rel = (upd - ref_upd).norm() / ref_upd.norm()
    assert torch.isfinite(y.float()).all() and rel < 0.05, rel.item()


def test_chunked_attention_is_exact():
    x, w, mod, seg, cos, sin = make(1)
    a = blk.DiTBlock(HEADS, HD)(x.clone(), w, mod, seg, cos, sin)
    b = blk.DiTBlock(HEADS, HD, attn_chunk=64)(x.clone(), w, mod, seg, cos, sin)
    assert torch.equal(a, b)


def test_single_rank_shard_spec_is_a_no_op():
    x, w, mod, seg, cos, sin = make(2)
    a = blk.DiTBlock(HEADS, HD)(x.clone(), w, mod, seg, cos, sin)
    b = blk.DiTBlock(HEADS, HD)(x.clone(), w, mod, seg, cos, sin, blk.ShardSpec(0, S, S))
    assert torch.equal(a, b)


def test_blocks_on_streamed_weights_equal_resident(tmp_path):
    """A forward over a 6-block store with 1 resident block and a 2-slot ring gives the same bytes as all-resident."""
    from minimax_h3_turbo_b200.h3 import stream as sm
    from minimax_h3_turbo_b200.h3.config import H3Config
    from minimax_h3_turbo_b200.h3.store import H3TFile
    from minimax_h3_turbo_b200.h3.synth import synthetic_store_tensors
    from minimax_h3_turbo_b200.h3.writer import write_h3t

    cfg = H3Config(hidden=HID, layers=6, refiner_layers=0, heads=HEADS, head_dim=HD, ffn=FFN, text_dim=64, video_channels=4,
                   audio_channels=8, quant_group=16)
    path = tmp_path / "b.h3t"
    write_h3t(path, cfg, synthetic_store_tensors(cfg, group=16, scale_dtype="fp8", seed=3))
    x0, _, mod, seg, cos, sin = make(3)
    block = blk.DiTBlock(HEADS, HD)
    with H3TFile(path) as store:
        x = x0.clone()
        for i in range(store.n_blocks):
            w = store.block_weights_cpu(i)
            w = BlockWeights(**{k: getattr(w, k).to(DEV) for k in ("qkv", "out", "fc1", "fc2", "norm1", "norm2", "q_norm", "k_norm")})
            x = block(x, w, mod, seg, cos, sin)
        with sm.StreamingProvider(store, DEV, resident=1, ring=2, prefetch=2) as p:
            for _ in range(2):
                y = x0.clone()
                p.begin_forward()
                for i in range(store.n_blocks):
                    y = block(y, p.acquire(i), mod, seg, cos, sin)
                    p.release(i)
                p.end_forward()
                assert torch.equal(x, y)
