"""The DiT block on the W4A8 kernels (GPU): against the same block in fp32 on the dequantized weights (the difference is
the int8 activation quantisation noise, ~1 % per linear), query chunking, and the block fed by the streaming provider."""
import pytest
import torch

import torch_ops as tops
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


def _dense_reference(w):
    """The same block in fp32 on the dequantized weights (original basis) with a plain dense linear."""
    dense = {k: ql.dequantize(getattr(w, k), torch.float32) for k in ("qkv", "out", "fc1", "fc2")}
    wd = BlockWeights(**dense, norm1=w.norm1.float(), norm2=w.norm2.float(), q_norm=w.q_norm.float(), k_norm=w.k_norm.float())

    def lin(t, wt, input_act=None):
        if input_act == "swiglu":
            g, u = t.chunk(2, dim=-1)
            t = torch.nn.functional.silu(g) * u
        return t @ wt.t()

    return blk.DiTBlock(HEADS, HD, linear=lin, ops=tops.TorchOps()), wd


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def test_attention_and_mlp_branches_match_the_dequantized_fp32_block():
    """The W4A8 branches differ from fp32 on the dequantized weights only by the int8 activation quantisation (~1 %
    per linear, outlier channels spread by the rotation) and bf16 intermediates."""
    x, w, mod, seg, cos, sin = make()
    ref_block, wd = _dense_reference(w)
    h = tops.rms(x, w.norm1, 1e-5)
    a = blk.DiTBlock(HEADS, HD).attention(h.clone(), w, cos, sin)
    a_ref = ref_block.attention(h.float(), wd, cos.float(), sin.float())
    m = blk.DiTBlock(HEADS, HD).mlp(h.clone(), w)
    m_ref = ref_block.mlp(h.float(), wd)
    assert _rel(a, a_ref) < 0.05 and _rel(m, m_ref) < 0.05, (_rel(a, a_ref), _rel(m, m_ref))


def test_block_matches_the_dequantized_fp32_block():
    x, w, _, seg, cos, sin = make()
    g = torch.Generator(device=DEV).manual_seed(9)
    mod = blk.Modulation(*(torch.randn(2, HID, generator=g, device=DEV) for _ in range(6)))  # unit-scale gates
    y = blk.DiTBlock(HEADS, HD)(x.clone(), w, mod, seg, cos, sin)
    ref_block, wd = _dense_reference(w)
    ref = ref_block(x.float(), wd, mod, seg, cos.float(), sin.float())
    assert torch.isfinite(y.float()).all()
    assert _rel(y.float() - x.float(), ref - x.float()) < 0.05


def test_chunked_attention_matches():
    """Query rows are independent, so chunking changes only which attention kernel runs and its summation order."""
    x, w, mod, seg, cos, sin = make(1)
    h = tops.rms(x, w.norm1, 1e-5)
    a = blk.DiTBlock(HEADS, HD).attention(h.clone(), w, cos, sin)
    b = blk.DiTBlock(HEADS, HD, attn_chunk=64).attention(h.clone(), w, cos, sin)
    assert _rel(b, a) < 1e-2


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


def test_attention_over_key_chunks_merges_to_full_attention():
    """cuDNN attention with its log-sum-exp over disjoint key chunks, merged, equals one attention call (the ring
    exchange of the token-sharded block relies on it)."""
    g = torch.Generator(device=DEV).manual_seed(3)
    q, k, v = (torch.randn(1, 4, n, 128, generator=g, device=DEV).to(torch.bfloat16) for n in (300, 700, 700))
    want = torch.nn.functional.scaled_dot_product_attention(q, k, v).float()
    acc = lse = None
    for a, b in ((0, 250), (250, 251), (251, 700)):
        o, l_ = blk.attention_lse(q, k[:, :, a:b], v[:, :, a:b])
        acc, lse = tops.merge_attention(acc, lse, o, l_)
    assert _rel(acc, want) < 1e-2, _rel(acc, want)


def test_ring_block_on_two_gpus_equals_one_gpu():
    """Token-sharded DiT block over 2 GPUs (ring and gather exchanges) against the same block on one GPU; run by
    torchrun in a child process when at least 2 GPUs are visible."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import subprocess
    import sys
    from pathlib import Path

    here = Path(__file__).resolve().parent
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2", "--master-addr=127.0.0.1",
           "--master-port=29531", str(here / "helpers" / "ring_block_check.py")]
    env = dict(__import__("os").environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    for tag in ("RING_OK", "GATHER_OK", "GATHER1_OK", "OVERLAP_OK"):
        assert tag in r.stdout, r.stdout[-3000:]


def test_fused_merge_kernel_equals_the_torch_merge():
    from minimax_h3_turbo_b200 import _lib

    g = torch.Generator(device=DEV).manual_seed(4)
    h, sq, d = 3, 257, 128
    q = torch.randn(1, h, sq, d, generator=g, device=DEV).to(torch.bfloat16)
    kv = [(torch.randn(1, h, n, d, generator=g, device=DEV).to(torch.bfloat16),
           torch.randn(1, h, n, d, generator=g, device=DEV).to(torch.bfloat16)) for n in (100, 37, 300)]
    acc = torch.empty(h, sq, d, device=DEV)
    lse_acc = torch.empty(h, sq, device=DEV)
    out = torch.empty(sq, h * d, dtype=torch.bfloat16, device=DEV)
    ref = ref_lse = None
    for i, (k, v) in enumerate(kv):
        o, lse = blk.attention_lse(q, k, v)
        ref, ref_lse = tops.merge_attention(ref, ref_lse, o, lse)
        lse = lse.reshape(h, sq).contiguous()
        _lib.check(_lib.lib().h3b_attn_merge(acc.data_ptr(), lse_acc.data_ptr(), o.data_ptr(), o.stride(1), o.stride(2),
                                             _lib.BF16, lse.data_ptr(), h, sq, d, int(i == 0),
                                             out.data_ptr() if i == len(kv) - 1 else None, h * d,
                                             _lib.stream_ptr(DEV)), "merge")
    want = ref[0].transpose(0, 1).reshape(sq, h * d)
    assert _rel(out, want) < 5e-3, _rel(out, want)


def test_merge_kernel_handles_empty_key_sets_and_refuses_other_dtypes():
    """A key set with no keys has log-sum-exp -inf: merging it changes nothing, and two empty sides give zeros (not NaN)."""
    from minimax_h3_turbo_b200 import _lib

    h, sq, d = 2, 40, 128
    g = torch.Generator(device=DEV).manual_seed(5)
    o = torch.randn(1, h, sq, d, generator=g, device=DEV).to(torch.bfloat16)
    lse = torch.randn(h, sq, generator=g, device=DEV)
    empty_o = torch.zeros_like(o)
    empty_lse = torch.full((h, sq), float("-inf"), device=DEV)
    acc = torch.empty(h, sq, d, device=DEV)
    acc_lse = torch.empty(h, sq, device=DEV)
    out = torch.empty(sq, h * d, dtype=torch.bfloat16, device=DEV)
    L = _lib.lib()

    def merge(oo, ll, first, last):
        _lib.check(L.h3b_attn_merge(acc.data_ptr(), acc_lse.data_ptr(), oo.data_ptr(), oo.stride(1), oo.stride(2), _lib.BF16,
                                    ll.data_ptr(), h, sq, d, int(first), out.data_ptr() if last else None, h * d,
                                    _lib.stream_ptr(DEV)), "merge")

    merge(empty_o, empty_lse, True, False)
    merge(o, lse, False, False)
    merge(empty_o, empty_lse, False, True)
    assert torch.equal(out, o[0].transpose(0, 1).reshape(sq, h * d))
    assert torch.equal(acc_lse, lse)
    merge(empty_o, empty_lse, True, False)
    merge(empty_o, empty_lse, False, True)
    assert torch.equal(out, torch.zeros_like(out))
    rc = L.h3b_attn_merge(acc.data_ptr(), acc_lse.data_ptr(), o.data_ptr(), o.stride(1), o.stride(2), _lib.FP16,
                          lse.data_ptr(), h, sq, d, 1, None, h * d, _lib.stream_ptr(DEV))
    assert rc == _lib.ERR_ARG and b"bf16" in L.h3b_last_error()
