"""Token sharding of the DiT block on CPU ranks (gloo, world size 2 and 3): the row split, the row all-gather and a
sharded block -- K/V all-gathered (at once or in head groups), or passed round a ring with the attention merged by
log-sum-exp; everything else
token-wise -- equal the unsharded block.  The W4A8 linear is CUDA-only,
so these ranks run the block with a dense fp32 linear; the GPU path swaps in the qlinear (tests/test_block_gpu.py)."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import conftest  # noqa: F401  -- registers the package (also in the spawned ranks, which re-import this module)
from minimax_h3_turbo_b200.h3 import block as blk
from minimax_h3_turbo_b200.h3.types import BlockWeights

HID, HEADS, HD, FFN, S = 64, 2, 32, 96, 37


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def dense(x, w, input_act=None):
    if input_act == "swiglu":
        g, u = x.chunk(2, dim=-1)
        x = torch.nn.functional.silu(g) * u
    return x @ w.t()


def make_case(seed=0):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    w = BlockWeights(qkv=r(3 * HID, HID) * 0.1, out=r(HID, HID) * 0.1, fc1=r(2 * FFN, HID) * 0.1, fc2=r(HID, FFN) * 0.1,
                     norm1=1 + 0.1 * r(HID), norm2=1 + 0.1 * r(HID), q_norm=1 + 0.1 * r(HD), k_norm=1 + 0.1 * r(HD))
    mod = blk.Modulation(*(0.1 * r(2, HID) for _ in range(6)))
    x = r(S, HID)
    pos = blk.video_audio_positions(3, 2, 5, S - 30, "cpu")
    cos, sin = blk.rope_tables(pos, torch.tensor([1.0, 0.5, 0.25, 0.125]), torch.float32)
    return x, w, mod, cos, sin


def _segments(a, b):
    """Rows [0, 30) use modulation row 0 (video), [30, S) row 1 (audio); clipped to the local shard [a, b)."""
    out = []
    for s0, s1, row in ((0, 30, 0), (30, S, 1)):
        lo, hi = max(a, s0), min(b, s1)
        if hi > lo:
            out.append((lo - a, hi - a, row))
    return out


def _worker(rank, world, port, q, exchange, groups):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, w, mod, cos, sin = make_case()
        a, b = blk.shard_rows(S, world, rank)
        spec = blk.ShardSpec(a, b, S, dist.group.WORLD, world, rank)
        g = blk.gather_rows(torch.arange(a, b, dtype=torch.float32).view(-1, 1), spec)
        ok_gather = torch.equal(g.view(-1), torch.arange(S, dtype=torch.float32))
        block = blk.DiTBlock(HEADS, HD, linear=dense, kv_exchange=exchange, kv_groups=groups)
        y = block(x[a:b].clone(), w, mod, _segments(a, b), cos[a:b], sin[a:b], spec)
        full = blk.gather_rows(y, spec)
        q.put((rank, ok_gather, full))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,exchange,groups", [(2, "gather", 1), (3, "gather", 1), (2, "gather", 2), (3, "gather", 2),
                                                  (2, "ring", 1), (3, "ring", 1)])
def test_sharded_block_equals_unsharded(world, exchange, groups):
    """groups = 2: the K/V all-gather in two head groups, both started before either group's attention."""
    x, w, mod, cos, sin = make_case()
    ref = blk.DiTBlock(HEADS, HD, linear=dense)(x.clone(), w, mod, _segments(0, S), cos, sin)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, exchange, groups)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=90) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, ok_gather, full in res:
        assert ok_gather
        assert torch.allclose(full, ref, rtol=1e-5, atol=1e-5), (rank, (full - ref).abs().max())


def test_shard_rows_cover_everything():
    for total in (0, 1, 7, 59440):
        for world in (1, 2, 3, 8):
            spans = [blk.shard_rows(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1
