"""Token sharding of the DiT block on CPU ranks (gloo, world size 2 to 4): the row split, the row all-gather and a sharded
block -- K/V exchanged point-to-point behind the local attention and merged by log-sum-exp ("overlap"), all-gathered
(at once or in head groups), or passed round a ring; everything else token-wise -- equal the unsharded block.  The
block's kernels are CUDA-only, so these ranks run it with a dense fp32 linear and the reference's torch operators
(tests/helpers/torch_ops.py); the GPU path runs the kernels (tests/test_block_gpu.py).  Also: a rank that leaves
between blocks, or never joins, makes the others raise within the process group's timeout instead of hanging."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import conftest  # noqa: F401  -- registers the package (also in the spawned ranks, which re-import this module)
import torch_ops as tops
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
        block = blk.DiTBlock(HEADS, HD, linear=dense, kv_exchange=exchange, kv_groups=groups, ops=tops.TorchOps())
        y = block(x[a:b].clone(), w, mod, _segments(a, b), cos[a:b], sin[a:b], spec)
        full = blk.gather_rows(y, spec)
        # by value (numpy), not as a torch tensor shared through a file descriptor: that handle dies with the worker
        q.put((rank, ok_gather, full.numpy().copy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,exchange,groups", [(2, "overlap", 1), (3, "overlap", 1), (4, "overlap", 1),
                                                  (2, "gather", 1), (3, "gather", 1), (2, "gather", 2), (3, "gather", 2),
                                                  (2, "ring", 1), (3, "ring", 1)])
def test_sharded_block_equals_unsharded(world, exchange, groups):
    """groups = 2: the K/V all-gather in two head groups, both started before either group's attention."""
    x, w, mod, cos, sin = make_case()
    ref = blk.DiTBlock(HEADS, HD, linear=dense, ops=tops.TorchOps())(x.clone(), w, mod, _segments(0, S), cos, sin)
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
        full = torch.from_numpy(full)
        assert ok_gather
        assert torch.allclose(full, ref, rtol=1e-5, atol=1e-5), (rank, (full - ref).abs().max())


def _tiny_worker(rank, world, port, q, exchange, n):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, w, mod, cos, sin = make_case()
        a, b = blk.shard_rows(n, world, rank)
        spec = blk.ShardSpec(a, b, n, dist.group.WORLD, world, rank)
        block = blk.DiTBlock(HEADS, HD, linear=dense, kv_exchange=exchange, ops=tops.TorchOps())
        y = block(x[a:b].clone(), w, mod, [(0, b - a, 0)] if b > a else [], cos[a:b], sin[a:b], spec)
        q.put((rank, blk.gather_rows(y, spec).numpy().copy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["overlap", "ring", "gather"])
def test_fewer_tokens_than_ranks(exchange):
    """2 tokens on 3 ranks: one rank owns no rows (its key set is empty, weight 0 in the merges)."""
    world, n = 3, 2
    x, w, mod, cos, sin = make_case()
    ref = blk.DiTBlock(HEADS, HD, linear=dense, ops=tops.TorchOps())(x[:n].clone(), w, mod, [(0, n, 0)], cos[:n], sin[:n])
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_tiny_worker, args=(r, world, port, q, exchange, n)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=90) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, full in res:
        full = torch.from_numpy(full)
        assert torch.isfinite(full).all()
        assert torch.allclose(full, ref, rtol=1e-5, atol=1e-5), (rank, (full - ref).abs().max())


def test_shard_rows_cover_everything():
    for total in (0, 1, 7, 59440):
        for world in (1, 2, 3, 8):
            spans = [blk.shard_rows(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1


def _post(q, item):
    """Send `item` and flush it to the parent before the caller's os._exit (a queue's feeder thread dies with it)."""
    q.put(item)
    q.close()
    q.join_thread()


def _dead_rank_worker(rank, world, port, q, leave_after):
    """Runs sharded blocks; rank `world - 1` leaves (exits without a word) after `leave_after` blocks.  The survivors
    must see their next collective fail within the process group's short timeout instead of waiting for ever."""
    import time
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=4))
    x, w, mod, cos, sin = make_case()
    a, b = blk.shard_rows(S, world, rank)
    spec = blk.ShardSpec(a, b, S, dist.group.WORLD, world, rank)
    block = blk.DiTBlock(HEADS, HD, linear=dense, ops=tops.TorchOps())
    y = x[a:b].clone()
    t0 = time.monotonic()
    for i in range(3):
        if rank == world - 1 and i == leave_after:
            _post(q, (rank, "left", None, 0.0))
            os._exit(0)  # between blocks: no collective of this rank is in flight
        try:
            y = block(y, w, mod, _segments(a, b), cos[a:b], sin[a:b], spec)
        except Exception as e:  # the survivor's K/V all-gather of block `i`
            _post(q, (rank, "raised", f"{type(e).__name__}: {str(e)[:200]}", time.monotonic() - t0))
            os._exit(0)
    _post(q, (rank, "finished", None, time.monotonic() - t0))
    os._exit(0)


@pytest.mark.parametrize("world", [2, 3])
def test_a_rank_that_leaves_between_blocks_makes_the_others_raise(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_dead_rank_worker, args=(r, world, port, q, 1)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        rank, what, err, t = q.get(timeout=120)
        res[rank] = (what, err, t)
    for p in procs:
        p.join(timeout=60)
        if p.exitcode is None:
            p.kill()
        assert p.exitcode == 0
    assert res[world - 1][0] == "left"
    for r in range(world - 1):
        what, err, t = res[r]
        assert what == "raised", res
        assert t < 60, res  # bounded by the process group's 4 s timeout (plus the blocks already run), not a hang


def _never_joins_worker(rank, world, port, q):
    import time
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    t0 = time.monotonic()
    try:
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=3))
        _post(q, (rank, "joined", None, time.monotonic() - t0))
    except Exception as e:
        _post(q, (rank, "raised", f"{type(e).__name__}: {str(e)[:200]}", time.monotonic() - t0))
    os._exit(0)


def test_a_rank_that_never_joins_makes_the_others_time_out():
    """World size 2, only rank 0 starts: its rendezvous gives up after the short timeout with an error."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_never_joins_worker, args=(0, 2, _port(), q))
    p.start()
    rank, what, err, t = q.get(timeout=120)
    p.join(timeout=60)
    if p.exitcode is None:
        p.kill()
    assert what == "raised", (what, err)
    assert t < 60
