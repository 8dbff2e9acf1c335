"""StreamingProvider state machine, run in CPU mode (identical bookkeeping, plain copies, no events) with faults injected
on the host through the `transfer=` hook: waits, overlap, slot reuse order, worker failures, timeouts, recovery after an
aborted forward, and resize/park.  The GPU copy path is covered by tests/test_stream_gpu.py."""
import threading
import time

import pytest
import torch

from minimax_h3_turbo_b200.h3 import stream as sm
from minimax_h3_turbo_b200.h3.config import H3Config
from minimax_h3_turbo_b200.h3.store import H3TFile
from minimax_h3_turbo_b200.h3.synth import synthetic_store_tensors
from minimax_h3_turbo_b200.h3.writer import write_h3t

CFG = H3Config(hidden=256, layers=6, refiner_layers=0, heads=2, head_dim=128, ffn=512, text_dim=64, video_channels=4,
               audio_channels=8, quant_group=16)


@pytest.fixture(scope="module")
def store(tmp_path_factory):
    path = tmp_path_factory.mktemp("stream") / "s.h3t"
    write_h3t(path, CFG, synthetic_store_tensors(CFG, group=16, scale_dtype="fp8", seed=9))
    f = H3TFile(path)
    yield f
    f.close()


def _forward(p, store, check=True, compute=None):
    p.begin_forward()
    try:
        for i in range(store.n_blocks):
            w = p.acquire(i)
            if check:
                assert torch.equal(w.fc1.q, store.block_weights_cpu(i).fc1.q), i
            if compute:
                compute()
            p.release(i)
    finally:
        p.end_forward()


def test_plans():
    class S:
        block_nbytes, n_blocks = 100, 10
    assert sm.plan_residency(S, 10_000) == 10
    assert sm.plan_residency(S, 700, ring=3) == 4  # 4 resident + 3 slots
    assert sm.plan_residency(S, 250, ring=3) == 0
    with pytest.raises(ValueError):
        sm.plan_residency(S, 1000, ring=0)
    assert sm.plan_pinned_blocks(S, 8, free_ram=10_000, pin_fraction=0.5, headroom=0) == 8
    assert sm.plan_pinned_blocks(S, 8, free_ram=1_000, pin_fraction=0.5, headroom=0) == 3


@pytest.mark.parametrize("resident,ring,prefetch", [(0, 1, 0), (0, 2, 1), (2, 3, 2), (1, 3, 4), (6, 3, 2)])
def test_every_block_arrives_with_its_bytes(store, resident, ring, prefetch):
    with sm.StreamingProvider(store, "cpu", resident=resident, ring=ring, prefetch=prefetch) as p:
        for _ in range(3):  # the lookahead wraps into the next forward
            _forward(p, store)
        s = p.stats()
        assert s["acquires"] == 3 * (6 - resident) and s["resident"] == resident


def test_acquire_waits_for_a_slow_copy(store):
    def slow(dst, src, nb):
        time.sleep(0.05)
        dst.copy_(src)

    with sm.StreamingProvider(store, "cpu", resident=0, ring=2, prefetch=0, transfer=slow) as p:
        _forward(p, store)
        assert p.stats()["waits"] >= 1 and p.stats()["wait_s"] > 0.02


def test_copies_overlap_compute(store):
    def slow(dst, src, nb):
        time.sleep(0.04)
        dst.copy_(src)

    compute = lambda: time.sleep(0.04)  # noqa: E731
    with sm.StreamingProvider(store, "cpu", resident=0, ring=3, prefetch=2, transfer=slow) as p:
        _forward(p, store, check=False, compute=compute)  # warm: the ring is primed
        t0 = time.perf_counter()
        _forward(p, store, check=False, compute=compute)
        overlapped = time.perf_counter() - t0
    serial = store.n_blocks * 0.08
    assert overlapped < 0.8 * serial, (overlapped, serial)


def test_no_slot_is_written_while_it_is_held(store):
    held = {}
    seen = []

    with sm.StreamingProvider(store, "cpu", resident=0, ring=2, prefetch=2) as p:
        def guarded(dst, src, nb):
            for s in p._slots:
                if s.buf.data_ptr() == dst.data_ptr():
                    seen.append(s.state)
                    assert s.state == sm.PENDING, "copy into a slot that is not pending"
            dst.copy_(src)

        p._transfer = guarded
        for _ in range(2):
            _forward(p, store)
    assert seen and all(st == sm.PENDING for st in seen)
    del held


def test_worker_failure_surfaces_and_close_still_works(store):
    calls = {"n": 0}

    def flaky(dst, src, nb):
        calls["n"] += 1
        if calls["n"] == 3:
            raise OSError("injected read failure")
        dst.copy_(src)

    p = sm.StreamingProvider(store, "cpu", resident=0, ring=2, prefetch=1, transfer=flaky)
    with pytest.raises(RuntimeError, match="injected read failure"):
        _forward(p, store, check=False)
    p.close()
    with pytest.raises(RuntimeError, match="closed"):
        p.acquire(0)


def test_timeout_reports_the_slot_states(store):
    gate = threading.Event()

    def stuck(dst, src, nb):
        gate.wait(5)
        dst.copy_(src)

    p = sm.StreamingProvider(store, "cpu", resident=0, ring=1, prefetch=0, transfer=stuck, wait_timeout=0.3)
    p.begin_forward()
    with pytest.raises(TimeoutError, match="slots 0:pending"):
        p.acquire(0)
    gate.set()
    p.end_forward()
    p.close()


def test_exception_mid_forward_is_recovered_by_end_forward(store):
    with sm.StreamingProvider(store, "cpu", resident=1, ring=2, prefetch=1) as p:
        p.begin_forward()
        p.acquire(0)
        p.acquire(1)  # never released: the forward "crashed"
        p.end_forward()
        _forward(p, store)
        p.begin_forward()
        p.acquire(2)
        p.begin_forward()  # a new forward without end_forward self-heals
        _forward(p, store)


def test_ring_exhaustion_and_double_acquire_are_errors(store):
    with sm.StreamingProvider(store, "cpu", resident=0, ring=1, prefetch=0) as p:
        p.begin_forward()
        p.acquire(0)
        with pytest.raises(RuntimeError, match="already acquired"):
            p.acquire(0)
        with pytest.raises(RuntimeError, match="ring slots are held"):
            p.acquire(1)
        with pytest.raises(RuntimeError, match="not acquired"):
            p.release(2)
        p.end_forward()
        with pytest.raises(IndexError):
            p.acquire(99)


def test_resize_and_park(store):
    with sm.StreamingProvider(store, "cpu", resident=1, ring=2, prefetch=1) as p:
        _forward(p, store)
        assert p.resize(0, 0) == 0 and p.parked
        with pytest.raises(RuntimeError, match="parked"):
            p.acquire(3)
        assert p.resize(3, 2) == 5 * store.block_nbytes and not p.parked
        _forward(p, store)
        assert p.resize(6, 3) == 6 * store.block_nbytes
        _forward(p, store)
        p.begin_forward()
        with pytest.raises(RuntimeError, match="during a forward"):
            p.resize(0, 1)
        p.end_forward()


def test_wait_prefetch_and_buffer_of(store):
    with sm.StreamingProvider(store, "cpu", resident=2, ring=3, prefetch=3) as p:
        p.wait_prefetch(10)
        assert torch.equal(p.buffer_of(2), store.block_tensor(2))
        assert p.buffer_of(0) is not None and p.buffer_of(5) is None
        assert "slots" in p.stats()["state"]
