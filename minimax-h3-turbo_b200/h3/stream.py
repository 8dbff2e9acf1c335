"""Block streaming for the H3 DiT: resident blocks plus a ring of device slots fed by one host -> device copy per block.

Same API and behaviour as the reference's `h3turbo/h3/stream.py` (StreamingProvider :115-623, plan_residency :61-71,
plan_pinned_blocks :74-78); the copy path runs in libh3b.so's native engine:

* The first `resident` blocks stay on the device; the others cycle through `ring` slots, each one uint8 buffer of
  `block_nbytes` whose typed tensors are zero-copy views (H3TFile.block_weights_from).
* A worker thread decides which block goes into which slot (the block asked for first, then the next `prefetch`
  streamed blocks in cyclic order; slots are reused FREE first, then released (IDLE) and then prefetched-but-unused
  (READY) ones, least recently used first) and hands each copy to the engine, which runs it on its own copy stream.
  Slot reuse is ordered on the device: a copy into a slot waits for the slot's `done` event (recorded by release() on
  the compute stream), and acquire() makes the compute stream wait for the slot's `ready` event.  The host only waits
  for a copy to be issued, so the CPU can run ahead of the GPU without overwriting weights a queued kernel still reads.
* Host sources per streamed block: the file mapping page-locked in place ("registered", zero copy), a page-locked copy
  ("pinned"), a multi-threaded memcpy into one of two page-locked staging buffers ("staged"), or pageable memory.
  pin="auto" bounds all page-locking by free RAM.
* device="cpu" runs the same state machine with plain copies and no events, so tests exercise the bookkeeping,
  ordering and failure paths without a GPU.  `transfer=` replaces the copy (fault injection, slow copies).
"""
from __future__ import annotations

import atexit
import ctypes
import os
import threading
import time
import weakref
from dataclasses import dataclass
from typing import Callable, Dict, List, Optional, Union

import numpy as np
import torch

from .. import _lib
from .store import H3TFile
from .types import BlockWeights

_GIB = 1 << 30
_CUDA_MARGIN = 512 << 20
FREE, PENDING, READY, ACQUIRED, IDLE = range(5)
_STATE_NAMES = ("free", "pending", "ready", "acquired", "idle")


def free_ram_bytes() -> int:
    """Physical memory available without swapping (includes reclaimable page cache)."""
    try:
        import psutil

        return int(psutil.virtual_memory().available)
    except ImportError:
        pass
    if os.path.exists("/proc/meminfo"):
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return int(line.split()[1]) * 1024
    raise RuntimeError("cannot determine free RAM (install psutil, or pass pin_blocks explicitly)")


def plan_residency(store: H3TFile, free_vram_bytes: int, reserve_bytes: int = 0, ring: int = 3) -> int:
    """The most leading blocks that can stay resident while the streaming ring (min(ring, streamed) slots) still fits
    into free_vram_bytes - reserve_bytes; 0 when not even the ring fits."""
    if ring < 1:
        raise ValueError("ring must be >= 1")
    avail, blk, n = free_vram_bytes - reserve_bytes, store.block_nbytes, store.n_blocks
    for r in range(n, -1, -1):
        if (r + min(ring, n - r)) * blk <= avail:
            return r
    return 0


def plan_pinned_blocks(store: H3TFile, streamed: int, free_ram: int, pin_fraction: float = 0.5, headroom: int = 4 * _GIB) -> int:
    """How many streamed blocks to page-lock: at most pin_fraction of free RAM, never below `headroom` of free RAM,
    with two staging buffers reserved out of the budget."""
    budget = min(free_ram * pin_fraction, free_ram - headroom) - 2 * store.block_nbytes
    return int(max(0, min(streamed, budget // store.block_nbytes)))


@dataclass
class _Slot:
    idx: int
    buf: torch.Tensor
    weights: BlockWeights
    state: int = FREE
    block: Optional[int] = None
    stamp: int = 0
    cpu_done: bool = True  # CPU mode: the copy into this slot has finished


class StreamingProvider:
    """BlockProvider over an H3TFile.  Use as a context manager or call close()."""

    def __init__(self, store: H3TFile, device: Union[str, torch.device] = "cuda", resident: Union[int, str] = "auto",
                 prefetch: int = 2, pin: Union[bool, str] = "auto", ring: int = 3, *, reserve_bytes: int = 1536 << 20,
                 free_vram_bytes: Optional[int] = None, pin_fraction: float = 0.5, ram_headroom_bytes: int = 4 * _GIB,
                 pin_blocks: Optional[int] = None, pin_mode: str = "auto",
                 transfer: Optional[Callable[[torch.Tensor, torch.Tensor, bool], None]] = None, wait_timeout: float = 600.0):
        if ring < 1 or prefetch < 0 or pin not in (True, False, "auto") or pin_mode not in ("auto", "register", "copy", "stage"):
            raise ValueError("ring >= 1, prefetch >= 0, pin in (True, False, 'auto'), pin_mode in ('auto', 'register', 'copy', 'stage')")
        if not (resident == "auto" or (isinstance(resident, int) and resident >= 0)):
            raise ValueError("resident must be 'auto' or a non-negative int")
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.store, self.device, self._cuda = store, dev, dev.type == "cuda"
        self.n_blocks, self._prefetch, self._timeout = store.n_blocks, prefetch, wait_timeout
        self._transfer = transfer
        self._cv = threading.Condition()
        self._slots: List[_Slot] = []
        self._by_block: Dict[int, _Slot] = {}
        self._resident: Dict[int, tuple] = {}
        self._kind: Dict[int, str] = {}
        self._host: Dict[int, torch.Tensor] = {}
        self._reg_ptrs: List[int] = []
        self._streamed: List[int] = []
        self._pos, self._demand, self._tick = -1, None, 0
        self._stop = self._closed = self._in_forward = False
        self._error: Optional[BaseException] = None
        self._thread: Optional[threading.Thread] = None
        self._inline = False  # copies issued by the caller's thread (see _start_worker)
        self._engine: Optional[int] = None
        self._n_staging = 0
        self._st = dict(acquires=0, waits=0, wait_s=0.0, copies=0, bytes=0, busy_s=0.0)
        self._plan_info: Dict[str, object] = {}
        _LIVE.add(self)
        try:
            self._build(resident, ring, pin, pin_mode, reserve_bytes, free_vram_bytes, pin_fraction, ram_headroom_bytes, pin_blocks)
        except BaseException:
            self.close()
            raise

    # ------------------------------------------------------------------ construction
    def _alloc(self) -> torch.Tensor:
        return torch.empty(self.store.block_nbytes, dtype=torch.uint8, device=self.device)

    def _make_engine(self, n_slots: int, staging: int) -> None:
        self._destroy_engine()
        if not self._cuda:
            return
        L = _lib.lib()
        h = ctypes.c_void_p()
        _lib.check(L.h3b_streamer_create(self.device.index, n_slots, staging, self.store.block_nbytes,
                                         min(16, os.cpu_count() or 8), ctypes.byref(h)), "streamer")
        self._engine = h.value

    def _destroy_engine(self) -> None:
        if self._engine is not None:
            _lib.lib().h3b_streamer_destroy(self._engine)
            self._engine = None

    def _build(self, resident, ring, pin, pin_mode, reserve, free_vram, pin_fraction, headroom, pin_blocks) -> None:
        st, n = self.store, self.store.n_blocks
        auto = resident == "auto"
        if auto:
            free = free_vram if free_vram is not None else (torch.cuda.mem_get_info(self.device)[0] if self._cuda else free_ram_bytes() // 2)
            resident = plan_residency(st, free, reserve + (_CUDA_MARGIN if self._cuda else 0), ring)
        for b in range(min(int(resident), n)):
            try:
                buf = self._alloc()
            except torch.cuda.OutOfMemoryError:
                if auto:
                    break
                raise
            buf.copy_(st.block_tensor(b))
            self._resident[b] = (buf, st.block_weights_from(buf))
        self._streamed = list(range(len(self._resident), n))
        for k in range(min(ring, len(self._streamed))):
            try:
                buf = self._alloc()
            except torch.cuda.OutOfMemoryError as e:
                raise torch.cuda.OutOfMemoryError(f"cannot allocate streaming slot {k + 1} ({st.block_nbytes / 2**20:.0f} MiB): "
                                                  "lower resident/ring or free VRAM") from e
            self._slots.append(_Slot(k, buf, st.block_weights_from(buf)))
        if self._streamed:
            self._plan_host(pin, pin_mode, pin_fraction, headroom, pin_blocks)
            self._make_engine(len(self._slots), self._n_staging)
            self._start_worker()

    def _register(self, t: torch.Tensor, read_only: bool) -> bool:
        L = _lib.lib()
        rc = L.h3b_host_register(t.data_ptr(), t.numel(), int(read_only))
        if rc == 0:
            self._reg_ptrs.append(t.data_ptr())
            return True
        self._plan_info["register_error" if read_only else "pin_error"] = (L.h3b_last_error() or b"").decode(errors="replace")
        return False

    def _plan_host(self, pin, pin_mode, pin_fraction, headroom, pin_blocks) -> None:
        st, S = self.store, self._streamed
        if pin is False or pin_mode == "stage":
            want = 0
        elif pin is True:
            want = len(S)
        elif pin_blocks is not None:
            want = max(0, min(len(S), pin_blocks))
        else:
            avail = free_ram_bytes() if self._cuda else 0
            self._plan_info["ram_available_gib"] = round(avail / _GIB, 2)
            want = plan_pinned_blocks(st, len(S), avail, pin_fraction, headroom) if self._cuda else 0
        self._plan_info["pinned_wanted"] = want
        mode = "copy" if pin_mode == "stage" else pin_mode
        for b in S[:want]:
            if not self._cuda:
                break
            t = None
            if mode in ("auto", "register"):
                view = st.block_tensor(b)  # the file pages themselves: zero copy, no second RAM copy
                if self._register(view, True):
                    t, self._kind[b] = view, "registered"
                elif pin_mode == "register":
                    break
                else:
                    mode = "copy"
            if t is None:
                if mode == "register":
                    break
                t = torch.empty(st.block_nbytes, dtype=torch.uint8)
                if not self._register(t, False):
                    break  # out of lockable memory: the rest is staged
                np.copyto(t.numpy(), st.block_bytes(b))
                self._kind[b] = "pinned"
            self._host[b] = t
        rest = [b for b in S if b not in self._kind]
        if rest and self._cuda and pin is not False:
            self._n_staging = 2
            self._kind.update({b: "staged" for b in rest})
        for b in rest:
            self._kind.setdefault(b, "pageable")

    # ------------------------------------------------------------------ worker
    def _start_worker(self) -> None:
        """Copies from pinned or registered host memory only enqueue work (a device-side wait, cudaMemcpyAsync, an event
        record), so they are issued inline by the thread that calls acquire/release ("inline" mode): no worker thread
        has to win the interpreter lock from a busy model thread before a copy starts.  Staged and pageable copies
        block the host, and test hooks may sleep, so those run on the worker thread (stream.py:305-331)."""
        self._inline = (self._cuda and self._transfer is None and bool(self._streamed)
                        and all(self._kind.get(b) in ("registered", "pinned") for b in self._streamed))
        self._plan_info["issue"] = "inline" if self._inline else "worker"
        if self._inline:
            self._pump()
            return
        self._thread = threading.Thread(target=self._run, name="h3b-stream", daemon=True)
        self._thread.start()

    def _pump(self) -> None:
        """Inline mode: issue every copy the lookahead window allows, on the calling thread."""
        if not self._inline:
            return
        while True:
            with self._cv:
                if self._closed or self._error is not None:
                    return
                job = self._next_job()
            if job is None:
                return
            try:
                self._issue(*job)
            except BaseException as e:
                with self._cv:
                    self._error = e
                raise
            with self._cv:
                job[0].state = READY

    def _targets(self) -> List[int]:
        S = self._streamed
        out = [self._demand] if self._demand is not None else []
        out += [S[(self._pos + 1 + k) % len(S)] for k in range(min(self._prefetch, len(S)))]
        return out

    def _pick_slot(self, protect) -> Optional[_Slot]:
        for s in self._slots:
            if s.state == FREE:
                return s
        for state in (IDLE, READY):
            cand = [s for s in self._slots if s.state == state and s.block not in protect]
            if cand:
                return min(cand, key=lambda s: s.stamp)
        return None

    def _next_job(self, commit: bool = True):
        targets = self._targets()
        for k, t in enumerate(targets):
            if t in self._by_block:
                continue
            slot = self._pick_slot(() if (k == 0 and t == self._demand) else targets)
            if slot is None:
                return None
            if commit:
                if slot.block is not None:
                    del self._by_block[slot.block]
                self._tick += 1
                slot.state, slot.block, slot.stamp = PENDING, t, self._tick
                self._by_block[t] = slot
            return slot, t
        return None

    def _run(self) -> None:
        with torch.inference_mode():  # slot buffers made under inference mode must be written under it too
            if self._cuda:
                torch.cuda.set_device(self.device)
            try:
                while True:
                    with self._cv:
                        while True:
                            if self._stop:
                                return
                            job = self._next_job()
                            if job:
                                break
                            self._cv.wait()
                    self._issue(*job)
                    with self._cv:
                        job[0].state = READY
                        self._cv.notify_all()
            except BaseException as e:  # surfaces in the next acquire()
                with self._cv:
                    self._error = e
                    self._cv.notify_all()

    def _source(self, b: int) -> torch.Tensor:
        return self._host.get(b) if b in self._host else self.store.block_tensor(b)

    def _issue(self, slot: _Slot, b: int) -> None:
        t0 = time.perf_counter()
        kind = self._kind[b]
        src = self._source(b)
        nb = self.store.block_nbytes
        if not self._cuda:
            slot.cpu_done = False
            (self._transfer or (lambda d, s, n: d.copy_(s)))(slot.buf, src, False)
            slot.cpu_done = True
        elif self._transfer is not None:
            L = _lib.lib()
            _lib.check(L.h3b_streamer_begin(self._engine, slot.idx), "streamer")
            with torch.cuda.stream(torch.cuda.ExternalStream(L.h3b_streamer_stream(self._engine), device=self.device)):
                self._transfer(slot.buf, src, kind != "pageable")
            _lib.check(L.h3b_streamer_end(self._engine, slot.idx, nb), "streamer")
        else:
            mode = {"registered": _lib.COPY_DIRECT, "pinned": _lib.COPY_DIRECT, "staged": _lib.COPY_STAGED}.get(kind, _lib.COPY_PAGEABLE)
            _lib.check(_lib.lib().h3b_streamer_copy(self._engine, slot.idx, slot.buf.data_ptr(), src.data_ptr(), nb, mode),
                       "streamer copy")
        with self._cv:
            self._st["copies"] += 1
            self._st["bytes"] += nb
            self._st["busy_s"] += time.perf_counter() - t0

    # ------------------------------------------------------------------ BlockProvider
    def _check(self) -> None:
        if self._closed:
            raise RuntimeError("StreamingProvider is closed")
        if self._error is not None:
            raise RuntimeError(f"H3 streaming worker failed: {self._error!r}") from self._error

    def begin_forward(self) -> None:
        if self._in_forward:  # the previous forward never reached end_forward
            self.end_forward()
        self._in_forward = True

    def acquire(self, i: int) -> BlockWeights:
        if not 0 <= i < self.n_blocks:
            raise IndexError(f"block {i} out of range [0, {self.n_blocks})")
        if self._closed:
            raise RuntimeError("StreamingProvider is closed")
        if i in self._resident:
            return self._resident[i][1]
        if not self._slots:
            raise RuntimeError("H3 streaming provider is parked (it holds no device memory); resize() it before a forward")
        t0 = time.perf_counter()
        deadline = t0 + self._timeout
        waited = False
        if self._inline:
            with self._cv:
                self._check()
                if i not in self._by_block:
                    if all(s.state == ACQUIRED for s in self._slots):
                        raise RuntimeError(f"all {len(self._slots)} ring slots are held; release() a block before acquiring block {i} (ring too small?)")
                    self._demand = i
            self._pump()
        with self._cv:
            self._check()
            while True:
                slot = self._by_block.get(i)
                if slot is None:
                    if all(s.state == ACQUIRED for s in self._slots):
                        raise RuntimeError(f"all {len(self._slots)} ring slots are held; release() a block before acquiring block {i} (ring too small?)")
                    self._demand = i
                    self._cv.notify_all()
                elif slot.state == ACQUIRED:
                    raise RuntimeError(f"block {i} is already acquired")
                elif slot.state in (READY, IDLE):
                    break
                waited = True
                left = deadline - time.perf_counter()
                if left <= 0:
                    raise TimeoutError(f"timed out after {self._timeout:.0f}s waiting for block {i}: {self._dump()}")
                self._cv.wait(min(left, 1.0))
                self._check()
            slot.state = ACQUIRED
            self._tick += 1
            slot.stamp = self._tick
            if self._demand == i:
                self._demand = None
            self._pos = self._streamed.index(i)
            self._st["acquires"] += 1
            if waited:
                self._st["waits"] += 1
                self._st["wait_s"] += time.perf_counter() - t0
            self._cv.notify_all()  # the lookahead window moved
        if self._cuda:
            _lib.check(_lib.lib().h3b_streamer_acquire(self._engine, slot.idx, _lib.stream_ptr(self.device)), "streamer acquire")
        self._pump()
        return slot.weights

    def release(self, i: int) -> None:
        if i in self._resident:
            return
        with self._cv:
            slot = self._by_block.get(i)
            if slot is None or slot.state != ACQUIRED:
                raise RuntimeError(f"release({i}) but block {i} is not acquired")
            if self._cuda:  # every kernel that reads the slot is already enqueued on the current stream
                _lib.check(_lib.lib().h3b_streamer_release(self._engine, slot.idx, _lib.stream_ptr(self.device)), "streamer release")
            slot.state = IDLE
            self._tick += 1
            slot.stamp = self._tick
            self._cv.notify_all()
        self._pump()

    def end_forward(self) -> None:
        """Reset for the next forward (safe after an exception): held slots are released behind the current stream and
        the lookahead restarts at the first streamed block."""
        with self._cv:
            for s in self._slots:
                if s.state == ACQUIRED:
                    if self._cuda and not self._closed and self._engine is not None:
                        _lib.lib().h3b_streamer_release(self._engine, s.idx, _lib.stream_ptr(self.device))
                    s.state = IDLE
            self._pos, self._demand, self._in_forward = -1, None, False
            self._cv.notify_all()
        if not self._closed:
            self._pump()

    # ------------------------------------------------------------------ residency changes (between forwards)
    def device_bytes(self) -> int:
        return (len(self._resident) + len(self._slots)) * self.store.block_nbytes

    def _stop_worker(self) -> None:
        if self._thread is None:
            return
        with self._cv:
            self._stop = True
            self._cv.notify_all()
        if self._thread is not threading.current_thread():
            self._thread.join(timeout=120)
        self._thread, self._stop = None, False

    def _lock_host(self, b: int, headroom: int) -> bool:
        if not self._cuda or self._kind.get(b) in ("registered", "pinned"):
            return self._kind.get(b) in ("registered", "pinned")
        try:
            if free_ram_bytes() - self.store.block_nbytes < headroom:
                return False
        except RuntimeError:
            return False
        view = self.store.block_tensor(b)
        if not self._register(view, True):
            return False
        self._host[b], self._kind[b] = view, "registered"
        return True

    def resize(self, resident: int, ring: int = 3, *, lock_host: bool = True, ram_headroom_bytes: int = 3 * _GIB) -> int:
        """Change the resident prefix and the ring between forwards, keeping the host side.  resize(0, 0) parks the
        provider (no device memory).  Returns the device bytes now held."""
        if self._closed:
            raise RuntimeError("StreamingProvider is closed")
        if self._in_forward:
            raise RuntimeError("resize() during a forward")
        self._stop_worker()
        self._inline = False
        if self._cuda:
            torch.cuda.synchronize(self.device)
        n = self.n_blocks
        resident = max(0, min(int(resident), n))
        with self._cv:
            self._slots, self._by_block = [], {}
            self._pos, self._demand = -1, None
        self._destroy_engine()
        for b in sorted(self._resident, reverse=True):
            if b >= resident:
                if lock_host:
                    self._lock_host(b, ram_headroom_bytes)
                del self._resident[b]
        if self._cuda:
            torch.cuda.empty_cache()
        for b in range(resident):
            if b in self._resident:
                continue
            try:
                buf = self._alloc()
            except torch.cuda.OutOfMemoryError:
                resident = b
                break
            buf.copy_(self._source(b))
            self._resident[b] = (buf, self.store.block_weights_from(buf))
        for b in [b for b in self._resident if b >= resident]:
            del self._resident[b]
        self._streamed = list(range(resident, n))
        if self._streamed:
            if lock_host:
                for b in self._streamed:
                    if not self._lock_host(b, ram_headroom_bytes):
                        break
            if self._cuda and any(self._kind.get(b) not in ("registered", "pinned") for b in self._streamed):
                self._n_staging = 2
            for b in self._streamed:
                if self._kind.get(b) not in ("registered", "pinned"):
                    self._kind[b] = "staged" if self._n_staging else "pageable"
            for k in range(min(max(0, ring), len(self._streamed))):
                try:
                    buf = self._alloc()
                except torch.cuda.OutOfMemoryError as e:
                    if k:
                        break
                    raise torch.cuda.OutOfMemoryError(f"cannot allocate a streaming slot ({self.store.block_nbytes / 2**20:.0f} MiB)") from e
                self._slots.append(_Slot(k, buf, self.store.block_weights_from(buf)))
            if self._slots:
                self._make_engine(len(self._slots), self._n_staging)
                self._start_worker()
        return self.device_bytes()

    @property
    def parked(self) -> bool:
        return bool(self._streamed) and not self._slots

    # ------------------------------------------------------------------ introspection / lifecycle
    def buffer_of(self, i: int) -> Optional[torch.Tensor]:
        if i in self._resident:
            return self._resident[i][0]
        with self._cv:
            s = self._by_block.get(i)
            return s.buf if s is not None and s.state in (READY, IDLE, ACQUIRED) else None

    def wait_prefetch(self, timeout: float = 60.0) -> None:
        """Block until the worker has nothing left to issue and every issued copy has landed."""
        deadline = time.perf_counter() + timeout
        self._pump()
        with self._cv:
            while self._thread is not None and not self._stop and self._error is None and (
                    any(s.state == PENDING for s in self._slots) or self._next_job(commit=False) is not None):
                left = deadline - time.perf_counter()
                if left <= 0:
                    raise TimeoutError(f"prefetch did not settle: {self._dump()}")
                self._cv.wait(min(left, 0.5))
            self._check()
            held = [s for s in self._slots if s.state in (READY, IDLE)]
        if self._cuda and self._engine is not None:
            for s in held:
                _lib.check(_lib.lib().h3b_streamer_wait(self._engine, s.idx, max(0.0, deadline - time.perf_counter())), "prefetch wait")

    def _dump(self) -> str:
        return ("slots " + ", ".join(f"{s.idx}:{_STATE_NAMES[s.state]}:{s.block}" for s in self._slots)
                + f"; pos={self._pos} demand={self._demand}")

    def stats(self) -> Dict[str, object]:
        with self._cv:
            kinds: Dict[str, int] = {}
            for k in self._kind.values():
                kinds[k] = kinds.get(k, 0) + 1
            blk = self.store.block_nbytes
            return dict(self._st, resident=len(self._resident), streamed=len(self._streamed), slots=len(self._slots),
                        host_kinds=kinds, gpu_bytes=(len(self._resident) + len(self._slots)) * blk,
                        locked_host_bytes=len(self._reg_ptrs) * blk, plan=dict(self._plan_info), state=self._dump())

    def reset_stats(self) -> None:
        with self._cv:
            self._st = dict(acquires=0, waits=0, wait_s=0.0, copies=0, bytes=0, busy_s=0.0)

    def close(self) -> None:
        if self._closed:
            return
        with self._cv:
            self._closed = self._stop = True
            self._cv.notify_all()
        if self._thread is not None and self._thread is not threading.current_thread():
            self._thread.join(timeout=120)
        if self._cuda:
            try:
                torch.cuda.synchronize(self.device)
            except Exception:
                pass
            self._destroy_engine()
            L = _lib.lib() if self._reg_ptrs else None
            for ptr in self._reg_ptrs:
                L.h3b_host_unregister(ptr)
        self._reg_ptrs = []
        self._slots, self._by_block, self._resident, self._host = [], {}, {}, {}
        self._kind = {}
        if self._cuda:
            torch.cuda.empty_cache()

    def __enter__(self) -> "StreamingProvider":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


_LIVE: "weakref.WeakSet[StreamingProvider]" = weakref.WeakSet()


@atexit.register
def _close_all() -> None:  # a forgotten close() must not leave the worker inside CUDA at interpreter exit
    for p in list(_LIVE):
        try:
            p.close()
        except Exception:
            pass
