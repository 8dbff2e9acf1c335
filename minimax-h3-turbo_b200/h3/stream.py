"""Block streaming for the H3 DiT: a resident prefix of blocks plus a ring of device slots refilled by one host -> device
copy per block, behind the reference's StreamingProvider interface (h3turbo/h3/stream.py: StreamingProvider :115-623,
plan_residency :61-71, plan_pinned_blocks :74-78).

Design:

* Slots are assigned by position, not by search: the j-th streamed block always lands in slot j mod `ring`.  A forward
  walks the blocks in order, so while block j computes, blocks j+1 .. j+prefetch (cyclically, into the next forward)
  are copied into the other slots; a slot is refilled as soon as the block it held has been released.  With
  prefetch >= ring the window simply stops at the slot still in use.
* Ordering is on the device.  The native engine of libh3b.so (h3b_streamer_*) owns a copy stream and two events per
  slot: a copy into a slot first waits (on the device) for the slot's `done` event, which release() records on the
  compute stream, and acquire() makes the compute stream wait for the slot's `ready` event.  The host never waits for
  the GPU, so the model thread can run ahead without a copy overwriting weights that queued kernels still read.
* Who issues a copy depends on the host source.  From page-locked memory (the file mapping registered in place, or a
  page-locked copy of the block) a copy is only enqueued, so the model thread issues it itself at acquire / release
  time ("inline").  Staged copies (a multi-threaded memcpy into page-locked bounce buffers), pageable copies and
  custom `transfer=` hooks block the host, so a copier thread runs them from a FIFO of (slot, block) jobs that the
  model thread schedules ("worker"); acquire() waits (bounded by `wait_timeout`) until its block's job has been issued.
* device="cpu" runs the same scheduling with plain copies (tests of the bookkeeping, ordering and failure paths).
"""
from __future__ import annotations

import atexit
import ctypes
import os
import queue
import threading
import time
import weakref
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Tuple, Union

import torch

from .. import _lib
from .store import H3TFile
from .types import BlockWeights

_GIB = 1 << 30
_CUDA_MARGIN = 512 << 20  # device memory kept free for the CUDA context and allocator slack when planning residency
FREE, PENDING, READY, ACQUIRED, IDLE = range(5)  # slot states: empty / copy queued / copy issued / in use / released
_STATE = ("free", "pending", "ready", "acquired", "idle")
_PAGE_LOCKED = ("registered", "pinned")


def free_ram_bytes() -> int:
    """Host memory available without swapping (MemAvailable, page cache included)."""
    try:
        import psutil

        return int(psutil.virtual_memory().available)
    except ImportError:
        pass
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemAvailable:"):
                    return 1024 * int(line.split()[1])
    except OSError:
        pass
    raise RuntimeError("cannot determine free RAM (install psutil, or pass pin_blocks explicitly)")


def plan_residency(store: H3TFile, free_vram_bytes: int, reserve_bytes: int = 0, ring: int = 3) -> int:
    """The largest resident prefix r such that r blocks plus the ring for the n - r streamed ones (min(ring, n - r)
    slots) fit in free_vram_bytes - reserve_bytes; 0 when not even the ring fits."""
    if ring < 1:
        raise ValueError("ring must be >= 1")
    fits = (free_vram_bytes - reserve_bytes) // store.block_nbytes  # whole blocks that fit
    n = store.n_blocks
    if fits >= n:
        return n
    # with r < n resident, r + min(ring, n - r) slots are needed; that count grows with r, so take the largest r
    best = 0
    for r in range(n):
        if r + min(ring, n - r) <= fits:
            best = r
    return best


def plan_pinned_blocks(store: H3TFile, streamed: int, free_ram: int, pin_fraction: float = 0.5,
                       headroom: int = 4 * _GIB) -> int:
    """How many of the streamed blocks to page-lock on the host: within pin_fraction of free RAM, leaving `headroom`
    free, after reserving two blocks for the staging buffers of the rest."""
    allowed = min(pin_fraction * free_ram, free_ram - headroom) - 2 * store.block_nbytes
    if allowed <= 0:
        return 0
    return min(streamed, int(allowed // store.block_nbytes))


@dataclass
class _Slot:
    idx: int
    buf: torch.Tensor  # uint8 [block_nbytes] on the device
    weights: BlockWeights  # typed views of buf
    state: int = FREE
    block: Optional[int] = None
    issued: threading.Event = field(default_factory=threading.Event)  # the copy of `block` has been issued (or done)


class _Engine:
    """The native copy engine of one provider (CUDA), or plain copies (CPU mode)."""

    def __init__(self, device: torch.device, n_slots: int, staging: int, block_nbytes: int):
        self.device, self.nbytes, self.handle = device, block_nbytes, None
        if device.type == "cuda":
            h = ctypes.c_void_p()
            _lib.check(_lib.lib().h3b_streamer_create(device.index, n_slots, staging, block_nbytes,
                                                      min(16, os.cpu_count() or 8), ctypes.byref(h)), "streamer")
            self.handle = h.value

    def copy(self, slot: _Slot, src: torch.Tensor, kind: str, transfer) -> None:
        if self.handle is None:
            (transfer or (lambda d, s, nb: d.copy_(s)))(slot.buf, src, False)
            return
        L = _lib.lib()
        if transfer is not None:  # a caller-supplied copy, run on the engine's copy stream between begin and end
            _lib.check(L.h3b_streamer_begin(self.handle, slot.idx), "streamer")
            with torch.cuda.stream(torch.cuda.ExternalStream(L.h3b_streamer_stream(self.handle), device=self.device)):
                transfer(slot.buf, src, kind != "pageable")
            _lib.check(L.h3b_streamer_end(self.handle, slot.idx, self.nbytes), "streamer")
            return
        mode = _lib.COPY_DIRECT if kind in _PAGE_LOCKED else (_lib.COPY_STAGED if kind == "staged" else _lib.COPY_PAGEABLE)
        _lib.check(L.h3b_streamer_copy(self.handle, slot.idx, slot.buf.data_ptr(), src.data_ptr(), self.nbytes, mode),
                   "streamer copy")

    def acquire(self, slot: _Slot) -> None:
        if self.handle is not None:
            _lib.check(_lib.lib().h3b_streamer_acquire(self.handle, slot.idx, _lib.stream_ptr(self.device)),
                       "streamer acquire")

    def release(self, slot: _Slot) -> None:
        if self.handle is not None:
            _lib.check(_lib.lib().h3b_streamer_release(self.handle, slot.idx, _lib.stream_ptr(self.device)),
                       "streamer release")

    def wait(self, slot: _Slot, timeout: float) -> None:
        if self.handle is not None:
            _lib.check(_lib.lib().h3b_streamer_wait(self.handle, slot.idx, max(0.0, timeout)), "streamer wait")

    def close(self) -> None:
        if self.handle is not None:
            _lib.lib().h3b_streamer_destroy(self.handle)
            self.handle = None


class StreamingProvider:
    """BlockProvider over an H3TFile (use as a context manager, or call close())."""

    def __init__(self, store: H3TFile, device: Union[str, torch.device] = "cuda", resident: Union[int, str] = "auto",
                 prefetch: int = 2, pin: Union[bool, str] = "auto", ring: int = 3, *, reserve_bytes: int = 1536 << 20,
                 free_vram_bytes: Optional[int] = None, pin_fraction: float = 0.5, ram_headroom_bytes: int = 4 * _GIB,
                 pin_blocks: Optional[int] = None, pin_mode: str = "auto",
                 transfer: Optional[Callable[[torch.Tensor, torch.Tensor, bool], None]] = None,
                 wait_timeout: float = 600.0):
        if ring < 1 or prefetch < 0 or pin not in (True, False, "auto") or pin_mode not in ("auto", "register", "copy", "stage"):
            raise ValueError("ring >= 1, prefetch >= 0, pin in (True, False, 'auto'), pin_mode in ('auto', 'register', 'copy', 'stage')")
        if resident != "auto" and not (isinstance(resident, int) and resident >= 0):
            raise ValueError("resident must be 'auto' or a non-negative int")
        dev = torch.device(device)
        if dev.type == "cuda" and dev.index is None:
            dev = torch.device("cuda", torch.cuda.current_device())
        self.store, self.device, self.n_blocks = store, dev, store.n_blocks
        self._cuda = dev.type == "cuda"
        self._prefetch, self._timeout, self._transfer = prefetch, wait_timeout, transfer
        self._lock = threading.Condition()
        self._resident: Dict[int, Tuple[torch.Tensor, BlockWeights]] = {}
        self._streamed: List[int] = []
        self._where: Dict[int, int] = {}  # streamed block -> its position j (slot j % ring)
        self._slots: List[_Slot] = []
        self._host: Dict[int, torch.Tensor] = {}  # streamed block -> its page-locked host source
        self._kind: Dict[int, str] = {}  # streamed block -> registered / pinned / staged / pageable
        self._locked: List[int] = []  # host pointers this provider page-locked (unlocked at close)
        self._engine: Optional[_Engine] = None
        self._jobs: "queue.Queue[Optional[Tuple[_Slot, int]]]" = queue.Queue()
        self._copier: Optional[threading.Thread] = None
        self._inline = False
        self._last = -1  # position of the last acquired streamed block in this forward (-1: the forward's start)
        self._forward = self._closed = False
        self._error: Optional[BaseException] = None
        self._st = self._zero_stats()
        self._plan: Dict[str, object] = {}
        _LIVE.add(self)
        try:
            n_res = self._choose_resident(resident, ring, reserve_bytes, free_vram_bytes)
            self._setup(n_res, ring)
            if self._streamed:
                self._plan_host(pin, pin_mode, pin_fraction, ram_headroom_bytes, pin_blocks)
                self._start()
        except BaseException:
            self.close()
            raise

    @staticmethod
    def _zero_stats() -> Dict[str, float]:
        return dict(acquires=0, waits=0, wait_s=0.0, copies=0, bytes=0, busy_s=0.0)

    # ------------------------------------------------------------------ construction
    def _choose_resident(self, resident, ring, reserve, free_vram) -> int:
        if resident != "auto":
            return min(int(resident), self.n_blocks)
        if free_vram is None:
            free_vram = torch.cuda.mem_get_info(self.device)[0] if self._cuda else free_ram_bytes() // 2
        return plan_residency(self.store, free_vram, reserve + (_CUDA_MARGIN if self._cuda else 0), ring)

    def _new_buffer(self) -> torch.Tensor:
        return torch.empty(self.store.block_nbytes, dtype=torch.uint8, device=self.device)

    def _setup(self, n_resident: int, ring: int, auto_shrink: bool = False) -> None:
        """Resident blocks [0, n_resident) on the device (copied from their host source) and min(ring, streamed) slots."""
        st = self.store
        for b in range(n_resident):
            if b in self._resident:
                continue
            try:
                buf = self._new_buffer()
            except torch.cuda.OutOfMemoryError:
                if auto_shrink:
                    n_resident = b
                    break
                raise
            buf.copy_(self._host.get(b, st.block_tensor(b)))
            self._resident[b] = (buf, st.block_weights_from(buf))
        for b in [b for b in self._resident if b >= n_resident]:
            del self._resident[b]
        self._streamed = list(range(n_resident, self.n_blocks))
        self._where = {b: j for j, b in enumerate(self._streamed)}
        self._slots = []
        for k in range(min(ring, len(self._streamed))):
            try:
                buf = self._new_buffer()
            except torch.cuda.OutOfMemoryError as e:
                raise torch.cuda.OutOfMemoryError(
                    f"cannot allocate streaming slot {k + 1} of {min(ring, len(self._streamed))} "
                    f"({st.block_nbytes / 2**20:.0f} MiB): lower resident/ring or free VRAM") from e
            self._slots.append(_Slot(k, buf, st.block_weights_from(buf)))

    def _page_lock(self, t: torch.Tensor, read_only: bool) -> bool:
        L = _lib.lib()
        if L.h3b_host_register(t.data_ptr(), t.numel(), int(read_only)) != 0:
            self._plan["register_error" if read_only else "pin_error"] = (L.h3b_last_error() or b"").decode(errors="replace")
            return False
        self._locked.append(t.data_ptr())
        return True

    def _lock_block(self, b: int, allow_copy: bool) -> bool:
        """Page-lock block b's host source: the file mapping in place (zero copy), else -- when allowed -- a page-locked
        copy of the block.  Returns whether the block is now page-locked."""
        if self._kind.get(b) in _PAGE_LOCKED:
            return True
        view = self.store.block_tensor(b)
        if self._page_lock(view, True):
            self._host[b], self._kind[b] = view, "registered"
            return True
        if not allow_copy:
            return False
        copy = torch.empty(self.store.block_nbytes, dtype=torch.uint8)
        if not self._page_lock(copy, False):
            return False
        copy.copy_(view)
        self._host[b], self._kind[b] = copy, "pinned"
        return True

    def _plan_host(self, pin, pin_mode, pin_fraction, headroom, pin_blocks) -> None:
        S = self._streamed
        if not self._cuda:
            self._kind = {b: "pageable" for b in S}
            return
        if pin is False or pin_mode == "stage":
            budget = 0
        elif pin is True:
            budget = len(S)
        elif pin_blocks is not None:
            budget = max(0, min(len(S), int(pin_blocks)))
        else:
            ram = free_ram_bytes()
            self._plan["ram_available_gib"] = round(ram / _GIB, 2)
            budget = plan_pinned_blocks(self.store, len(S), ram, pin_fraction, headroom)
        self._plan["pinned_wanted"] = budget
        for b in S[:budget]:
            if pin_mode == "copy":
                ok = self._copy_lock(b)
            else:
                ok = self._lock_block(b, allow_copy=pin_mode == "auto")
            if not ok:
                break
        for b in S:
            self._kind.setdefault(b, "pageable" if pin is False else "staged")

    def _copy_lock(self, b: int) -> bool:
        copy = torch.empty(self.store.block_nbytes, dtype=torch.uint8)
        if not self._page_lock(copy, False):
            return False
        copy.copy_(self.store.block_tensor(b))
        self._host[b], self._kind[b] = copy, "pinned"
        return True

    def _start(self) -> None:
        """Create the engine and pick the issue mode (inline when every source is page-locked and no hook is set)."""
        staging = 2 if self._cuda and any(self._kind[b] == "staged" for b in self._streamed) else 0
        self._engine = _Engine(self.device, len(self._slots), staging, self.store.block_nbytes)
        self._inline = self._cuda and self._transfer is None and all(self._kind[b] in _PAGE_LOCKED for b in self._streamed)
        self._plan["issue"] = "inline" if self._inline else "worker"
        if not self._inline:
            self._jobs = queue.Queue()
            self._copier = threading.Thread(target=self._copier_main, name="h3b-stream", daemon=True)
            self._copier.start()
        with self._lock:
            self._schedule()

    # ------------------------------------------------------------------ copies
    def _source(self, b: int) -> torch.Tensor:
        return self._host[b] if b in self._host else self.store.block_tensor(b)

    def _do_copy(self, slot: _Slot, b: int) -> None:
        t0 = time.perf_counter()
        self._engine.copy(slot, self._source(b), self._kind[b], self._transfer)
        with self._lock:
            self._st["copies"] += 1
            self._st["bytes"] += self.store.block_nbytes
            self._st["busy_s"] += time.perf_counter() - t0
            if slot.block == b and slot.state == PENDING:
                slot.state = READY
            slot.issued.set()
            self._lock.notify_all()

    def _copier_main(self) -> None:
        with torch.inference_mode():  # slot buffers made under inference mode are written under it
            if self._cuda:
                torch.cuda.set_device(self.device)
            while True:
                job = self._jobs.get()
                if job is None:
                    return
                try:
                    self._do_copy(*job)
                except BaseException as e:  # reported by the next acquire()
                    with self._lock:
                        self._error = e
                        job[0].issued.set()
                        self._lock.notify_all()
                    return

    def _refill(self, slot: _Slot, b: int) -> None:
        """Point `slot` at block b and queue (or, inline, issue) its copy.  Called with the lock held."""
        slot.block, slot.state = b, PENDING
        slot.issued.clear()
        if self._inline:
            self._lock.release()
            try:
                self._do_copy(slot, b)
            except BaseException as e:
                self._lock.acquire()
                self._error = e
                raise
            self._lock.acquire()
        else:
            self._jobs.put((slot, b))

    def _window(self) -> List[int]:
        """The streamed blocks wanted next: the `prefetch` after the last acquired one, cyclically."""
        S = self._streamed
        return [S[(self._last + 1 + k) % len(S)] for k in range(min(self._prefetch, len(S)))]

    def _schedule(self) -> None:
        """Queue copies for the lookahead window into slots whose block is no longer needed.  Lock held."""
        if not self._slots or self._closed or self._error is not None:
            return
        R = len(self._slots)
        window = self._window()
        wanted = set(window)
        for b in window:
            slot = self._slots[self._where[b] % R]
            if slot.block == b or slot.state in (ACQUIRED, PENDING):
                continue  # already there (or on its way), or the slot's current block is still in use
            if slot.block in wanted:
                continue  # the slot holds a block of the window that is needed sooner (prefetch >= ring)
            self._refill(slot, b)

    # ------------------------------------------------------------------ BlockProvider
    def _raise_if_broken(self) -> None:
        if self._closed:
            raise RuntimeError("StreamingProvider is closed")
        if self._error is not None:
            raise RuntimeError(f"H3 streaming worker failed: {self._error!r}") from self._error

    def begin_forward(self) -> None:
        if self._forward:  # the previous forward never reached end_forward (an exception): recover first
            self.end_forward()
        self._forward = True

    def acquire(self, i: int) -> BlockWeights:
        if i < 0 or i >= self.n_blocks:
            raise IndexError(f"block {i} out of range [0, {self.n_blocks})")
        if self._closed:
            raise RuntimeError("StreamingProvider is closed")
        if i in self._resident:
            return self._resident[i][1]
        if not self._slots:
            raise RuntimeError("H3 streaming provider is parked (it holds no device memory); resize() it before a forward")
        t0 = time.perf_counter()
        waited = False
        with self._lock:
            self._raise_if_broken()
            slot = self._slots[self._where[i] % len(self._slots)]
            if slot.block == i and slot.state == ACQUIRED:
                raise RuntimeError(f"block {i} is already acquired")
            if slot.block != i:
                if slot.state == ACQUIRED:
                    raise RuntimeError(f"all {len(self._slots)} ring slots are held; release() a block before "
                                       f"acquiring block {i} (ring too small?)")
                while slot.state == PENDING:  # a prefetch of another block is on its way into this slot
                    waited = True
                    self._wait_locked(slot, t0, i)
                self._refill(slot, i)
            while slot.state == PENDING:
                waited = True
                self._wait_locked(slot, t0, i)
            self._raise_if_broken()
            slot.state = ACQUIRED
            self._last = self._where[i]
            self._st["acquires"] += 1
            if waited:
                self._st["waits"] += 1
                self._st["wait_s"] += time.perf_counter() - t0
        self._engine.acquire(slot)  # the compute stream waits for the copy (device side)
        with self._lock:
            self._schedule()
        return slot.weights

    def _wait_locked(self, slot: _Slot, t0: float, i: int) -> None:
        left = self._timeout - (time.perf_counter() - t0)
        if left <= 0:
            raise TimeoutError(f"timed out after {self._timeout:.0f}s waiting for block {i}: {self._dump()}")
        self._lock.wait(min(left, 0.5))
        self._raise_if_broken()

    def release(self, i: int) -> None:
        if i in self._resident:
            return
        with self._lock:
            slot = self._slots[self._where[i] % len(self._slots)] if self._slots and i in self._where else None
            if slot is None or slot.block != i or slot.state != ACQUIRED:
                raise RuntimeError(f"release({i}) but block {i} is not acquired")
            self._engine.release(slot)  # kernels reading the slot are already queued on the compute stream
            slot.state = IDLE
            self._schedule()

    def end_forward(self) -> None:
        """Close the forward (also after an exception): slots still held are released behind the compute stream and the
        lookahead restarts at the first streamed block, prefetching it for the next forward."""
        with self._lock:
            for s in self._slots:
                if s.state == ACQUIRED:
                    if self._engine is not None and not self._closed:
                        self._engine.release(s)
                    s.state = IDLE
            self._last, self._forward = -1, False
            if not self._closed:
                self._schedule()

    # ------------------------------------------------------------------ residency changes between forwards
    def device_bytes(self) -> int:
        return (len(self._resident) + len(self._slots)) * self.store.block_nbytes

    def _stop_copier(self) -> None:
        if self._copier is not None:
            self._jobs.put(None)
            if self._copier is not threading.current_thread():
                self._copier.join(timeout=120)
            self._copier = None

    def resize(self, resident: int, ring: int = 3, *, lock_host: bool = True, ram_headroom_bytes: int = 3 * _GIB) -> int:
        """Change the resident prefix and the ring size between forwards, keeping what the host side already holds.
        resize(0, 0) parks the provider (no device memory).  Returns the device bytes now held."""
        if self._closed:
            raise RuntimeError("StreamingProvider is closed")
        if self._forward:
            raise RuntimeError("resize() during a forward")
        self._stop_copier()
        if self._cuda:
            torch.cuda.synchronize(self.device)
        if self._engine is not None:
            self._engine.close()
            self._engine = None
        with self._lock:
            self._slots, self._last = [], -1
        keep = max(0, min(int(resident), self.n_blocks))
        if self._cuda:
            for b in sorted(self._resident):  # blocks that start streaming keep (or get) a page-locked host source
                if b >= keep and lock_host:
                    self._lock_if_room(b, ram_headroom_bytes)
            for b in [b for b in self._resident if b >= keep]:
                del self._resident[b]
            torch.cuda.empty_cache()
        self._setup(keep, max(0, ring), auto_shrink=True)
        if self._streamed:
            if lock_host and self._cuda:
                for b in self._streamed:
                    if not self._lock_if_room(b, ram_headroom_bytes):
                        break
            for b in self._streamed:
                if self._kind.get(b) not in _PAGE_LOCKED:
                    self._kind[b] = "staged" if self._cuda else "pageable"
            if self._slots:
                self._start()
        return self.device_bytes()

    def _lock_if_room(self, b: int, headroom: int) -> bool:
        if self._kind.get(b) in _PAGE_LOCKED:
            return True
        try:
            room = free_ram_bytes() - self.store.block_nbytes >= headroom
        except RuntimeError:
            room = False
        return room and self._lock_block(b, allow_copy=False)

    @property
    def parked(self) -> bool:
        return bool(self._streamed) and not self._slots

    # ------------------------------------------------------------------ introspection / lifecycle
    def buffer_of(self, i: int) -> Optional[torch.Tensor]:
        """The device buffer holding block i, if it is resident or its copy into a slot has been issued."""
        if i in self._resident:
            return self._resident[i][0]
        with self._lock:
            if not self._slots or i not in self._where:
                return None
            s = self._slots[self._where[i] % len(self._slots)]
            return s.buf if s.block == i and s.state in (READY, IDLE, ACQUIRED) else None

    def wait_prefetch(self, timeout: float = 60.0) -> None:
        """Block until every scheduled copy has been issued and has landed."""
        t_end = time.perf_counter() + timeout
        with self._lock:
            while any(s.state == PENDING for s in self._slots) and self._error is None:
                left = t_end - time.perf_counter()
                if left <= 0:
                    raise TimeoutError(f"prefetch did not settle: {self._dump()}")
                self._lock.wait(min(left, 0.5))
            self._raise_if_broken()
            landed = [s for s in self._slots if s.state in (READY, IDLE)]
        for s in landed:
            self._engine.wait(s, t_end - time.perf_counter())

    def _dump(self) -> str:
        slots = ", ".join(f"{s.idx}:{_STATE[s.state]}:{s.block}" for s in self._slots)
        return f"slots {slots}; last={self._last} window={self._window() if self._slots else []}"

    def stats(self) -> Dict[str, object]:
        with self._lock:
            kinds: Dict[str, int] = {}
            for k in self._kind.values():
                kinds[k] = kinds.get(k, 0) + 1
            return dict(self._st, resident=len(self._resident), streamed=len(self._streamed), slots=len(self._slots),
                        host_kinds=kinds, gpu_bytes=self.device_bytes(),
                        locked_host_bytes=len(self._locked) * self.store.block_nbytes, plan=dict(self._plan),
                        state=self._dump())

    def reset_stats(self) -> None:
        with self._lock:
            self._st = self._zero_stats()

    def close(self) -> None:
        if self._closed:
            return
        with self._lock:
            self._closed = True
            self._lock.notify_all()
        self._stop_copier()
        if self._cuda:
            try:
                torch.cuda.synchronize(self.device)
            except Exception:
                pass
        if self._engine is not None:
            self._engine.close()
            self._engine = None
        if self._locked:
            L = _lib.lib()
            for p in self._locked:
                L.h3b_host_unregister(p)
        self._locked, self._slots, self._resident, self._host, self._kind = [], [], {}, {}, {}
        if self._cuda:
            torch.cuda.empty_cache()

    def __enter__(self) -> "StreamingProvider":
        return self

    def __exit__(self, *exc) -> None:
        self.close()


_LIVE: "weakref.WeakSet[StreamingProvider]" = weakref.WeakSet()


@atexit.register
def _close_all() -> None:
    """Close providers left open, so no copier thread is inside CUDA when the interpreter exits."""
    for p in list(_LIVE):
        try:
            p.close()
        except Exception:
            pass
