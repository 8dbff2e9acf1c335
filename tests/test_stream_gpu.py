"""StreamingProvider on a GPU: the native copy engine's bytes, device-side ordering and the W4A8 linear on streamed
weights (the reference's CUDA checks: device bytes == file, kernel ordering, pinned staging ring)."""
import pytest
import torch

from minimax_h3_turbo_b200 import _lib
from minimax_h3_turbo_b200.h3 import qlinear as ql
from minimax_h3_turbo_b200.h3 import stream as sm
from minimax_h3_turbo_b200.h3.config import H3Config
from minimax_h3_turbo_b200.h3.store import H3TFile
from minimax_h3_turbo_b200.h3.synth import synthetic_store_tensors
from minimax_h3_turbo_b200.h3.writer import write_h3t

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
CFG = H3Config(hidden=512, layers=6, refiner_layers=0, heads=4, head_dim=128, ffn=1024, text_dim=64, video_channels=4,
               audio_channels=8, quant_group=128)


@pytest.fixture(scope="module")
def store(tmp_path_factory):
    path = tmp_path_factory.mktemp("sgpu") / "s.h3t"
    write_h3t(path, CFG, synthetic_store_tensors(CFG, group=128, scale_dtype="fp16", seed=4),
              quant={"format": "asym_w4a8_int8", "group_size": 128, "convrot_groupsize": 256})
    f = H3TFile(path)
    yield f
    f.close()


def _expected(store):
    return [store.block_tensor(i).to(DEV) for i in range(store.n_blocks)]


@pytest.mark.parametrize("pin,pin_mode", [(True, "register"), (True, "copy"), ("auto", "stage"), (False, "auto")])
def test_device_bytes_equal_the_file_in_every_host_mode(store, pin, pin_mode):
    want = _expected(store)
    with sm.StreamingProvider(store, DEV, resident=1, ring=2, prefetch=2, pin=pin, pin_mode=pin_mode) as p:
        for _ in range(2):
            p.begin_forward()
            for i in range(store.n_blocks):
                p.acquire(i)
                assert torch.equal(p.buffer_of(i), want[i]), (pin, pin_mode, i)
                p.release(i)
            p.end_forward()
        kinds = p.stats()["host_kinds"]
        issue = p.stats()["plan"]["issue"]
    assert issue == ("inline" if set(kinds) <= {"registered", "pinned"} else "worker"), (kinds, issue)
    if pin is False:
        assert set(kinds) == {"pageable"}
    elif pin_mode == "stage":
        assert set(kinds) == {"staged"}


def test_compute_stream_waits_for_a_slow_copy(store):
    """The copy stream is held back by a long GPU sleep before each copy; a kernel enqueued right after acquire() must
    still read the new block (acquire orders the compute stream after the copy, not the host)."""
    want = _expected(store)

    def slow(dst, src, nb):
        torch.cuda._sleep(20_000_000)  # ~10 ms on the copy stream
        dst.copy_(src, non_blocking=nb)

    sums = []
    with sm.StreamingProvider(store, DEV, resident=0, ring=2, prefetch=1, pin=True, transfer=slow) as p:
        p.begin_forward()
        for i in range(store.n_blocks):
            w = p.acquire(i)
            sums.append(w.fc1.q.view(torch.uint8).sum(dtype=torch.int64))
            p.release(i)
        p.end_forward()
        torch.cuda.synchronize()
    for i, s in enumerate(sums):
        assert s.item() == store.block_weights_cpu(i).fc1.q.view(torch.uint8).sum(dtype=torch.int64).item(), i
    del want


def test_linear_on_streamed_weights_equals_resident(store):
    x = torch.randn(96, CFG.hidden, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16).to(DEV)
    resident = [store.block_weights_cpu(i) for i in range(store.n_blocks)]
    outs_res = [ql.linear(x, w.qkv.to(DEV)) for w in resident]
    with sm.StreamingProvider(store, DEV, resident=0, ring=2, prefetch=2) as p:
        p.begin_forward()
        for i in range(store.n_blocks):
            w = p.acquire(i)
            assert torch.equal(ql.linear(x, w.qkv), outs_res[i])
            p.release(i)
        p.end_forward()
        st = p.stats()
    assert st["copies"] >= store.n_blocks and st["bytes"] >= store.n_blocks * store.block_nbytes


def test_engine_rejects_bad_slots():
    import ctypes

    L = _lib.lib()
    h = ctypes.c_void_p()
    _lib.check(L.h3b_streamer_create(torch.cuda.current_device(), 2, 0, 0, 4, ctypes.byref(h)), "create")
    try:
        assert L.h3b_streamer_acquire(h.value, 5, None) == _lib.ERR_ARG
        assert L.h3b_streamer_wait(h.value, -1, 1.0) == _lib.ERR_ARG
    finally:
        L.h3b_streamer_destroy(h.value)
