"""h3t store: writer -> reader round trip, layout invariants and rejection of damaged files (CPU only; the reference's
tests/test_h3_store.py checks the same properties of its own implementation)."""
import json
import os
import struct

import pytest
import torch

from minimax_h3_turbo_b200.h3 import store as st
from minimax_h3_turbo_b200.h3.config import H3Config
from minimax_h3_turbo_b200.h3.synth import synthetic_store_tensors
from minimax_h3_turbo_b200.h3.types import W4A8Weight
from minimax_h3_turbo_b200.h3.writer import write_h3t

CFG = H3Config(hidden=256, layers=3, refiner_layers=0, heads=2, head_dim=128, ffn=512, text_dim=64, video_channels=4,
               audio_channels=8, quant_group=16, quant_convrot=256)


@pytest.fixture(scope="module", params=["fp8", "fp16"])
def written(tmp_path_factory, request):
    fmt = request.param
    group = 16 if fmt == "fp8" else 128
    path = tmp_path_factory.mktemp("h3t") / f"tiny_{fmt}.h3t"
    tensors = synthetic_store_tensors(CFG, group=group, scale_dtype=fmt, seed=3)
    summary = write_h3t(path, CFG, tensors, quant={"format": "asym_w4a8_int8", "group_size": group, "convrot_groupsize": 256})
    ref = {k: (v.read() if hasattr(v, "read") else v) for k, v in tensors.items()}
    return path, summary, ref, group


def test_round_trip_is_bit_identical(written):
    path, summary, ref, group = written
    with st.H3TFile(path) as f:
        assert f.n_blocks == 3 and f.block_nbytes % st.BLOCK_ALIGN == 0 and f.quant_group == group
        for name, t in ref.items():
            got = f.tensor(name)
            assert got.dtype == t.dtype and got.shape == t.shape
            assert torch.equal(got.view(torch.uint8), t.contiguous().view(torch.uint8)), name
        for i in range(3):
            bw = f.block_weights_cpu(i)
            assert isinstance(bw.qkv, W4A8Weight) and bw.qkv.group_size == group
            assert torch.equal(bw.fc2.q, ref[f"blocks.{i}.mlp.fc2.weight"])
            assert bw.adaln_w is None
        assert os.path.getsize(path) == summary["file_size"]


def test_layout_alignment_and_contiguous_blocks(written):
    path = written[0]
    with st.H3TFile(path) as f:
        assert f.data_start % st.BLOCK_ALIGN == 0 and f.blocks_start % st.BLOCK_ALIGN == 0
        for e in f.block_layout:
            assert e.offset % st.TENSOR_ALIGN == 0
        for i in range(f.n_blocks):
            a, b = f.block_range(i)
            assert b - a == f.block_nbytes and a % st.BLOCK_ALIGN == 0
            assert f.block_tensor(i).numel() == f.block_nbytes
        assert f.tensor("video_patch_proj.weight").shape == (256, 16)


def test_block_views_into_a_device_style_buffer(written):
    path = written[0]
    with st.H3TFile(path) as f:
        buf = f.block_tensor(1).clone()
        bw = f.block_weights_from(buf)
        assert bw.qkv.q.data_ptr() - buf.data_ptr() == f._lay["attn.qkv_proj.weight"].offset
        with pytest.raises(ValueError, match="uint8 buffer"):
            f.block_weights_from(buf[:-1])


def test_damaged_files_are_rejected(written, tmp_path):
    path = written[0]
    raw = path.read_bytes()
    (tmp_path / "trunc.h3t").write_bytes(raw[:-4096])
    with pytest.raises(st.H3TError, match="truncated|outside"):
        st.H3TFile(tmp_path / "trunc.h3t")
    (n,) = struct.unpack("<Q", raw[:8])
    hdr = json.loads(raw[8:8 + n])
    hdr["__metadata__"]["format"] = "something-else"
    enc = json.dumps(hdr).encode()
    enc += b" " * (n - len(enc))
    (tmp_path / "fmt.h3t").write_bytes(raw[:8] + enc + raw[8 + n:])
    with pytest.raises(st.H3TError, match="not an h3t"):
        st.H3TFile(tmp_path / "fmt.h3t")
    (tmp_path / "tiny.h3t").write_bytes(b"\x01\x00")
    with pytest.raises(st.H3TError, match="too small"):
        st.H3TFile(tmp_path / "tiny.h3t")


def test_failed_write_leaves_no_file(tmp_path):
    tensors = synthetic_store_tensors(CFG, group=16, scale_dtype="fp8", seed=1, with_globals=False)
    tensors["blocks.2.norm1.weight"] = torch.zeros(7, dtype=torch.bfloat16)  # block 2 differs from block 0
    with pytest.raises(st.H3TError, match="block 0"):
        write_h3t(tmp_path / "bad.h3t", CFG, tensors)
    assert not (tmp_path / "bad.h3t").exists() and not (tmp_path / "bad.h3t.part").exists()


@pytest.mark.parametrize("case", ["fp8_g16", "fp16_g128"])
def test_writer_output_is_byte_identical_to_the_reference_writer(case, tmp_path):
    """tests/golden/h3t_golden.json holds the size and sha256 of the file the REFERENCE writer produced from these same
    seeded tensors (tests/golden/make_h3t_golden.py)."""
    import hashlib
    from pathlib import Path

    gold = json.loads((Path(__file__).resolve().parent / "golden" / "h3t_golden.json").read_text())[case]
    cfg = H3Config(hidden=256, layers=3, refiner_layers=0, heads=2, head_dim=128, ffn=512, text_dim=64, video_channels=4,
                   audio_channels=8, quant_group=gold["group"])
    path = tmp_path / f"{case}.h3t"
    write_h3t(path, cfg, synthetic_store_tensors(cfg, group=gold["group"], scale_dtype=gold["format"], seed=gold["seed"]))
    raw = path.read_bytes()
    assert len(raw) == gold["size"]
    assert hashlib.sha256(raw).hexdigest() == gold["sha256"]
