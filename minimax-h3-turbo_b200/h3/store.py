"""Reader of the h3t weight store (the writer is writer.py).

An h3t file is a safetensors file laid out so that a DiT block can move host -> device in ONE copy and be used in place:
globals first, then blocks 0..N-1, each block one BLOCK_ALIGN-aligned byte range with the same tensor layout, every
tensor on a TENSOR_ALIGN boundary, the gaps filled by explicit `__pad.<n>` U8 tensors so the safetensors index covers
every byte.  The format (header, metadata keys, alignments, ordering) is the reference's (h3turbo/h3/store.py:1-60,
writer.py:137-262), so files written by either implementation are read by both.

Reading is a validation pass over the header followed by a read-only memory map of the file: `block_tensor(i)` is the
block's bytes in the mapping (the source of a device copy), and `block_weights_from(buf)` turns any 1-D uint8 buffer
holding a block (a device slot, a pinned host copy) into zero-copy typed `BlockWeights` views.
"""
from __future__ import annotations

import hashlib
import json
import math
import mmap
import os
import re
import struct
import sys
import warnings
from typing import Callable, Dict, List, NamedTuple, Optional, Sequence, Tuple

import numpy as np
import torch

from .config import H3Config
from .types import BlockWeights, W4A8Weight, Weight

if sys.byteorder != "little":  # pragma: no cover -- safetensors data is little-endian
    raise ImportError("h3t files are little-endian")

# ---- format constants (shared with the reference's files)
FORMAT = "h3turbo-h3"
VERSION = 1
TENSOR_ALIGN = 256  # tensor starts: the kernels' vector loads and TMA descriptors need 16 B; 256 leaves room
BLOCK_ALIGN = 4096  # block starts and sizes: page-aligned, so a block can be page-locked where it lies
PAD_PREFIX = "__pad."
LINEARS = ("attn.qkv_proj", "attn.out_proj", "mlp.fc1", "mlp.fc2")
QUANT_PARTS = ("weight", "weight_s_rel", "weight_s_channel", "weight_codebook", "comfy_quant")
BLOCK_RE = re.compile(r"^blocks\.(\d+)\.(.+)$")
HEADER_LIMIT = 100_000_000  # safetensors' own cap on the JSON header

# safetensors dtype name -> (torch dtype, bytes per element)
_ST = (("F64", torch.float64), ("F32", torch.float32), ("F16", torch.float16), ("BF16", torch.bfloat16),
       ("I64", torch.int64), ("I32", torch.int32), ("I16", torch.int16), ("I8", torch.int8), ("U8", torch.uint8),
       ("BOOL", torch.bool), ("F8_E4M3", torch.float8_e4m3fn), ("F8_E5M2", torch.float8_e5m2))
_TORCH_OF = {name: dt for name, dt in _ST}
_SIZE_OF = {name: torch.empty((), dtype=dt).element_size() for name, dt in _ST}
_NAME_OF = {dt: name for name, dt in _ST}


class H3TError(ValueError):
    """Not a valid h3t container, or an inconsistent write request."""


def itemsize(dtype: str) -> int:
    if dtype not in _SIZE_OF:
        raise H3TError(f"unsupported safetensors dtype {dtype!r}")
    return _SIZE_OF[dtype]


def torch_dtype(dtype: str) -> torch.dtype:
    itemsize(dtype)
    return _TORCH_OF[dtype]


def st_dtype(t: torch.dtype) -> str:
    if t not in _NAME_OF:
        raise H3TError(f"torch dtype {t} has no safetensors name")
    return _NAME_OF[t]


def nbytes_of(dtype: str, shape: Sequence[int]) -> int:
    return itemsize(dtype) * math.prod(shape)


def align(x: int, a: int) -> int:
    return (x + a - 1) // a * a


class Header(NamedTuple):
    tensors: Dict[str, dict]  # name -> {"dtype", "shape", "data_offsets"} (offsets relative to the data section)
    meta: Dict[str, str]
    data_start: int
    file_size: int
    raw: bytes  # the JSON bytes as stored (for fingerprints)


class BlockEntry(NamedTuple):
    name: str  # block-relative tensor name
    dtype: str
    shape: Tuple[int, ...]
    offset: int  # byte offset inside the block
    nbytes: int


class TensorInfo(NamedTuple):
    dtype: str
    shape: Tuple[int, ...]
    start: int  # absolute file offset
    nbytes: int


def _entry_fields(name: str, e) -> Tuple[str, list, int, int]:
    try:
        (a, b), dtype, shape = e["data_offsets"], e["dtype"], e["shape"]
        return dtype, list(shape), int(a), int(b)
    except (KeyError, TypeError, ValueError):
        raise H3TError(f"malformed header entry for {name!r}") from None


def read_header(path) -> Header:
    """The safetensors header of `path`, checked for internal consistency (every entry inside the data section, with
    the size its dtype and shape imply); no tensor data is read."""
    size = os.path.getsize(path)
    with open(path, "rb") as f:
        prefix = f.read(8)
        if len(prefix) != 8:
            raise H3TError(f"{path}: file too small to be safetensors ({size} bytes)")
        hlen = struct.unpack("<Q", prefix)[0]
        if hlen > HEADER_LIMIT or hlen + 8 > size:
            raise H3TError(f"{path}: implausible safetensors header size {hlen} (file is {size} bytes)")
        raw = f.read(hlen)
    if raw[:1] != b"{" and not raw.lstrip(b" ").startswith(b"{"):
        raise H3TError(f"{path}: safetensors header does not start with '{{'")
    try:
        doc = json.loads(raw)
    except ValueError as e:
        raise H3TError(f"{path}: unreadable safetensors header: {e}") from None
    meta = doc.pop("__metadata__", None) or {}
    span = size - 8 - hlen
    for name, e in doc.items():
        try:
            dtype, shape, a, b = _entry_fields(name, e)
        except H3TError as err:
            raise H3TError(f"{path}: {err}") from None
        if a < 0 or b < a or b > span:
            raise H3TError(f"{path}: tensor {name!r} range [{a}, {b}) is outside the data section ({span} bytes); "
                           "truncated file?")
        if dtype in _SIZE_OF and nbytes_of(dtype, shape) != b - a:
            raise H3TError(f"{path}: tensor {name!r} declares {b - a} bytes but {dtype}{shape} needs "
                           f"{nbytes_of(dtype, shape)}")
    return Header(doc, meta, 8 + hlen, size, raw)


def header_sha256(path) -> str:
    return hashlib.sha256(read_header(path).raw).hexdigest()


def quant_linear_names(names) -> List[str]:
    """The linears of LINEARS stored in W4A8 form (they carry a codebook)."""
    have = set(names)
    return [lin for lin in LINEARS if lin + ".weight_codebook" in have]


def typed_view(buf: torch.Tensor, off: int, dtype: str, shape: Sequence[int]) -> torch.Tensor:
    """Zero-copy `dtype`/`shape` tensor over bytes [off, off + size) of a 1-D uint8 tensor (on any device)."""
    raw = buf.narrow(0, off, nbytes_of(dtype, shape))
    tdt = torch_dtype(dtype)
    return (raw if tdt == torch.uint8 else raw.view(tdt)).view(tuple(shape))


def build_block_weights(get: Callable[[str], torch.Tensor], has: Callable[[str], bool], group: int, convrot: int,
                        adaln: bool = True) -> BlockWeights:
    """BlockWeights from block-relative names: a linear with a codebook becomes a W4A8Weight, any other a dense
    matrix."""

    def linear(prefix: str) -> Weight:
        if not has(prefix + ".weight_codebook"):
            return get(prefix + ".weight")
        parts = [get(f"{prefix}.{p}") for p in ("weight", "weight_s_rel", "weight_s_channel", "weight_codebook")]
        return W4A8Weight(*parts, group, convrot)

    mod = adaln and has("adaln_proj.linear.weight")
    return BlockWeights(
        qkv=linear("attn.qkv_proj"), out=linear("attn.out_proj"), fc1=linear("mlp.fc1"), fc2=linear("mlp.fc2"),
        norm1=get("norm1.weight"), norm2=get("norm2.weight"), q_norm=get("attn.q_norm.weight"),
        k_norm=get("attn.k_norm.weight"), adaln_w=get("adaln_proj.linear.weight") if mod else None,
        adaln_b=get("adaln_proj.linear.bias") if mod else None)


class _Layout(NamedTuple):
    """What the metadata says about the block area, parsed."""

    cfg: H3Config
    n_blocks: int
    block_nbytes: int
    blocks_start: int
    entries: List[BlockEntry]
    ranges: list
    quant: dict


def _parse_meta(path: str, m: Dict[str, str]) -> _Layout:
    if m.get("format") != FORMAT:
        raise H3TError(f"{path}: not an h3t file (metadata format={m.get('format')!r}, expected {FORMAT!r})")
    if str(m.get("version")) != str(VERSION):
        raise H3TError(f"{path}: unsupported h3t version {m.get('version')!r} (this reader supports {VERSION})")
    try:
        entries = [BlockEntry(str(n), str(d), tuple(int(v) for v in s), int(o), int(b))
                   for n, d, s, o, b in json.loads(m["block_layout"])]
        return _Layout(H3Config.from_json(m["config"]), int(m["n_blocks"]), int(m["block_nbytes"]),
                       int(m["blocks_start"]), entries, json.loads(m["block_ranges"]), json.loads(m.get("quant") or "{}"))
    except (KeyError, ValueError, TypeError, IndexError) as e:
        raise H3TError(f"{path}: corrupt h3t metadata: {e!r}") from None


def _check_layout(path: str, h: Header, lay: _Layout) -> None:
    """Every invariant the zero-copy block views rely on, checked once at open."""
    n, bnb, b0 = lay.n_blocks, lay.block_nbytes, lay.blocks_start
    if n < 1 or n != lay.cfg.layers:
        raise H3TError(f"{path}: n_blocks={n} disagrees with config.layers={lay.cfg.layers}")
    if any(v % BLOCK_ALIGN for v in (h.data_start, b0, bnb)):
        raise H3TError(f"{path}: data/block offsets are not {BLOCK_ALIGN}-aligned")
    need = h.data_start + b0 + n * bnb
    if need != h.file_size:
        raise H3TError(f"{path}: file is {h.file_size} bytes, layout needs exactly {need} (truncated or trailing data?)")
    if [list(r) for r in lay.ranges] != [[b0 + i * bnb, b0 + (i + 1) * bnb] for i in range(n)]:
        raise H3TError(f"{path}: block_ranges disagree with blocks_start/block_nbytes for {n} blocks")
    # the header must list every block's tensors exactly where the shared layout puts them
    for i in range(n):
        base = b0 + i * bnb
        for e in lay.entries:
            want = {"dtype": e.dtype, "shape": list(e.shape), "data_offsets": [base + e.offset, base + e.offset + e.nbytes]}
            got = h.tensors.get(f"blocks.{i}.{e.name}")
            if got is None or {k: (list(v) if k != "dtype" else v) for k, v in got.items() if k in want} != want:
                raise H3TError(f"{path}: blocks.{i}.{e.name} does not match the block layout")
    # the index covers the data section without holes or overlaps; real tensors are aligned
    spans = sorted((e["data_offsets"][0], e["data_offsets"][1], name) for name, e in h.tensors.items())
    end = 0
    for a, b, name in spans:
        if a != end:
            raise H3TError(f"{path}: hole or overlap before {name!r}")
        if a % TENSOR_ALIGN and not name.startswith(PAD_PREFIX):
            raise H3TError(f"{path}: {name!r} starts at {a}, not {TENSOR_ALIGN}-aligned")
        end = b
    if end != h.file_size - h.data_start:
        raise H3TError(f"{path}: tensors cover {end} bytes, data section has {h.file_size - h.data_start}")
    names = {e.name for e in lay.entries}
    for lin in quant_linear_names(names):
        gone = [p for p in QUANT_PARTS if f"{lin}.{p}" not in names]
        if gone:
            raise H3TError(f"{path}: W4A8 linear {lin} lacks {gone}")


class H3TFile:
    """A read-only memory-mapped h3t file.  Accessors return zero-copy views of the mapping; close the file only after
    the providers and page-locked ranges derived from it are closed."""

    def __init__(self, path):
        self.path = os.fspath(path)
        h = read_header(self.path)
        lay = _parse_meta(self.path, h.meta)
        _check_layout(self.path, h, lay)
        self.cfg, self.n_blocks, self.block_nbytes, self.blocks_start = lay.cfg, lay.n_blocks, lay.block_nbytes, lay.blocks_start
        self.block_layout, self.quant, self.meta = lay.entries, lay.quant, dict(h.meta)
        self.data_start, self.file_size = h.data_start, h.file_size
        self.source_name = h.meta.get("source_name", "")
        self.source_size = int(h.meta.get("source_size") or 0)
        self.quant_group = int(lay.quant.get("group_size", lay.cfg.quant_group))
        self.quant_convrot = int(lay.quant.get("convrot_groupsize", lay.cfg.quant_convrot))
        self._lay = {e.name: e for e in lay.entries}
        self._tensors: Dict[str, TensorInfo] = {}
        for name, e in h.tensors.items():
            if not name.startswith(PAD_PREFIX):
                a, b = e["data_offsets"]
                self._tensors[name] = TensorInfo(e["dtype"], tuple(e["shape"]), h.data_start + a, b - a)
        with open(self.path, "rb") as fh:
            self._mm: Optional[mmap.mmap] = mmap.mmap(fh.fileno(), 0, access=mmap.ACCESS_READ)
        self._np: Optional[np.ndarray] = np.frombuffer(self._mm, dtype=np.uint8)
        with warnings.catch_warnings():  # torch warns that the buffer is not writable; nothing writes through it
            warnings.simplefilter("ignore")
            self._u8: Optional[torch.Tensor] = torch.frombuffer(self._mm, dtype=torch.uint8)

    # ---- raw bytes
    def _open(self) -> None:
        if self._mm is None:
            raise ValueError("H3TFile is closed")

    def block_range(self, i: int) -> Tuple[int, int]:
        """Absolute file byte range of block i."""
        if i < 0 or i >= self.n_blocks:
            raise IndexError(f"block {i} out of range [0, {self.n_blocks})")
        start = self.data_start + self.blocks_start + i * self.block_nbytes
        return start, start + self.block_nbytes

    def block_bytes(self, i: int) -> np.ndarray:
        self._open()
        a, b = self.block_range(i)
        return self._np[a:b]

    def block_tensor(self, i: int) -> torch.Tensor:
        """Block i as a uint8 tensor over the mapping (the source of one host -> device copy)."""
        self._open()
        a, b = self.block_range(i)
        return self._u8[a:b]

    @property
    def block_layout_size(self) -> int:
        """Bytes of a block actually used by tensors (the rest up to block_nbytes is alignment)."""
        last = max(self.block_layout, key=lambda e: e.offset)
        return last.offset + last.nbytes

    # ---- typed access
    def keys(self) -> List[str]:
        return list(self._tensors)

    def info(self, name: str) -> TensorInfo:
        t = self._tensors.get(name)
        if t is None:
            raise KeyError(f"{name!r} is not in {self.path}")
        return t

    def tensor(self, name: str) -> torch.Tensor:
        self._open()
        t = self.info(name)
        return typed_view(self._u8, t.start, t.dtype, t.shape)

    def block_weights_from(self, buf: torch.Tensor) -> BlockWeights:
        """Typed zero-copy views of a block held in `buf`: a 1-D uint8 tensor of block_nbytes on any device."""
        if buf.dim() != 1 or buf.dtype != torch.uint8 or buf.numel() != self.block_nbytes:
            raise ValueError(f"expected a 1-D uint8 buffer of {self.block_nbytes} bytes, got {tuple(buf.shape)} {buf.dtype}")
        lay = self._lay

        def get(rel: str) -> torch.Tensor:
            e = lay[rel]
            return typed_view(buf, e.offset, e.dtype, e.shape)

        return build_block_weights(get, lay.__contains__, self.quant_group, self.quant_convrot)

    def block_weights_cpu(self, i: int) -> BlockWeights:
        return self.block_weights_from(self.block_tensor(i))

    # ---- lifecycle
    def close(self) -> None:
        mm = self._mm
        if mm is None:
            return
        self._mm = self._np = self._u8 = None
        try:
            mm.close()
        except BufferError:  # views are still alive; the mapping is released with the last of them
            pass

    def __enter__(self) -> "H3TFile":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    def __del__(self) -> None:
        try:
            self.close()
        except Exception:
            pass

    def __repr__(self) -> str:
        return f"H3TFile({self.path!r}, blocks={self.n_blocks}, block={self.block_nbytes / 2**20:.1f} MiB)"


def __getattr__(name: str):
    """The writer's API is importable from this module too, as from the reference's store module."""
    if name in ("write_h3t", "TensorSource", "TorchSource", "LazySource", "as_source", "classify"):
        from . import writer

        return getattr(writer, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
