"""Write h3t stores (format in store.py): globals and token refiner first, then every block as one BLOCK_ALIGN-aligned
range with an identical layout, tensors TENSOR_ALIGN-aligned, explicit `__pad.*` gaps (writer.py:137-262 of the
reference produces the same byte format).  Writes go to `<dst>.part`, are fsync'ed and then renamed, so an interrupted
write never leaves a file that looks valid; peak memory is one chunk plus the header."""
from __future__ import annotations

import json
import os
import re
import struct
from typing import Callable, Dict, Iterable, Iterator, List, Mapping, Optional, Sequence, Tuple, Union

import torch

from .config import H3Config
from .store import (BLOCK_ALIGN, BLOCK_RE, FORMAT, PAD_PREFIX, TENSOR_ALIGN, VERSION, BlockEntry, H3TError, align,
                    nbytes_of, quant_linear_names, st_dtype, typed_view)

_REFINER_RE = re.compile(r"^token_refiner\.blocks\.(\d+)\.(.+)$")


class TensorSource:
    """Something that can stream the bytes of one tensor: dtype (safetensors name), shape, chunks()."""

    dtype: str
    shape: Tuple[int, ...]
    nbytes: int

    def chunks(self, chunk_bytes: int) -> Iterator[memoryview]:
        raise NotImplementedError

    def read(self) -> torch.Tensor:
        data = bytearray()
        for c in self.chunks(32 << 20):
            data += c
        buf = torch.frombuffer(data, dtype=torch.uint8) if self.nbytes else torch.empty(0, dtype=torch.uint8)
        return typed_view(buf, 0, self.dtype, self.shape)


class TorchSource(TensorSource):
    def __init__(self, t: torch.Tensor):
        t = t.detach()
        if t.device.type != "cpu":
            t = t.cpu()
        self._t = t.contiguous()
        self.dtype, self.shape = st_dtype(t.dtype), tuple(t.shape)
        self.nbytes = nbytes_of(self.dtype, self.shape)

    def chunks(self, chunk_bytes: int) -> Iterator[memoryview]:
        if self.nbytes == 0:
            return
        mv = memoryview(self._t.reshape(-1).view(torch.uint8).numpy())
        for a in range(0, self.nbytes, chunk_bytes):
            yield mv[a: a + chunk_bytes]


class LazySource(TensorSource):
    """Produces its tensor only while it is being written (bounded memory for large synthetic stores)."""

    def __init__(self, dtype: str, shape: Sequence[int], fn: Callable[[], torch.Tensor]):
        self.dtype, self.shape, self._fn = dtype, tuple(shape), fn
        self.nbytes = nbytes_of(dtype, shape)

    def chunks(self, chunk_bytes: int) -> Iterator[memoryview]:
        src = TorchSource(self._fn())
        if (src.dtype, src.shape) != (self.dtype, self.shape):
            raise H3TError(f"lazy tensor produced {src.dtype}{src.shape}, declared {self.dtype}{self.shape}")
        yield from src.chunks(chunk_bytes)


def as_source(x: Union[TensorSource, torch.Tensor]) -> TensorSource:
    return x if isinstance(x, TensorSource) else TorchSource(x)


def classify(names: Iterable[str]):
    """(globals, {refiner block: names}, other token_refiner.* names, {block: block-relative names})."""
    glob, ref_blocks, ref_other, blocks = [], {}, [], {}
    for n in names:
        if n.startswith(PAD_PREFIX):
            raise H3TError(f"tensor name {n!r} uses the reserved padding prefix {PAD_PREFIX!r}")
        m = BLOCK_RE.match(n)
        if m:
            blocks.setdefault(int(m.group(1)), []).append(m.group(2))
            continue
        m = _REFINER_RE.match(n)
        if m:
            ref_blocks.setdefault(int(m.group(1)), []).append(m.group(2))
        elif n.startswith("token_refiner."):
            ref_other.append(n)
        else:
            glob.append(n)
    return glob, ref_blocks, ref_other, blocks


def _place(entries: Sequence[Tuple[str, str, Tuple[int, ...]]]) -> Tuple[List[BlockEntry], int]:
    out, cur = [], 0
    for name, dt, shape in entries:
        cur = align(cur, TENSOR_ALIGN)
        nb = nbytes_of(dt, shape)
        out.append(BlockEntry(name, dt, tuple(shape), cur, nb))
        cur += nb
    return out, cur


def write_h3t(dst, cfg: H3Config, tensors: Mapping[str, Union[TensorSource, torch.Tensor]], *,
              quant: Optional[Mapping[str, object]] = None, source_name: str = "", source_size: int = 0,
              source_sha256: str = "", extra_meta: Optional[Mapping[str, str]] = None, chunk_bytes: int = 32 << 20,
              progress: Optional[Callable[[str, int, int], None]] = None) -> Dict[str, int]:
    """Write `tensors` (ComfyUI-layout names: `blocks.<i>.<...>`, `token_refiner.*`, globals) as an h3t file."""
    if chunk_bytes < 4096 or chunk_bytes % 8:
        raise ValueError("chunk_bytes must be a multiple of 8 and at least 4096")
    src = {k: as_source(v) for k, v in tensors.items()}
    glob, ref_blocks, ref_other, blocks = classify(src)
    n_blocks = cfg.layers
    if n_blocks < 1 or sorted(blocks) != list(range(n_blocks)):
        raise H3TError(f"config says {n_blocks} blocks but the tensors carry block indices {sorted(blocks)[:8]}...")
    rel0 = sorted(blocks[0])  # one layout for every block: the tensor set, dtypes and shapes must agree
    sig0 = {r: (src[f"blocks.0.{r}"].dtype, src[f"blocks.0.{r}"].shape) for r in rel0}
    for i in range(1, n_blocks):
        if set(blocks[i]) != set(rel0):
            raise H3TError(f"block {i} tensor set differs from block 0")
        for r in rel0:
            s = src[f"blocks.{i}.{r}"]
            if (s.dtype, s.shape) != sig0[r]:
                raise H3TError(f"blocks.{i}.{r} is {s.dtype}{s.shape}, block 0 has {sig0[r][0]}{sig0[r][1]}")
    blk_layout, blk_end = _place([(r, *sig0[r]) for r in rel0])
    block_nbytes = align(blk_end, BLOCK_ALIGN)
    g_names = sorted(glob)
    for j in sorted(ref_blocks):
        g_names += [f"token_refiner.blocks.{j}.{r}" for r in sorted(ref_blocks[j])]
    g_names += sorted(ref_other)
    g_layout, g_end = _place([(n, src[n].dtype, src[n].shape) for n in g_names])
    blocks_start = align(g_end, BLOCK_ALIGN)
    qmeta = dict(quant) if quant else ({"format": "asym_w4a8_int8", "group_size": cfg.quant_group,
                                         "convrot_groupsize": cfg.quant_convrot} if quant_linear_names(rel0) else {})
    data_end = blocks_start + n_blocks * block_nbytes

    plan = [(e.offset, e.name, e.nbytes, src[e.name]) for e in g_layout]
    for i in range(n_blocks):
        base = blocks_start + i * block_nbytes
        plan += [(base + e.offset, f"blocks.{i}.{e.name}", e.nbytes, src[f"blocks.{i}.{e.name}"]) for e in blk_layout]
    plan.sort(key=lambda p: p[0])
    flat, cur, npad = [], 0, 0
    for off, name, nb, s in plan:
        if off < cur:
            raise H3TError(f"internal layout overlap at {name!r}")
        if off > cur:
            flat.append((cur, f"{PAD_PREFIX}{npad}", off - cur, None))
            npad += 1
        flat.append((off, name, nb, s))
        cur = off + nb
    if cur < data_end:
        flat.append((cur, f"{PAD_PREFIX}{npad}", data_end - cur, None))
        npad += 1

    lay = lambda L: json.dumps([[e.name, e.dtype, list(e.shape), e.offset, e.nbytes] for e in L], separators=(",", ":"))  # noqa: E731
    meta = {"format": FORMAT, "version": str(VERSION), "config": cfg.to_json(), "n_blocks": str(n_blocks),
            "tensor_align": str(TENSOR_ALIGN), "block_align": str(BLOCK_ALIGN), "block_nbytes": str(block_nbytes),
            "blocks_start": str(blocks_start),
            "block_ranges": json.dumps([[blocks_start + i * block_nbytes, blocks_start + (i + 1) * block_nbytes]
                                        for i in range(n_blocks)], separators=(",", ":")),
            "block_layout": lay(blk_layout), "globals_layout": lay(g_layout), "quant": json.dumps(qmeta, sort_keys=True),
            "source_name": source_name, "source_size": str(source_size), "source_header_sha256": source_sha256}
    meta.update({str(k): str(v) for k, v in (extra_meta or {}).items()})
    header: Dict[str, object] = {"__metadata__": meta}
    for off, name, nb, s in flat:
        header[name] = {"dtype": s.dtype if s else "U8", "shape": list(s.shape) if s else [nb], "data_offsets": [off, off + nb]}
    hdr = json.dumps(header, separators=(",", ":")).encode("ascii")
    data_start = align(8 + len(hdr), BLOCK_ALIGN)
    hdr += b" " * (data_start - 8 - len(hdr))  # JSON whitespace: page-aligns the data section

    dst = os.fspath(dst)
    tmp = dst + ".part"
    total = sum(nb for _, name, nb, _ in flat if not name.startswith(PAD_PREFIX))
    done = 0
    try:
        with open(tmp, "wb") as f:
            f.write(struct.pack("<Q", data_start - 8))
            f.write(hdr)
            pos = 0
            for off, name, nb, s in flat:
                if off != pos:
                    raise H3TError(f"internal layout error at {name!r}")
                if s is None:
                    f.write(bytes(nb))
                else:
                    wrote = 0
                    for chunk in s.chunks(chunk_bytes):
                        f.write(chunk)
                        wrote += len(chunk)
                    if wrote != nb:
                        raise H3TError(f"{name}: source produced {wrote} bytes, expected {nb}")
                    done += nb
                    if progress and nb >= (1 << 20):
                        progress(name, done, total)
                pos += nb
            f.flush()
            os.fsync(f.fileno())
        os.replace(tmp, dst)
    except BaseException:
        try:
            os.remove(tmp)
        except OSError:
            pass
        raise
    return {"file_size": data_start + data_end, "data_start": data_start, "blocks_start": blocks_start,
            "block_nbytes": block_nbytes, "n_blocks": n_blocks, "n_pads": npad, "n_tensors": len(flat) - npad}
