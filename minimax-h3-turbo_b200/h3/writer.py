"""Writer of h3t weight stores (the format is described in store.py).

`write_h3t` plans the whole file before writing a byte: the block-relative tensor set of block 0 fixes one layout that
every block must match, globals and token-refiner tensors go first, each region is placed with TENSOR_ALIGN-aligned
tensor starts and BLOCK_ALIGN-aligned block starts and sizes, and every gap becomes an explicit `__pad.<n>` U8 entry.
The header (metadata: the layout, block ranges, config and quantisation parameters) is then serialised, padded with
JSON whitespace so the data section starts on a BLOCK_ALIGN boundary, and the tensors are streamed in file order in
bounded chunks -- a source may produce its tensor only when its turn comes (LazySource).  The bytes go to
`<dst>.part`, are fsync'ed and renamed into place, so an interrupted write never leaves a file that looks valid.  The
resulting layout (tensor order, alignment, pad names, metadata keys) is the reference's byte format (writer.py:81-262
of h3turbo/h3), so the reference reads these files and this package reads the reference's.
"""
from __future__ import annotations

import json
import os
import re
import struct
from typing import Callable, Dict, Iterable, Iterator, List, Mapping, Optional, Sequence, Tuple, Union

import torch

from .config import H3Config
from .store import (BLOCK_ALIGN, BLOCK_RE, FORMAT, LINEARS, PAD_PREFIX, QUANT_PARTS, TENSOR_ALIGN, VERSION, BlockEntry,
                    H3TError, align, nbytes_of, quant_linear_names, st_dtype, typed_view)

_REFINER_BLOCK = re.compile(r"^token_refiner\.blocks\.(\d+)\.(.+)$")


# ---------------------------------------------------------------------------------------------------- tensor sources
class TensorSource:
    """The bytes of one tensor, produced in chunks: `dtype` (safetensors name), `shape`, `chunks(n)`."""

    dtype: str
    shape: Tuple[int, ...]

    @property
    def nbytes(self) -> int:
        return nbytes_of(self.dtype, self.shape)

    def chunks(self, chunk_bytes: int) -> Iterator[memoryview]:
        raise NotImplementedError

    def read(self) -> torch.Tensor:
        """The whole tensor on the CPU (assembled from the chunks)."""
        out = torch.empty(self.nbytes, dtype=torch.uint8)
        pos = 0
        for c in self.chunks(32 << 20):
            out[pos:pos + len(c)] = torch.frombuffer(bytearray(c), dtype=torch.uint8)
            pos += len(c)
        if pos != self.nbytes:
            raise H3TError(f"source produced {pos} bytes, expected {self.nbytes}")
        return typed_view(out, 0, self.dtype, self.shape)


class TorchSource(TensorSource):
    """A tensor already in memory (moved to the CPU and made contiguous once)."""

    def __init__(self, t: torch.Tensor):
        self._cpu = t.detach().to("cpu").contiguous()
        self.dtype, self.shape = st_dtype(self._cpu.dtype), tuple(self._cpu.shape)

    def chunks(self, chunk_bytes: int) -> Iterator[memoryview]:
        n = self.nbytes
        if n:
            flat = memoryview(self._cpu.reshape(-1).view(torch.uint8).numpy())
            for a in range(0, n, chunk_bytes):
                yield flat[a:min(n, a + chunk_bytes)]


class LazySource(TensorSource):
    """A tensor produced by `fn()` only when it is written (bounded memory for large synthetic stores); it must have
    the declared dtype and shape."""

    def __init__(self, dtype: str, shape: Sequence[int], fn: Callable[[], torch.Tensor]):
        self.dtype, self.shape, self._make = dtype, tuple(shape), fn

    def chunks(self, chunk_bytes: int) -> Iterator[memoryview]:
        made = TorchSource(self._make())
        if made.dtype != self.dtype or made.shape != self.shape:
            raise H3TError(f"lazy tensor produced {made.dtype}{made.shape}, declared {self.dtype}{self.shape}")
        return made.chunks(chunk_bytes)


def as_source(x: Union[TensorSource, torch.Tensor]) -> TensorSource:
    if isinstance(x, TensorSource):
        return x
    if isinstance(x, torch.Tensor):
        return TorchSource(x)
    raise TypeError(f"expected a Tensor or TensorSource, got {type(x).__name__}")


# ---------------------------------------------------------------------------------------------------- naming / order
def _canonical_block_order() -> Tuple[str, ...]:
    """Block-relative names in the order they are laid out: modulation, the attention half, the MLP half."""
    q = lambda lin: tuple(f"{lin}.{p}" for p in QUANT_PARTS)  # noqa: E731
    return ("adaln_proj.linear.weight", "adaln_proj.linear.bias", "norm1.weight", "attn.q_norm.weight",
            "attn.k_norm.weight") + q(LINEARS[0]) + q(LINEARS[1]) + ("norm2.weight",) + q(LINEARS[2]) + q(LINEARS[3])


_BLOCK_ORDER = _canonical_block_order()
_GLOBAL_ORDER = tuple(f"{m}.{p}" for m in ("video_patch_proj", "audio_patch_proj", "condition_proj") for p in ("weight", "bias")) + (
    "adaln_t_table", "rope.inv_freq", "final_layer.norm.weight", "final_layer.adaln_proj.linear.weight",
    "final_layer.adaln_proj.linear.bias") + tuple(f"final_layer.{m}.{p}" for m in ("video_out", "audio_out")
                                                  for p in ("weight", "bias"))


def _ordered(names: Iterable[str], first: Sequence[str]) -> List[str]:
    """The names of `first` that are present, in that order, then the rest alphabetically."""
    have = set(names)
    lead = [n for n in first if n in have]
    return lead + sorted(have - set(lead))


def classify(names: Iterable[str]):
    """Split tensor names into (globals, {refiner block index: relative names}, other token_refiner.* names,
    {block index: relative names})."""
    glob, ref_blocks, ref_other, blocks = [], {}, [], {}
    for name in names:
        if name.startswith(PAD_PREFIX):
            raise H3TError(f"tensor name {name!r} uses the reserved padding prefix {PAD_PREFIX!r}")
        hit = BLOCK_RE.match(name)
        if hit:
            blocks.setdefault(int(hit.group(1)), []).append(hit.group(2))
        elif (hit := _REFINER_BLOCK.match(name)):
            ref_blocks.setdefault(int(hit.group(1)), []).append(hit.group(2))
        elif name.startswith("token_refiner."):
            ref_other.append(name)
        else:
            glob.append(name)
    return glob, ref_blocks, ref_other, blocks


# ---------------------------------------------------------------------------------------------------- planning
def _pack(items: Sequence[Tuple[str, str, Tuple[int, ...]]]) -> Tuple[List[BlockEntry], int]:
    """Consecutive TENSOR_ALIGN-aligned placement from offset 0: (entries, end of the last tensor)."""
    placed, end = [], 0
    for name, dtype, shape in items:
        start = align(end, TENSOR_ALIGN)
        size = nbytes_of(dtype, shape)
        placed.append(BlockEntry(name, dtype, tuple(shape), start, size))
        end = start + size
    return placed, end


def _block_signature(src: Mapping[str, TensorSource], i: int, rels: Sequence[str]) -> Dict[str, Tuple[str, tuple]]:
    return {r: (src[f"blocks.{i}.{r}"].dtype, tuple(src[f"blocks.{i}.{r}"].shape)) for r in rels}


def _compact(entries) -> str:
    return json.dumps([[e.name, e.dtype, list(e.shape), e.offset, e.nbytes] for e in entries], separators=(",", ":"))


def write_h3t(dst, cfg: H3Config, tensors: Mapping[str, Union[TensorSource, torch.Tensor]], *,
              quant: Optional[Mapping[str, object]] = None, source_name: str = "", source_size: int = 0,
              source_sha256: str = "", extra_meta: Optional[Mapping[str, str]] = None, chunk_bytes: int = 32 << 20,
              progress: Optional[Callable[[str, int, int], None]] = None) -> Dict[str, int]:
    """Write `tensors` (ComfyUI-layout names: `blocks.<i>.<rel>`, globals, `token_refiner.*`) as an h3t file at `dst`.
    Peak memory is one chunk plus the header.  Returns a summary (file_size, data_start, blocks_start, block_nbytes,
    n_blocks, n_pads, n_tensors)."""
    if chunk_bytes < 4096 or chunk_bytes % 8:
        raise ValueError("chunk_bytes must be a multiple of 8 and at least 4096")
    src = {name: as_source(t) for name, t in tensors.items()}
    glob, ref_blocks, ref_other, blocks = classify(src)
    n_blocks = cfg.layers
    if n_blocks < 1 or sorted(blocks) != list(range(n_blocks)):
        raise H3TError(f"config says {n_blocks} blocks but the tensors carry block indices {sorted(blocks)[:8]}...")

    # one layout for all blocks: block 0 defines it, every other block must carry the same names, dtypes and shapes
    rels = _ordered(blocks[0], _BLOCK_ORDER)
    sig = _block_signature(src, 0, rels)
    for i in range(1, n_blocks):
        if set(blocks[i]) != set(rels):
            missing, extra = sorted(set(rels) - set(blocks[i])), sorted(set(blocks[i]) - set(rels))
            raise H3TError(f"block {i} tensor set differs from block 0: missing {missing[:4]}, extra {extra[:4]}")
        for r, (dt, shape) in _block_signature(src, i, rels).items():
            if (dt, shape) != sig[r]:
                raise H3TError(f"blocks.{i}.{r} is {dt}{shape}, block 0 has {sig[r][0]}{sig[r][1]}")
    block_entries, block_used = _pack([(r, *sig[r]) for r in rels])
    block_nbytes = align(block_used, BLOCK_ALIGN)

    head_names = _ordered(glob, _GLOBAL_ORDER)
    for j in sorted(ref_blocks):
        head_names.extend(f"token_refiner.blocks.{j}.{r}" for r in _ordered(ref_blocks[j], _BLOCK_ORDER))
    head_names.extend(_ordered(ref_other, ("token_refiner.final_norm.weight",)))
    head_entries, head_used = _pack([(n, src[n].dtype, tuple(src[n].shape)) for n in head_names])
    blocks_start = align(head_used, BLOCK_ALIGN)
    data_end = blocks_start + n_blocks * block_nbytes

    # the file's tensors in order, with the gaps made explicit
    placed = [(e.offset, e.name, e.nbytes, src[e.name]) for e in head_entries]
    for i in range(n_blocks):
        base = blocks_start + i * block_nbytes
        placed.extend((base + e.offset, f"blocks.{i}.{e.name}", e.nbytes, src[f"blocks.{i}.{e.name}"])
                      for e in block_entries)
    placed.sort(key=lambda p: p[0])
    ordered: List[Tuple[int, str, int, Optional[TensorSource]]] = []
    pos = 0
    for off, name, size, s in placed + [(data_end, None, 0, None)]:
        if off < pos:
            raise H3TError(f"internal layout overlap at {name!r}")
        if off > pos:
            ordered.append((pos, f"{PAD_PREFIX}{sum(1 for o in ordered if o[3] is None)}", off - pos, None))
        if name is not None:
            ordered.append((off, name, size, s))
        pos = off + size
    n_pads = sum(1 for o in ordered if o[3] is None)

    qmeta = dict(quant) if quant else ({"format": "asym_w4a8_int8", "group_size": cfg.quant_group,
                                        "convrot_groupsize": cfg.quant_convrot} if quant_linear_names(rels) else {})
    meta = {"format": FORMAT, "version": str(VERSION), "config": cfg.to_json(), "n_blocks": str(n_blocks),
            "tensor_align": str(TENSOR_ALIGN), "block_align": str(BLOCK_ALIGN), "block_nbytes": str(block_nbytes),
            "blocks_start": str(blocks_start),
            "block_ranges": json.dumps([[blocks_start + i * block_nbytes, blocks_start + (i + 1) * block_nbytes]
                                        for i in range(n_blocks)], separators=(",", ":")),
            "block_layout": _compact(block_entries), "globals_layout": _compact(head_entries),
            "quant": json.dumps(qmeta, sort_keys=True), "source_name": source_name, "source_size": str(source_size),
            "source_header_sha256": source_sha256}
    meta.update({str(k): str(v) for k, v in (extra_meta or {}).items()})
    index: Dict[str, object] = {"__metadata__": meta}
    for off, name, size, s in ordered:
        index[name] = {"dtype": "U8" if s is None else s.dtype, "shape": [size] if s is None else list(s.shape),
                       "data_offsets": [off, off + size]}
    body = json.dumps(index, separators=(",", ":")).encode("ascii")
    data_start = align(8 + len(body), BLOCK_ALIGN)
    body = body.ljust(data_start - 8, b" ")  # JSON whitespace: the data section starts block-aligned

    final = os.fspath(dst)
    part = final + ".part"
    total = sum(size for _, _, size, s in ordered if s is not None)
    written = 0
    try:
        with open(part, "wb") as f:
            f.write(struct.pack("<Q", len(body)))
            f.write(body)
            for off, name, size, s in ordered:
                if s is None:
                    f.write(b"\0" * size)
                    continue
                got = 0
                for chunk in s.chunks(chunk_bytes):
                    f.write(chunk)
                    got += len(chunk)
                if got != size:
                    raise H3TError(f"{name}: source produced {got} bytes, expected {size}")
                written += size
                if progress is not None and size >= (1 << 20):
                    progress(name, written, total)
            f.flush()
            os.fsync(f.fileno())  # the data is on disk before the rename makes the file visible
        os.replace(part, final)
    except BaseException:
        if os.path.exists(part):
            os.remove(part)
        raise
    return {"file_size": data_start + data_end, "data_start": data_start, "blocks_start": blocks_start,
            "block_nbytes": block_nbytes, "n_blocks": n_blocks, "n_pads": n_pads, "n_tensors": len(ordered) - n_pads}
