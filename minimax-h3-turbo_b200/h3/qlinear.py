"""W4A8 ConvRot linear on B200: the public API of the reference's `h3turbo/h3/qlinear.py`, running on libh3b.so.

Same functions, arguments, results and errors as the reference module (citations are file:line there), so the H3
model, engine and ComfyUI node can call it unchanged.  All W4A8 work runs in the sm_100a kernels:

  rotate / quantize_activation   kernel KA  (in-register fp32 block Hadamard + per-token int8 absmax)
  decode_int8_grid               int4 -> int8 grid decode
  linear(precision="a8")         KA -> KB (tcgen05 kind::i8 GEMM, TMEM accumulators, fused scale/bias epilogue)

There is no CPU path and no second backend: W4A8 inputs must be CUDA tensors, and if libh3b.so is missing every call
raises.  backend "auto", "b200" and "ck" (the name the reference uses for its fused CUDA kernel) all select these kernels.
precision="a16" (unquantised activations; not the hot path) rotates with kernel KA and multiplies the exact int8 levels
with a bf16/fp32 tensor-core GEMM through torch, as the reference's CUDA a16 path does (qlinear.py:407-424).
"""
from __future__ import annotations

import math
from typing import Any, Dict, Optional, Tuple

import torch
import torch.nn.functional as F

from .. import _lib
from .types import W4A8Weight, Weight

CONVROT = 256  # qlinear.py:30
_H4 = ((1, 1, 1, -1), (1, 1, -1, 1), (1, -1, 1, 1), (-1, 1, 1, 1))  # qlinear.py:31
_HAD_CACHE: Dict[Tuple[int, str, int, torch.dtype], torch.Tensor] = {}
_BACKENDS = ("auto", "b200", "ck")
_OUT_DTYPES = (torch.bfloat16, torch.float16, torch.float32)
_DECODE_ELEMS = 1 << 24  # int8 grid elements per a16 slab (bounds the temporary, as qlinear.py:38)


# --------------------------------------------------------------------------------------------- Hadamard
def hadamard_regular(size: int, device="cpu", dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """kron(H4, ..., H4) / sqrt(size): symmetric and involutory, entries +-2^-j (qlinear.py:44-66).  Cached; do not mutate.
    A small constant matrix (used by `dequantize`); the kernels never materialise it."""
    n = size
    while n > 1 and n % 4 == 0:
        n //= 4
    if size < 4 or n != 1:
        raise ValueError(f"regular Hadamard size must be a power of 4 (>= 4), got {size}")
    dev = torch.device(device)
    if dev.type == "cuda" and dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    key = (size, dev.type, -1 if dev.index is None else dev.index, dtype)
    h = _HAD_CACHE.get(key)
    if h is None:
        h4 = torch.tensor(_H4, dtype=torch.float64)
        full = h4
        while full.shape[0] < size:
            full = torch.kron(full, h4)
        h = (full / math.sqrt(size)).to(device=dev, dtype=dtype).contiguous()
        _HAD_CACHE[key] = h
    return h


# --------------------------------------------------------------------------------------------- helpers
def _need_cuda(*ts: torch.Tensor) -> torch.device:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("the b200 W4A8 kernels need CUDA tensors (there is no CPU path); move the inputs to the GPU")
    return ts[0].device


def _rows(x2: torch.Tensor) -> torch.Tensor:
    """[M, W] with unit stride along W and a 16-byte aligned base / row stride (copy only if the view is unusable)."""
    es = x2.element_size()
    if x2.stride(-1) != 1 or (x2.stride(0) * es) % 16 or x2.data_ptr() % 16 or (x2.shape[0] > 1 and x2.stride(0) < x2.shape[1]):
        x2 = x2.contiguous()
        if x2.data_ptr() % 16:
            x2 = x2.clone()
    return x2


def _ld(x2: torch.Tensor) -> int:
    return x2.stride(0) if x2.shape[0] > 1 else x2.shape[1]


def _check_mode(mode: str) -> None:
    if mode not in ("ck", "eager"):
        raise ValueError(f"quant_mode must be 'ck' or 'eager', got {mode!r}")


def _check_weight(w: W4A8Weight) -> Tuple[int, int]:
    """Shape / dtype validation of a W4A8 layer (qlinear.py:140-154)."""
    if w.q.dim() != 2 or w.q.dtype not in (torch.int8, torch.uint8):
        raise ValueError(f"W4A8 q must be a 2D int8 tensor, got {tuple(w.q.shape)} {w.q.dtype}")
    n, k = w.q.shape[0], w.q.shape[1] * 2
    gs, cr = w.group_size, w.convrot
    if gs < 4 or k % 16 or k % gs or k % cr or (16 % gs and gs % 16):
        raise ValueError(f"K={k} must be divisible by 16, group_size={gs} and convrot={cr}; group_size >= 4 dividing 16 or a multiple of 16")
    if tuple(w.s_rel.shape) != (n, k // gs):
        raise ValueError(f"s_rel must have shape {(n, k // gs)}, got {tuple(w.s_rel.shape)}")
    if tuple(w.s_ch.shape) != (n,):
        raise ValueError(f"s_ch must have shape {(n,)}, got {tuple(w.s_ch.shape)}")
    if tuple(w.codebook.shape) != (16,):
        raise ValueError(f"codebook must have shape (16,), got {tuple(w.codebook.shape)}")
    return n, k


class _WeightArgs:
    """The C-ABI view of a W4A8Weight: pointers, strides and dtype codes (no copies unless a tensor is unusable)."""

    def __init__(self, w: W4A8Weight):
        self.n, self.k = _check_weight(w)
        q = w.q if w.q.stride(-1) == 1 and w.q.data_ptr() % 8 == 0 and w.q.stride(0) % 8 == 0 else w.q.contiguous()
        if q.data_ptr() % 8:
            q = q.clone()
        s = w.s_rel if w.s_rel.stride(-1) == 1 else w.s_rel.contiguous()
        self.q, self.s = q, s
        self.ldq = q.stride(0) if q.shape[0] > 1 else q.shape[1]
        self.lds = s.stride(0) if s.shape[0] > 1 else s.shape[1]
        self.s_dtype = _lib.scale_code(s.dtype)
        self.s_ch = w.s_ch if (w.s_ch.dtype == torch.float32 and w.s_ch.is_contiguous()) else w.s_ch.float().contiguous()
        self.cb = w.codebook if (w.codebook.dtype == torch.float32 and w.codebook.is_contiguous()) else w.codebook.float().contiguous()
        self.group, self.convrot = w.group_size, w.convrot
        _need_cuda(q, s, self.s_ch, self.cb)


# --------------------------------------------------------------------------------------------- rotation / quantiser
def rotate(x: torch.Tensor, size: int = CONVROT) -> torch.Tensor:
    """x[..., K] -> per-`size`-block x @ H in x.dtype (qlinear.py:118-132).  fp32 transform, one rounding to x.dtype."""
    if not x.is_floating_point():
        raise ValueError(f"rotate expects a floating tensor, got {x.dtype}")
    k = x.shape[-1]
    if k % size:
        raise ValueError(f"last dim {k} is not a multiple of the rotation block {size}")
    if x.numel() == 0:
        return x.clone()
    dev = _need_cuda(x)
    x2 = _rows(x.reshape(-1, k))
    y = torch.empty(x2.shape[0], k, dtype=x.dtype, device=dev)
    code = _lib.act_code(x.dtype)
    L = _lib.lib()
    _lib.check(L.h3b_rotate(x2.data_ptr(), code, x2.shape[0], k, _ld(x2), size, y.data_ptr(), code, k, _lib.stream_ptr(dev)),
               "rotate")
    return y.reshape(x.shape)


def _quantize_rows(x2: torch.Tensor, size: int, mode: str, swiglu: bool = False) -> Tuple[torch.Tensor, torch.Tensor]:
    """Rotate (+ SwiGLU first) and quantise rows: (int8 [M, K], fp32 [M, 1]) -- kernel KA (qlinear.py:267-292)."""
    dev = _need_cuda(x2)
    x2 = _rows(x2)
    m, w = x2.shape
    k = w // 2 if swiglu else w
    q = torch.empty(m, k, dtype=torch.int8, device=dev)
    xs = torch.empty(m, 1, dtype=torch.float32, device=dev)
    if m:
        _lib.check(_lib.lib().h3b_rotq(x2.data_ptr(), _lib.act_code(x2.dtype), m, k, _ld(x2), size, int(swiglu),
                                       _lib.QMODE[mode], q.data_ptr(), k, xs.data_ptr(), _lib.stream_ptr(dev)),
                   "quantize_activation")
    return q, xs


def quantize_activation(x: torch.Tensor, *, size: int = CONVROT, quant_mode: str = "ck") -> Tuple[torch.Tensor, torch.Tensor]:
    """x[..., K] -> (int8 [..., K], fp32 scale [..., 1]) of the rotated activation (qlinear.py:295-303)."""
    _check_mode(quant_mode)
    k = x.shape[-1]
    if k % size:
        raise ValueError(f"last dim {k} is not a multiple of the rotation block {size}")
    with torch.no_grad():
        q, s = _quantize_rows(x.reshape(math.prod(x.shape[:-1]), k), size, quant_mode)
    return q.reshape(x.shape), s.reshape(*x.shape[:-1], 1)


# --------------------------------------------------------------------------------------------- weights
@torch.no_grad()
def decode_int8_grid(w: W4A8Weight) -> torch.Tensor:
    """int8 [N, K]: the exact grid the int8 GEMM consumes (qlinear.py:194-204), decoded on the GPU."""
    a = _WeightArgs(w)
    grid = torch.empty(a.n, a.k, dtype=torch.int8, device=a.q.device)
    if a.n:
        _lib.check(_lib.lib().h3b_decode_grid(a.q.data_ptr(), a.n, a.k, a.ldq, a.s.data_ptr(), a.s_dtype, a.lds,
                                              a.cb.data_ptr(), a.group, grid.data_ptr(), a.k, _lib.stream_ptr(a.q.device)),
                   "decode_int8_grid")
    return grid


@torch.no_grad()
def dequantize(w: W4A8Weight, dtype: torch.dtype = torch.float32, rotated: bool = False, *, rows: Optional[slice] = None) -> torch.Tensor:
    """Dense [N, K] weight (qlinear.py:207-226).  rotated=True: grid * s_ch in the ConvRot basis; False: the original
    basis (the fp32 block rotation of the rotated weight, rounded once to `dtype`).  `rows`: a contiguous row slice."""
    n, k = _check_weight(w)
    if rows is not None and rows.step not in (None, 1):
        raise ValueError("rows must be a contiguous slice")
    r0, r1, _ = (rows or slice(0, n)).indices(n)
    r1 = max(r1, r0)
    sub = W4A8Weight(w.q[r0:r1], w.s_rel[r0:r1], w.s_ch[r0:r1], w.codebook, w.group_size, w.convrot)
    if r1 == r0:
        return torch.empty(0, k, dtype=dtype, device=w.q.device)
    wr = decode_int8_grid(sub).float().mul_(sub.s_ch.float().unsqueeze(1))
    if not rotated:
        wr = rotate(wr, w.convrot)  # H is symmetric and involutory: W = W_rot @ H per block
    return wr.to(dtype)


# --------------------------------------------------------------------------------------------- GEMM (parity helper)
def _int8_mm(a: torch.Tensor, w8: torch.Tensor) -> torch.Tensor:
    """Exact int32 a[M, K] @ w8[N, K]^T on the tcgen05 tensor cores (qlinear.py:236-254)."""
    m, k = a.shape
    n = w8.shape[0]
    dev = _need_cuda(a, w8)
    c = torch.zeros(m, n, dtype=torch.int32, device=dev)
    if m == 0 or n == 0 or k == 0:
        return c
    a2, b2 = _rows(a), _rows(w8)
    _lib.check(_lib.lib().h3b_int8_gemm_s32(a2.data_ptr(), _ld(a2), m, b2.data_ptr(), _ld(b2), n, k, c.data_ptr(), n,
                                            _lib.stream_ptr(dev)), "int8 GEMM")
    return c


def _gemm_codes(qa: torch.Tensor, xs: torch.Tensor, w: W4A8Weight, bias: Optional[torch.Tensor] = None,
                out_dtype: torch.dtype = torch.bfloat16, quant_mode: str = "ck") -> torch.Tensor:
    """Kernel KB alone on given activation codes and scales: decode -> int8 GEMM -> epilogue (qlinear.py:396-405).
    out_dtype=torch.int32 returns the raw accumulator.  With the reference's own codes and scales as input the result is
    bit-identical to the reference's output (everything after the quantiser is exact integer or fixed-order fp32)."""
    a = _WeightArgs(w)
    dev = _need_cuda(qa, xs)
    qa2 = _rows(qa)
    m = qa2.shape[0]
    out = torch.empty(m, a.n, dtype=out_dtype, device=dev)
    if m == 0:
        return out
    code = _lib.INT32 if out_dtype == torch.int32 else _lib.act_code(out_dtype)
    b = None if bias is None or out_dtype == torch.int32 else bias.to(device=dev, dtype=out_dtype).contiguous()
    xs1 = xs.reshape(-1).float().contiguous()
    L = _lib.lib()
    ws_bytes = int(L.h3b_gemm_workspace_bytes(m, a.n, a.k))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    _lib.check(L.h3b_w4a8_gemm(qa2.data_ptr(), _ld(qa2), xs1.data_ptr(), m, a.q.data_ptr(), a.ldq, a.s.data_ptr(), a.s_dtype,
                               a.lds, a.s_ch.data_ptr(), a.cb.data_ptr(), a.group, _lib.ptr(b), out.data_ptr(), code, a.n,
                               a.n, a.k, _lib.QMODE[quant_mode], ws.data_ptr(), ws_bytes, _lib.stream_ptr(dev)), "W4A8 GEMM")
    return out


# --------------------------------------------------------------------------------------------- backends
def available_backends() -> Dict[str, Dict[str, Any]]:
    """{"b200": {...}, "ck": {...}}: availability of the sm_100a kernels ("ck", the reference's name for its fused CUDA
    backend, reports the same kernels so callers that probe it -- H3Engine.linear_backend -- keep working)."""
    cuda = torch.cuda.is_available()
    why = None
    if not _lib.available():
        why = f"libh3b.so is not built or cannot be loaded ({_lib.LIB_PATH})"
    elif not cuda:
        why = "no CUDA device"
    elif torch.cuda.get_device_capability() < (10, 0):
        why = f"needs an sm_100 GPU (B200), found sm_{''.join(map(str, torch.cuda.get_device_capability()))}"
    info = {"available": why is None, "reason": why, "version": f"h3b-{_lib.ABI_VERSION}"}
    return {"b200": dict(info), "ck": dict(info)}


def resolve_backend(x: torch.Tensor, w: Weight, backend: str = "auto", precision: str = "a8") -> str:
    """The backend `linear` will use: "b200", or "dense" for a dense weight (qlinear.py:345-361)."""
    if backend not in _BACKENDS:
        raise ValueError(f"backend must be 'auto', 'b200' or 'ck', got {backend!r}")
    if precision not in ("a8", "a16"):
        raise ValueError(f"precision must be 'a8' or 'a16', got {precision!r}")
    if not isinstance(w, W4A8Weight):
        return "dense"
    if not x.is_cuda or not w.q.is_cuda:
        raise RuntimeError("backend 'b200' unavailable: needs CUDA tensors (there is no CPU path)")
    return "b200"


def _swiglu(x: torch.Tensor) -> torch.Tensor:
    gate, up = x.chunk(2, dim=-1)
    return F.silu(gate).mul_(up)


# --------------------------------------------------------------------------------------------- linear
def _a8(x2: torch.Tensor, a: _WeightArgs, bias: Optional[torch.Tensor], out: torch.Tensor, swiglu: bool, mode: str) -> None:
    """One fused call: (swiglu) -> rotate+quantise -> int8 GEMM -> epilogue, into `out` (a [rows, N] view)."""
    dev = x2.device
    x2 = _rows(x2)
    m = x2.shape[0]
    L = _lib.lib()
    ws_bytes = int(L.h3b_linear_workspace_bytes(m, a.n, a.k))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    _lib.check(L.h3b_w4a8_linear(x2.data_ptr(), _lib.act_code(x2.dtype), m, a.k, _ld(x2), int(swiglu), a.q.data_ptr(), a.ldq,
                                 a.s.data_ptr(), a.s_dtype, a.lds, a.s_ch.data_ptr(), a.cb.data_ptr(), a.group, a.convrot,
                                 _lib.ptr(bias), out.data_ptr(), _lib.act_code(out.dtype), out.stride(0), a.n,
                                 _lib.QMODE[mode], ws.data_ptr(), ws_bytes, _lib.stream_ptr(dev)), "W4A8 linear")


def _a16(x2: torch.Tensor, w: W4A8Weight, a: _WeightArgs, bias: Optional[torch.Tensor], out: torch.Tensor, swiglu: bool) -> None:
    """Unquantised activations (qlinear.py:407-424): rotated x (rounded to x.dtype) times the exact int8 levels, fp32
    accumulation, per-channel scale (and bias) in fp32, one rounding to out_dtype."""
    xc = _swiglu(x2) if swiglu else x2
    dt = xc.dtype
    xr = rotate(xc, a.convrot)
    cdt = dt if dt in (torch.bfloat16, torch.float16) else torch.float32
    xg = xr.to(cdt)
    w8 = decode_int8_grid(w)
    step = max(1, _DECODE_ELEMS // a.k)
    for r0 in range(0, a.n, step):
        r1 = min(r0 + step, a.n)
        lv = w8[r0:r1].to(cdt).t()
        y = torch.mm(xg, lv, out_dtype=torch.float32) if cdt != torch.float32 else torch.mm(xg, lv)
        y.mul_(a.s_ch[r0:r1])
        if bias is not None:
            y.add_(bias[r0:r1].to(y.dtype))
        out[:, r0:r1] = y


@torch.no_grad()
def _linear_w4a8(x2, w, bias, out_dtype, precision, swiglu, chunk_tokens, quant_mode):
    a = _WeightArgs(w)
    kx = x2.shape[-1] // (2 if swiglu else 1)
    if kx != a.k:
        raise ValueError(f"input features {kx}{' (after swiglu)' if swiglu else ''} do not match the weight's K={a.k}")
    if x2.device != w.q.device:
        raise ValueError(f"input on {x2.device} but weight on {w.q.device}")
    if bias is not None and tuple(bias.shape) != (a.n,):
        raise ValueError(f"bias must have shape {(a.n,)}, got {tuple(bias.shape)}")
    if out_dtype not in _OUT_DTYPES:
        raise ValueError(f"out_dtype must be bf16, fp16 or fp32 on the b200 backend, got {out_dtype}")
    m = x2.shape[0]
    out = torch.empty(m, a.n, dtype=out_dtype, device=x2.device)
    if m == 0:
        return out
    step = min(chunk_tokens or m, m)
    if precision == "a8":
        b = None if bias is None else bias.to(device=x2.device, dtype=out_dtype).contiguous()  # qlinear.py:405
        for r in range(0, m, step):
            _a8(x2[r:r + step], a, b, out[r:r + step], swiglu, quant_mode)
    else:
        b = None if bias is None else bias.to(device=x2.device)
        for r in range(0, m, step):
            _a16(x2[r:r + step], w, a, b, out[r:r + step], swiglu)
    return out


def linear(
    x: torch.Tensor,
    w: Weight,
    bias: Optional[torch.Tensor] = None,
    *,
    out_dtype: Optional[torch.dtype] = None,
    backend: str = "auto",
    precision: str = "a8",
    input_act: Optional[str] = None,
    chunk_tokens: Optional[int] = None,
    quant_mode: str = "ck",
) -> torch.Tensor:
    """out = act(x) @ W^T + bias over the last dim of x (qlinear.py:466-523).

    w: W4A8Weight (the b200 kernels) or a dense [N, K] tensor (plain F.linear in x.dtype, on the GPU).
    input_act="swiglu": x is [gate | up]; silu(gate) * up in x.dtype is applied inside the rotate+quantise kernel.
    chunk_tokens bounds the per-call activation scratch; a8 is token-wise, so chunking never changes the result.
    quant_mode "ck" (the reference's CUDA profile) or "eager"; precision "a8" (int8 activations) or "a16".
    """
    if not x.is_floating_point():
        raise ValueError(f"x must be floating point, got {x.dtype}")
    if input_act not in (None, "none", "swiglu"):
        raise ValueError(f"input_act must be None or 'swiglu', got {input_act!r}")
    if chunk_tokens is not None and chunk_tokens < 1:
        raise ValueError("chunk_tokens must be >= 1")
    _check_mode(quant_mode)
    swiglu = input_act == "swiglu"
    if swiglu and x.shape[-1] % 2:
        raise ValueError(f"swiglu needs an even last dim, got {x.shape[-1]}")
    out_dtype = out_dtype or x.dtype
    kind = resolve_backend(x, w, backend, precision)
    lead = x.shape[:-1]
    x2 = x.reshape(math.prod(lead), x.shape[-1])
    if kind != "dense":
        y = _linear_w4a8(x2, w, bias, out_dtype, precision, swiglu, chunk_tokens, quant_mode)
        return y.reshape(*lead, y.shape[-1])
    _need_cuda(x, w)
    if x2.shape[-1] // (2 if swiglu else 1) != w.shape[-1]:
        raise ValueError(f"input features {x2.shape[-1]} do not match the dense weight {tuple(w.shape)}")
    xc = _swiglu(x2) if swiglu else x2
    y = F.linear(xc, w.to(x.dtype), None if bias is None else bias.to(x.dtype)).to(out_dtype)
    return y.reshape(*lead, y.shape[-1])

