"""Per-head q/k RMSNorm + split-half rotary embedding (h3turbo/h3/layout.py:265-356).

`norm_rope_` keeps the reference's signature.  impl "b200" (what "auto" picks for bf16/fp16 CUDA tensors) runs the fused
kernel `h3b_qk_norm_rope`, bit-identical to the reference's "torch" form of comfy_kitchen's fused op; "torch" and
"eager" are the reference's two torch formulas (the bit-exact fused order, and ComfyUI's portable path, which the
reference also uses for fp32).  The torch formulas serve fp32 and CPU tensors (the CPU ranks of the sharding tests).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn.functional as F

from .. import _lib


def rope_angles(position_ids: torch.Tensor, inv_freq: torch.Tensor, device) -> torch.Tensor:
    """[S, 3] positions -> [S, 3 F] fp32 angles: all t frequencies, then h, then w (layout.py:265-273)."""
    pos = position_ids.to(torch.float32).to(device)
    ang = pos.unsqueeze(-1) * inv_freq.to(device=device, dtype=torch.float32).view(1, 1, -1)
    return ang.reshape(pos.shape[0], -1)


def rms_norm_fused_order(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """Per-head RMSNorm with the fused kernel's summation order (layout.py:309-326): lane l sums the squares of
    elements l, l + 32, ... in fp32, then a halving tree over the 32 lanes; x * rsqrt(sum / d + eps) * w rounded once."""
    d = x.shape[-1]
    if x.dtype == torch.float32 or d % 32:
        return F.rms_norm(x, (d,), weight.to(x.dtype), eps)
    xf = x.to(torch.float32)
    sq = xf.square().reshape(*x.shape[:-1], d // 32, 32)
    acc = sq[..., 0, :]
    for j in range(1, d // 32):
        acc = acc + sq[..., j, :]
    for off in (16, 8, 4, 2, 1):
        acc = acc[..., :off] + acc[..., off:2 * off]
    return (xf * torch.rsqrt(acc / d + eps) * weight.to(torch.float32)).to(x.dtype)


def _kernel_ok(x: torch.Tensor) -> bool:
    d = x.shape[-1]
    return x.is_cuda and x.dtype in (torch.bfloat16, torch.float16) and d in (32, 64, 128, 256)


def _fused(q: Optional[torch.Tensor], k: Optional[torch.Tensor], wq, wk, eps: float, cos: torch.Tensor,
           sin: torch.Tensor) -> None:
    ref = q if q is not None else k
    s, heads, d = ref.shape
    for t in (q, k):
        if t is not None and (t.shape != ref.shape or t.dtype != ref.dtype or t.stride(2) != 1 or t.stride(1) != d):
            raise ValueError("q and k must be [S, heads, D] views with contiguous heads and the same shape/dtype")
    half = cos.shape[1]
    if sin.shape != cos.shape or cos.shape[0] != s or cos.stride(1) != 1 or sin.stride() != cos.stride():
        raise ValueError("cos/sin must be [S, half] with unit column stride and equal strides")
    if cos.device != ref.device:
        raise ValueError("cos/sin must be on the q/k device")
    ws = [None if w is None else w.contiguous() for w in (wq, wk)]
    wdt = _lib.act_code((ws[0] if ws[0] is not None else ws[1]).dtype)
    if ws[0] is not None and ws[1] is not None and ws[0].dtype != ws[1].dtype:
        ws[1] = ws[1].to(ws[0].dtype)
    L = _lib.lib()
    _lib.check(L.h3b_qk_norm_rope(_lib.ptr(q), 0 if q is None else q.stride(0), _lib.ptr(k), 0 if k is None else k.stride(0),
                                  _lib.act_code(ref.dtype), s, heads, d, _lib.ptr(ws[0]), _lib.ptr(ws[1]), wdt, float(eps),
                                  cos.data_ptr(), sin.data_ptr(), cos.stride(0), _lib.act_code(cos.dtype), half,
                                  _lib.stream_ptr(ref.device)), "qk_norm_rope")


@torch.no_grad()
def norm_rope_(q: torch.Tensor, k: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, eps: float, cos: torch.Tensor,
               sin: torch.Tensor, impl: str = "auto", table=None, chunk: int = 1024) -> None:
    """In place on [S, heads, D] views: per-head RMSNorm, then split-half rotation of the leading 2 * half dims
    (layout.py:329-356; `table` is accepted for the reference's "ck" signature and ignored)."""
    if impl not in ("auto", "b200", "ck", "torch", "eager"):
        raise ValueError(f"rope_impl must be auto/b200/ck/torch/eager, got {impl!r}")
    if impl in ("auto", "b200", "ck"):
        if all(t is None or _kernel_ok(t) for t in (q, k)):
            _fused(q, k, wq, wk, eps, cos, sin)
            return
        if impl != "auto":
            raise RuntimeError("the fused q/k norm+RoPE kernel needs bf16/fp16 CUDA tensors with head_dim 32/64/128/256")
        impl = "torch"
    half = cos.shape[1]
    for x, w in ((q, wq), (k, wk)):
        if x is None:
            continue
        for a in range(0, x.shape[0], chunk):
            sl = slice(a, a + chunk)
            c, s = cos[sl].unsqueeze(1), sin[sl].unsqueeze(1)
            if impl == "eager" or x.dtype == torch.float32:
                xn = F.rms_norm(x[sl], (x.shape[-1],), w.to(x.dtype), eps)
                t1, t2 = xn[..., :half], xn[..., half:2 * half]
                o1, o2 = (t1 * c).addcmul_(t2, -s), (t2 * c).addcmul_(t1, s)
            else:
                xn = rms_norm_fused_order(x[sl], w, eps)
                c, s = c.to(torch.float32), s.to(torch.float32)
                x1, x2 = xn[..., :half].to(torch.float32), xn[..., half:2 * half].to(torch.float32)
                o1, o2 = x1 * c - x2 * s, x1 * s + x2 * c
            xn[..., :half], xn[..., half:2 * half] = o1, o2
            x[sl] = xn
