"""Per-head q/k RMSNorm + split-half rotary embedding (h3turbo/h3/layout.py:265-356).

`norm_rope_` keeps the reference's signature and runs the fused kernel `h3b_qk_norm_rope`, which is bit-identical to the
reference's "torch" form of comfy_kitchen's fused op (rms_norm_fused_order, layout.py:309-326, then the fp32 rotation):
impl "auto", "b200", "ck" and "torch" all mean that kernel.  ComfyUI's portable "eager" formula (other roundings) is not
built, and neither is a CPU or fp32 path: such calls raise RuntimeError.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import _lib


def rope_angles(position_ids: torch.Tensor, inv_freq: torch.Tensor, device) -> torch.Tensor:
    """[S, 3] positions -> [S, 3 F] fp32 angles: all t frequencies, then h, then w (layout.py:265-273)."""
    pos = position_ids.to(torch.float32).to(device)
    ang = pos.unsqueeze(-1) * inv_freq.to(device=device, dtype=torch.float32).view(1, 1, -1)
    return ang.reshape(pos.shape[0], -1)


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
    (layout.py:329-356; `table` and `chunk` are accepted for the reference's signature and ignored)."""
    if impl not in ("auto", "b200", "ck", "torch", "eager"):
        raise ValueError(f"rope_impl must be auto/b200/ck/torch/eager, got {impl!r}")
    if impl == "eager":
        raise RuntimeError("rope_impl 'eager' (ComfyUI's portable formula) is not built; 'torch' / 'b200' run the fused "
                           "kernel, bit-identical to the reference's 'torch' form")
    if not all(t is None or _kernel_ok(t) for t in (q, k)):
        raise RuntimeError("the fused q/k norm+RoPE kernel needs bf16/fp16 CUDA tensors with head_dim 32/64/128/256 "
                           "(there is no CPU or fp32 path)")
    _fused(q, k, wq, wk, eps, cos, sin)
