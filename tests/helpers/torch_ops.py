"""The reference's torch formulas of the DiT block's operators -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.

The product block (`minimax_h3_turbo_b200.h3.block`) runs only on this library's kernels (bf16/fp16 CUDA).  The tests
need the same block on CPU ranks (the gloo sharding tests), in fp32 on the dequantized weights (the accuracy checks),
and the reference's own torch forms to compare the kernels with.  `TorchOps` provides them, restated from the
reference:

  rms / scale_shift_ / gate_        h3turbo/h3/model.py:_rms :64-66, _scale_shift_ :106-109, _gate_ :111-115
  rms_norm_fused_order / rope       h3turbo/h3/layout.py:309-356 ("torch" form; "eager" is ComfyUI's portable form)
  attention / attention_lse / merge torch SDPA on CUDA, the explicit fp32 softmax elsewhere; log-sum-exp merge in fp32
Pass `ops=TorchOps()` to `DiTBlock`.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch
import torch.nn.functional as F


def rms(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """F.rms_norm over the last dim with the weight in x.dtype (model.py:64-66)."""
    return F.rms_norm(x, (x.shape[-1],), weight if weight.dtype == x.dtype else weight.to(x.dtype), eps)


def scale_shift_(h: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, segments: Sequence) -> torch.Tensor:
    for a, b, row in segments:
        if b > a:
            h[a:b].mul_(1.0 + scale[row].to(h.dtype)).add_(shift[row].to(h.dtype))
    return h


def rms_modulate(x, weight, eps, shift, scale, segments):
    return scale_shift_(rms(x, weight, eps), shift, scale, segments)


def gate_(x, gate, other, segments):
    for a, b, row in segments:
        if b > a:
            x[a:b].addcmul_(other[a:b], gate[row].to(x.dtype))
    return x


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


@torch.no_grad()
def norm_rope_(q, k, wq, wk, eps, cos, sin, impl: str = "torch", chunk: int = 1024) -> None:
    """The reference's torch ("torch": bit-exact fused order; "eager": ComfyUI's portable form, also used for fp32)
    per-head RMSNorm + split-half RoPE, in place (layout.py:329-356)."""
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


def attention_lse(q, k, v) -> Tuple[torch.Tensor, torch.Tensor]:
    """(o, lse) of softmax attention, fp32 math (cuDNN's fused kernel for bf16 CUDA tensors)."""
    if q.is_cuda and q.dtype == torch.bfloat16:
        r = torch.ops.aten._scaled_dot_product_cudnn_attention(q, k, v, None, True)
        return r[0], r[1].reshape(q.shape[:-1]).to(torch.float32)
    sc = torch.matmul(q.float(), k.float().transpose(-1, -2)) * (q.shape[-1] ** -0.5)
    lse = torch.logsumexp(sc, dim=-1)
    return torch.matmul(torch.exp(sc - lse.unsqueeze(-1)), v.float()).to(q.dtype), lse


def merge_attention(acc: Optional[torch.Tensor], acc_lse: Optional[torch.Tensor], o: torch.Tensor,
                    lse: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Combine attention over disjoint key sets: softmax weights renormalised by the log-sum-exps, in fp32 (an empty
    key set, lse -inf, has weight 0)."""
    if acc is None:
        return o.float(), lse
    new = torch.logaddexp(acc_lse, lse)
    safe = torch.where(torch.isinf(new), torch.zeros_like(new), new)
    wa = torch.where(torch.isinf(acc_lse), torch.zeros_like(new), torch.exp(acc_lse - safe))
    wb = torch.where(torch.isinf(lse), torch.zeros_like(new), torch.exp(lse - safe))
    acc = acc * wa.unsqueeze(-1) + o.float() * wb.unsqueeze(-1)
    return acc, new


class TorchMerger:
    def __init__(self, heads, queries, head_dim, device):
        self.h, self.s, self.d = heads, queries, head_dim
        self.acc = self.lse = None

    def add(self, o, lse, last=False):
        self.acc, self.lse = merge_attention(self.acc, self.lse, o, lse.reshape(1, self.h, self.s))
        if last:
            return self.acc[0].transpose(0, 1).reshape(self.s, self.h * self.d).to(o.dtype)
        return None


class TorchOps:
    """The block's operators as the reference's torch formulas (any device, any float dtype)."""

    rms_modulate = staticmethod(rms_modulate)
    gate_ = staticmethod(gate_)

    @staticmethod
    def norm_rope_(q, k, wq, wk, eps, cos, sin):
        norm_rope_(q, k, wq, wk, eps, cos, sin, impl="torch")

    @staticmethod
    def attention(q, k, v):
        return F.scaled_dot_product_attention(q, k, v)  # what the reference's _attention calls (model.py:196-228)

    attention_lse = staticmethod(attention_lse)

    @staticmethod
    def merger(heads, queries, head_dim, device):
        return TorchMerger(heads, queries, head_dim, device)
