"""Data contracts shared by the qlinear ops, the weight store and the block streamer.

These mirror `h3turbo/h3/types.py` of the reference field for field (same names, order and defaults), because they are
the drop-in interface: a caller that builds `W4A8Weight(q, s_rel, s_ch, codebook, group_size, convrot)` or hands a
`BlockProvider` to the model must not notice which implementation it talks to.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Protocol, Union

import torch


@dataclass
class W4A8Weight:
    """A ConvRot W4A8 linear weight (out = x @ W^T); all tensors on one device.

    The weight in the rotated basis is grid[n, k] * s_ch[n] with
        grid[n, k] = clamp(rint(codebook[nib[n, k]] * s_rel[n, k // group_size]), -127, 127)
    where nib[n, 2j] / nib[n, 2j + 1] are the low / high nibble of byte q[n, j]; activations are rotated by the same
    block Hadamard (block `convrot`) before the int8 product.  Reference: types.py:10-47.
    """

    q: torch.Tensor  # int8 (or uint8) [N, K // 2], packed nibbles
    s_rel: torch.Tensor  # [N, K // group_size]: float8_e4m3fn (real checkpoints) or fp16 / bf16 / fp32
    s_ch: torch.Tensor  # fp32 [N]
    codebook: torch.Tensor  # fp32 [16]
    group_size: int = 16
    convrot: int = 256

    @property
    def out_features(self) -> int:
        return self.q.shape[0]

    @property
    def in_features(self) -> int:
        return self.q.shape[1] * 2

    @property
    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.q, self.s_rel, self.s_ch, self.codebook))

    def to(self, device, non_blocking: bool = False) -> "W4A8Weight":
        mv = lambda t: t.to(device, non_blocking=non_blocking)  # noqa: E731
        return W4A8Weight(mv(self.q), mv(self.s_rel), mv(self.s_ch), mv(self.codebook), self.group_size, self.convrot)


Weight = Union[W4A8Weight, torch.Tensor]  # a W4A8 layer or a dense [N, K] matrix


@dataclass
class BlockWeights:
    """The tensors of one DiT block on the compute device (types.py:54-68)."""

    qkv: Weight  # [3 * inner, hidden]
    out: Weight  # [hidden, inner]
    fc1: Weight  # [2 * ffn, hidden] (SwiGLU: gate then up)
    fc2: Weight  # [hidden, ffn]
    norm1: torch.Tensor  # [hidden]
    norm2: torch.Tensor  # [hidden]
    q_norm: torch.Tensor  # [head_dim]
    k_norm: torch.Tensor  # [head_dim]
    adaln_w: Optional[torch.Tensor] = None  # [6 * hidden * 3, t_dim]; None for refiner blocks
    adaln_b: Optional[torch.Tensor] = None  # [6 * hidden * 3]


@dataclass
class GlobalWeights:
    """Non-block tensors of the DiT (types.py:70-90); small and always resident."""

    video_patch_w: torch.Tensor
    video_patch_b: torch.Tensor
    audio_patch_w: torch.Tensor
    audio_patch_b: torch.Tensor
    condition_w: torch.Tensor
    condition_b: torch.Tensor
    adaln_t_table: Optional[torch.Tensor]
    rope_inv_freq: torch.Tensor
    final_norm: torch.Tensor
    final_adaln_w: torch.Tensor
    final_adaln_b: torch.Tensor
    video_out_w: torch.Tensor
    video_out_b: torch.Tensor
    audio_out_w: torch.Tensor
    audio_out_b: torch.Tensor
    refiner: List[BlockWeights] = field(default_factory=list)
    refiner_final_norm: Optional[torch.Tensor] = None


class BlockProvider(Protocol):
    """Supplies block i's weights on the compute device (types.py:93-107).

    Per forward the model calls begin_forward(); then for each block acquire(i) (may wait for an in-flight copy) ...
    release(i); then end_forward().  A resident provider returns the same objects every time.
    """

    def begin_forward(self) -> None: ...

    def acquire(self, i: int) -> BlockWeights: ...

    def release(self, i: int) -> None: ...

    def end_forward(self) -> None: ...
