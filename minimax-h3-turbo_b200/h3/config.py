"""Architecture record of the official H3 DiT (config.py:11-85 of the reference): the same fields and JSON form, because
h3t files store it in their metadata and both implementations must read each other's files."""
from __future__ import annotations

import json
from dataclasses import asdict, dataclass
from typing import Tuple


@dataclass(frozen=True)
class H3Config:
    hidden: int = 5376
    layers: int = 50
    refiner_layers: int = 2
    heads: int = 56
    head_dim: int = 128
    ffn: int = 14336  # SwiGLU width; fc1 emits 2 * ffn
    video_channels: int = 24
    audio_channels: int = 32
    patch: Tuple[int, int, int] = (1, 2, 2)
    text_dim: int = 5120
    t_dim: int = 8
    curve_grid: int = 1025
    rope_inv_freq_len: int = 16
    norm_eps: float = 1e-5
    qk_norm_eps: float = 1e-5
    final_norm_eps: float = 1e-5
    sigma_shift_video: float = 12.0
    sigma_shift_audio: float = 3.0
    quant_group: int = 16  # weights per group scale
    quant_convrot: int = 256  # ConvRot (regular Hadamard) block along K

    @property
    def video_patch_dim(self) -> int:
        return self.video_channels * self.patch[0] * self.patch[1] * self.patch[2]

    @property
    def inner(self) -> int:
        return self.heads * self.head_dim

    def to_json(self) -> str:
        return json.dumps(asdict(self), sort_keys=True)

    @classmethod
    def from_json(cls, s: str) -> "H3Config":
        d = json.loads(s)
        d["patch"] = tuple(d["patch"])
        return cls(**d)
