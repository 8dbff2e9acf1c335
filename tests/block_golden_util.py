"""Loads tests/golden/block_golden.npz (one H3 DiT block produced by the reference's own code) into torch tensors."""
from pathlib import Path

import numpy as np
import torch

from minimax_h3_turbo_b200.h3 import block as blk
from minimax_h3_turbo_b200.h3.types import BlockWeights, W4A8Weight

PATH = Path(__file__).resolve().parent / "golden" / "block_golden.npz"


def bf16(a: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(a.astype(np.uint16).view(np.int16).copy()).view(torch.bfloat16)


def load(device="cpu"):
    with np.load(PATH) as z:
        g = {k: z[k] for k in z.files}
    lin = {nm: W4A8Weight(torch.from_numpy(g[f"{nm}/q"]).to(device), torch.from_numpy(g[f"{nm}/s_rel"]).to(device),
                          torch.from_numpy(g[f"{nm}/s_ch"]).to(device), torch.from_numpy(g[f"{nm}/cb"]).to(device), 128, 256)
           for nm in ("qkv", "out", "fc1", "fc2")}
    w = BlockWeights(**lin, **{nm: bf16(g[nm]).to(device) for nm in ("norm1", "norm2", "q_norm", "k_norm")})
    mod = blk.Modulation(*(bf16(g["mod"][i]).to(device) for i in range(6)))
    segs = [tuple(int(v) for v in row) for row in g["segments"]]
    hid, heads, hd, ffn, f = (int(v) for v in g["dims"])
    t = {k: bf16(g[k]).to(device) for k in ("x", "h1", "qkv", "qkv_normed", "x_mid", "h2", "y", "cos", "sin")}
    return w, mod, segs, (hid, heads, hd, ffn), [float(e) for e in g["eps"]], t
