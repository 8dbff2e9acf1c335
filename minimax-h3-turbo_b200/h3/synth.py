"""Seeded synthetic W4A8 layers and activations for benchmarks, built on the GPU with torch.

The benchmark configurations quote "symmetric int4, group 128, fp16 scales, then ConvRot" weights; this maps that onto
the reference's W4A8Weight format (types.py:10-47):
  1. W ~ N(0, 0.02) fp32 [N, K]
  2. W_rot = W @ H per 256-block (the ConvRot basis; H is symmetric and involutory)
  3. per (row, 128-group): sc = max|W_rot| / 7, code = clamp(rint(W_rot / sc), -7, 7), nibble = code + 8, codebook i - 8
  4. s_ch[n] = max_g sc[n, g] * 7 / 127 (fp32), s_rel = fp16(sc / s_ch), so |codebook * s_rel| reaches ~127
  5. q[n, j] = nibble[n, 2j] | nibble[n, 2j + 1] << 4
Activations: x ~ N(0, 1) with a fraction of outlier channels scaled x20, cast to bf16.  Generation is chunked over rows
so 13824 x 27648 layers need no more than a few hundred MB of temporaries.
"""
from __future__ import annotations

from typing import Optional

import torch

from .qlinear import hadamard_regular
from .types import W4A8Weight


@torch.no_grad()
def synthetic_w4a8(n: int, k: int, *, group: int = 128, convrot: int = 256, seed: int = 0, device="cuda",
                   rows_per_chunk: int = 2048) -> W4A8Weight:
    if k % group or k % convrot:
        raise ValueError("K must be a multiple of the group size and the ConvRot block")
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed)
    h = hadamard_regular(convrot, dev, torch.float32)
    q = torch.empty(n, k // 2, dtype=torch.int8, device=dev)
    s_rel = torch.empty(n, k // group, dtype=torch.float16, device=dev)
    s_ch = torch.empty(n, dtype=torch.float32, device=dev)
    for r0 in range(0, n, rows_per_chunk):
        r1 = min(n, r0 + rows_per_chunk)
        w = torch.randn(r1 - r0, k, generator=gen, device=dev) * 0.02
        w_rot = (w.view(r1 - r0, k // convrot, convrot) @ h).view(r1 - r0, k // group, group)
        sc = (w_rot.abs().amax(-1) / 7.0).clamp_min(1e-12)
        code = torch.clamp(torch.round(w_rot / sc[..., None]), -7, 7).to(torch.int32).view(r1 - r0, k) + 8
        ch = sc.amax(-1) * (7.0 / 127.0)
        s_ch[r0:r1] = ch
        s_rel[r0:r1] = (sc / ch[:, None]).to(torch.float16)
        q[r0:r1] = (code[:, 0::2] | (code[:, 1::2] << 4)).to(torch.uint8).view(torch.int8)
    codebook = torch.arange(16, dtype=torch.float32, device=dev) - 8.0
    return W4A8Weight(q, s_rel, s_ch, codebook, group_size=group, convrot=convrot)


@torch.no_grad()
def synthetic_w4a8_fp8(n: int, k: int, *, seed: int = 0, device="cuda") -> W4A8Weight:
    """A seeded layer in the real checkpoints' format (h3turbo/h3/types.py:10-47): random 4-bit codebook indices, fp8
    e4m3 group scales per 16 weights drawn from [20, 200] (so |level| reaches the +-127 clamp), a 16-level codebook in
    [-1, 1] and fp32 per-channel scales -- the shape of the reference's own test weights (tests/test_h3_qlinear.py:46-53)."""
    if k % 256:
        raise ValueError("K must be a multiple of 256 (the ConvRot block)")
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randint(-128, 128, (n, k // 2), generator=gen, device=dev, dtype=torch.int8)
    s_rel = (torch.rand(n, k // 16, generator=gen, device=dev) * 180 + 20).to(torch.float8_e4m3fn)
    s_ch = torch.rand(n, generator=gen, device=dev) * 0.02 + 0.005
    return W4A8Weight(q, s_rel, s_ch, torch.linspace(-1.0, 1.0, 16, device=dev), group_size=16, convrot=256)


@torch.no_grad()
def synthetic_activation(m: int, k: int, *, outlier_frac: float = 0.005, n_outliers: Optional[int] = None, seed: int = 0,
                         dtype: torch.dtype = torch.bfloat16, device="cuda") -> torch.Tensor:
    dev = torch.device(device)
    gen = torch.Generator(device=dev).manual_seed(seed + 1000)
    x = torch.randn(m, k, generator=gen, device=dev, dtype=torch.float32)
    cnt = n_outliers if n_outliers is not None else max(1, round(outlier_frac * k))
    ch = torch.randperm(k, generator=gen, device=dev)[:cnt]
    x[:, ch] *= 20.0
    return x.to(dtype)


def synthetic_store_tensors(cfg, *, group: int = 128, scale_dtype: str = "fp16", seed: int = 0, with_globals: bool = True,
                            device="cpu"):
    """Seeded random h3t tensors (ComfyUI-layout names) for a store of cfg.layers W4A8 blocks, each produced lazily while
    it is written.  Weights are random packed nibbles; group scales fp16 in [8, 15] with the integer codebook (levels up
    to +-120), or fp8 e4m3 in [20, 200] with a 16-level codebook in [-1, 1] (the real checkpoints' format).  `device`:
    where the random linear-layer tensors are drawn (a GPU generates multi-GB stores fast); they are written from host
    copies, and the values depend on the device."""
    from .writer import LazySource

    hid, inner, ffn, hd = cfg.hidden, cfg.inner, cfg.ffn, cfg.head_dim
    fp8 = scale_dtype == "fp8"
    cb = torch.linspace(-1.0, 1.0, 16) if fp8 else torch.arange(16, dtype=torch.float32) - 8.0
    linears = {"attn.qkv_proj": (3 * inner, hid), "attn.out_proj": (hid, inner), "mlp.fc1": (2 * ffn, hid), "mlp.fc2": (hid, ffn)}
    out = {}

    dev = torch.device(device)

    def gen(i: int, salt: int, on=None):
        return torch.Generator(device=on or "cpu").manual_seed(seed * 100003 + i * 97 + salt)

    for i in range(cfg.layers):
        for j, (name, (n, k)) in enumerate(linears.items()):
            p = f"blocks.{i}.{name}."
            out[p + "weight"] = LazySource("I8", (n, k // 2), lambda i=i, j=j, n=n, k=k: torch.empty(n, k // 2, dtype=torch.uint8, device=dev).random_(generator=gen(i, j, dev)).view(torch.int8).cpu())
            if fp8:
                out[p + "weight_s_rel"] = LazySource("F8_E4M3", (n, k // group), lambda i=i, j=j, n=n, k=k: (torch.rand(n, k // group, generator=gen(i, 10 + j, dev), device=dev) * 180 + 20).to(torch.float8_e4m3fn).cpu())
            else:
                out[p + "weight_s_rel"] = LazySource("F16", (n, k // group), lambda i=i, j=j, n=n, k=k: (torch.rand(n, k // group, generator=gen(i, 10 + j, dev), device=dev) * 7 + 8).to(torch.float16).cpu())
            out[p + "weight_s_channel"] = LazySource("F32", (n,), lambda i=i, j=j, n=n: torch.rand(n, generator=gen(i, 20 + j)) * 4e-4 + 1e-4)
            out[p + "weight_codebook"] = cb.clone()
            out[p + "comfy_quant"] = torch.frombuffer(bytearray(f'{{"format":"w4a8_int8","group_size":{group}}}'.encode()), dtype=torch.uint8).clone()
        for nm, size in (("norm1.weight", hid), ("norm2.weight", hid), ("attn.q_norm.weight", hd), ("attn.k_norm.weight", hd)):
            out[f"blocks.{i}.{nm}"] = (1.0 + 0.1 * torch.randn(size, generator=gen(i, 30))).to(torch.bfloat16)
    if with_globals:
        g = torch.Generator().manual_seed(seed + 7)
        vp, ac = cfg.video_patch_dim, cfg.audio_channels
        glob = {"video_patch_proj.weight": (hid, vp), "video_patch_proj.bias": (hid,), "audio_patch_proj.weight": (hid, ac),
                "audio_patch_proj.bias": (hid,), "condition_proj.weight": (hid, cfg.text_dim), "condition_proj.bias": (hid,),
                "rope.inv_freq": (cfg.rope_inv_freq_len,), "final_layer.norm.weight": (hid,),
                "final_layer.adaln_proj.linear.weight": (2 * hid, cfg.t_dim), "final_layer.adaln_proj.linear.bias": (2 * hid,),
                "final_layer.video_out.weight": (vp, hid), "final_layer.video_out.bias": (vp,),
                "final_layer.audio_out.weight": (ac, hid), "final_layer.audio_out.bias": (ac,)}
        for nm, shape in glob.items():
            dt = torch.bfloat16 if nm in ("condition_proj.weight", "final_layer.norm.weight", "final_layer.adaln_proj.linear.weight") else torch.float32
            out[nm] = (0.02 * torch.randn(*shape, generator=g)).to(dt)
    return out
