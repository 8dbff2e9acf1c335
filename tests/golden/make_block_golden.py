"""Generate golden vectors of one H3 DiT block from the REFERENCE's own block code (CPU, qlinear backend "torch", a8/ck,
q/k norm + RoPE in its exact "torch" form) and store inputs, intermediates and output in tests/golden/block_golden.npz.

The block body is the reference's `H3Model._block` (h3turbo/h3/model.py:234-242) with the AdaLN modulation rows given
directly (the benchmark precomputes them); `_attention` (:196-228) and `_mlp` (:186-194) are the reference's methods,
bound to a small stand-in object that carries the attributes they read, so no checkpoint or engine is needed.

This script needs the reference source tree (argv[1]); it runs once on a machine that has it and the .npz is committed.
Usage:  python tests/golden/make_block_golden.py /path/to/reference
"""
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))  # repo root, for the oracle's synthetic weight generator

HID, HEADS, HD, FFN, F_ROPE = 256, 2, 128, 512, 16
FRAMES, PH, PW, AUDIO = 5, 4, 4, 16  # 80 video tokens + 16 audio tokens


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main(ref_root: str) -> None:
    sys.path.insert(0, ref_root)
    from h3turbo.h3 import layout as lay  # noqa: E402  (the reference)
    from h3turbo.h3 import model as mdl  # noqa: E402
    from h3turbo.h3.config import H3Config  # noqa: E402
    from h3turbo.h3.types import BlockWeights, W4A8Weight  # noqa: E402
    from oracle import qlinear_oracle as orc

    torch.manual_seed(0)
    torch.set_num_threads(8)
    bf = torch.bfloat16
    cfg = H3Config(hidden=HID, layers=1, refiner_layers=0, heads=HEADS, head_dim=HD, ffn=FFN, rope_inv_freq_len=F_ROPE,
                   quant_group=128)
    out = {}
    lin = {}
    for j, (name, (n, k)) in enumerate({"qkv": (3 * HID, HID), "out": (HID, HID), "fc1": (2 * FFN, HID),
                                        "fc2": (HID, FFN)}.items()):
        q, s_rel, s_ch, cb = orc.synth_weight_int4_g128(n, k, seed=50 + j)
        lin[name] = W4A8Weight(torch.from_numpy(q), torch.from_numpy(s_rel), torch.from_numpy(s_ch), torch.from_numpy(cb), 128, 256)
        out[f"{name}/q"], out[f"{name}/s_rel"], out[f"{name}/s_ch"], out[f"{name}/cb"] = q, s_rel, s_ch, cb
    g = torch.Generator().manual_seed(1)
    norms = {nm: (1.0 + 0.1 * torch.randn(size, generator=g)).to(bf) for nm, size in
             (("norm1", HID), ("norm2", HID), ("q_norm", HD), ("k_norm", HD))}
    for nm, t in norms.items():
        out[nm] = bits(t)
    w = BlockWeights(qkv=lin["qkv"], out=lin["out"], fc1=lin["fc1"], fc2=lin["fc2"], **norms)
    mods = [(0.5 * torch.randn(2, HID, generator=g)).to(bf) for _ in range(6)]  # sh_a, sc_a, g_a, sh_m, sc_m, g_m
    out["mod"] = np.stack([bits(m) for m in mods])
    s = FRAMES * PH * PW + AUDIO
    segments = [(0, FRAMES * PH * PW, 0), (FRAMES * PH * PW, s, 1)]
    out["segments"] = np.array(segments, dtype=np.int64)
    t = torch.arange(FRAMES).view(-1, 1, 1).expand(FRAMES, PH, PW)
    yy = torch.arange(PH).view(1, -1, 1).expand(FRAMES, PH, PW)
    xx = torch.arange(PW).view(1, 1, -1).expand(FRAMES, PH, PW)
    pos = torch.cat([torch.stack([t, yy, xx], -1).reshape(-1, 3),
                     torch.stack([torch.arange(AUDIO), torch.zeros(AUDIO, dtype=torch.long), torch.zeros(AUDIO, dtype=torch.long)], -1)])
    inv_freq = 1.0 / (10000.0 ** (torch.arange(F_ROPE, dtype=torch.float32) / F_ROPE))
    ang = lay.rope_angles(pos, inv_freq, "cpu")
    cos, sin = torch.cos(ang).to(bf), torch.sin(ang).to(bf)
    out["cos"], out["sin"] = bits(cos), bits(sin)
    x = torch.from_numpy(orc.synth_activation(s, HID, seed=5, n_outliers=3).view(np.int16)).view(bf)
    out["x"] = bits(x)

    obj = types.SimpleNamespace(cfg=cfg, backend="torch", precision="a8", mlp_chunk=None, attn_chunk=None,
                                rope_chunk=1024, rope_impl="torch", _sdpa_prio=None, _int8_attention=None, dtype=bf)
    for meth in ("_matmul", "_attention", "_mlp"):
        setattr(obj, meth, types.MethodType(getattr(mdl.H3Model, meth), obj))
    eps = cfg.norm_eps
    sh_a, sc_a, g_a, sh_m, sc_m, g_m = mods
    with torch.no_grad():
        # the reference's _block body (model.py:239-242) on the given modulation rows
        h1 = mdl._scale_shift_(mdl._rms(x, w.norm1, eps), sh_a, sc_a, segments)
        qkv = obj._matmul(h1, w.qkv)
        qkv_normed = qkv.clone()
        q, k, _ = (u.view(s, HEADS, HD) for u in qkv_normed.split(HEADS * HD, dim=-1))
        lay.norm_rope_(q, k, w.q_norm, w.k_norm, cfg.qk_norm_eps, cos, sin, impl="torch")
        xb = x.clone()
        mdl._gate_(xb, g_a, obj._attention(h1, w, (cos, sin, None)), segments)
        x_mid = xb.clone()
        h2 = mdl._scale_shift_(mdl._rms(xb, w.norm2, eps), sh_m, sc_m, segments)
        y = mdl._gate_(xb, g_m, obj._mlp(h2, w), segments)
    out.update({"h1": bits(h1), "qkv": bits(qkv), "qkv_normed": bits(qkv_normed), "x_mid": bits(x_mid), "h2": bits(h2),
                "y": bits(y), "dims": np.array([HID, HEADS, HD, FFN, F_ROPE], dtype=np.int64),
                "eps": np.array([cfg.norm_eps, cfg.qk_norm_eps], dtype=np.float64)})
    np.savez_compressed(HERE / "block_golden.npz", **out)
    print("wrote", HERE / "block_golden.npz", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main(sys.argv[1])
