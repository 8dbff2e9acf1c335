"""CPU oracle for the W4A8 ConvRot quantised linear -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.

A numpy restatement of the reference's portable CPU path, `h3turbo/h3/qlinear.py` with `backend="torch"` and
`quant_mode="ck"` (or "eager"), the numerics the reference pins as its CUDA kernel's profile
(`tests/test_h3_qlinear.py:337-349`).  Each function names the reference lines it restates.

Only `tests/`, `__graft_entry__.smoke()` and the CPU legs of `bench.py` (`cpu_baseline`, `--impl reference`) may import
this module, and only as the checker or as the timed CPU baseline.  The product path (the `minimax_h3_turbo_b200`
package and `libh3b.so`) never imports it.

Parity is pinned: `tests/golden/make_golden.py` runs the reference itself on seeded inputs and stores its outputs in
`tests/golden/*.npz`; `tests/test_oracle_golden.py` checks this module against every one of them bit for bit.

Dtype conventions.  numpy has no bfloat16, so a bf16 array is carried as its uint16 bit pattern; fp16 is np.float16 and
fp32 np.float32.  Every rounding step of the reference is made explicit: `_to_dt` is "round an fp32 value to the
activation dtype" (round to nearest even, as torch's casts do).
"""
from __future__ import annotations

import math
from typing import Optional, Tuple

import numpy as np

CONVROT = 256  # h3turbo/h3/qlinear.py:30
EPS_SCALE = np.float32(1e-30)  # qlinear.py:35, the per-row scale floor
EXACT_K = 1024  # qlinear.py:36, K chunk of the exact fp32 integer GEMM
_H4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=np.float64)  # qlinear.py:31

DTYPES = ("bf16", "fp16", "fp32")


# ----------------------------------------------------------------------------------------------------------- dtypes
def bf16_bits_from_f32(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit pattern, round to nearest even; NaN stays a quiet NaN (torch's c10::BFloat16 rounding)."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    with np.errstate(over="ignore"):
        r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)  # wraps only for NaN payloads, fixed below
    nan = np.isnan(a)
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def f32_from_bf16_bits(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def to_f32(x: np.ndarray, dt: str) -> np.ndarray:
    """Values of an activation array of dtype `dt` as fp32 (exact)."""
    if dt == "bf16":
        return f32_from_bf16_bits(x)
    return np.asarray(x).astype(np.float32)


def from_f32(a: np.ndarray, dt: str) -> np.ndarray:
    """fp32 values rounded once to `dt`, in that dtype's storage form."""
    if dt == "bf16":
        return bf16_bits_from_f32(a)
    if dt == "fp16":
        return np.asarray(a, dtype=np.float32).astype(np.float16)
    return np.asarray(a, dtype=np.float32)


def _to_dt(a: np.ndarray, dt: str) -> np.ndarray:
    """Round fp32 values to `dt` and return them as fp32 again (the value a torch tensor of that dtype holds)."""
    return to_f32(from_f32(a, dt), dt)


_TINY = {"bf16": np.float32(2.0 ** -126), "fp16": np.float32(2.0 ** -14), "fp32": np.float32(2.0 ** -126)}  # torch.finfo(dt).tiny


def fp8_e4m3fn_table() -> np.ndarray:
    """fp32 value of each of the 256 OCP E4M3FN bytes (bias 7, subnormals below 2^-6, S.1111.111 is NaN, no infinities).
    The format the reference stores group scales in (`h3turbo/h3/types.py:21`)."""
    out = np.empty(256, dtype=np.float32)
    for b in range(256):
        sign = -1.0 if b & 0x80 else 1.0
        e, m = (b >> 3) & 0xF, b & 7
        if e == 0xF and m == 7:
            out[b] = np.nan
        elif e == 0:
            out[b] = sign * (m / 8.0) * 2.0 ** -6
        else:
            out[b] = sign * (1 + m / 8.0) * 2.0 ** (e - 7)
    return out


_FP8 = fp8_e4m3fn_table()


# ----------------------------------------------------------------------------------------------------------- Hadamard
def hadamard_regular(size: int) -> np.ndarray:
    """kron(H4, ..., H4) / sqrt(size) in fp64 (qlinear.py:44-66): symmetric, involutory, entries +-2^-j."""
    n = size
    while n > 1 and n % 4 == 0:
        n //= 4
    if size < 4 or n != 1:
        raise ValueError(f"regular Hadamard size must be a power of 4 (>= 4), got {size}")
    h = _H4
    while h.shape[0] < size:
        h = np.kron(h, _H4)
    return h / math.sqrt(size)


def rot32(xf: np.ndarray, size: int = CONVROT) -> np.ndarray:
    """Per-`size`-block x @ H accumulated in fp64 and rounded once to fp32: the reference's CPU rotation
    (qlinear.py:105-115).  For bf16/fp16 inputs every fp64 partial sum is exact, so this is the correctly rounded value."""
    m, k = xf.shape
    if k % size:
        raise ValueError(f"last dim {k} is not a multiple of the rotation block {size}")
    h = hadamard_regular(size)
    y = np.matmul(xf.astype(np.float64).reshape(m, k // size, size), h)
    return y.reshape(m, k).astype(np.float32)


# ----------------------------------------------------------------------------------------------------------- quantiser
def quantize_rows(x: np.ndarray, dt: str, size: int = CONVROT, mode: str = "ck") -> Tuple[np.ndarray, np.ndarray]:
    """Rotate + per-row int8 quantisation, `_quantize_rows` (qlinear.py:267-292).

    mode "ck": absmax of the UNROUNDED fp32 rotation; "eager": absmax of the rotation rounded to `dt`.  Both divide the
    dt-rounded rotation by the dt-rounded scale in fp32, round the quotient to dt, round half-to-even, clamp to
    [-128, 127].  Returns (int8 [M, K], fp32 scale [M])."""
    if mode not in ("ck", "eager"):
        raise ValueError(f"quant_mode must be 'ck' or 'eager', got {mode!r}")
    xf = to_f32(x, dt)
    m, k = xf.shape
    if m == 0:
        return np.zeros((0, k), np.int8), np.zeros((0,), np.float32)
    y32 = rot32(xf, size)
    y = _to_dt(y32, dt) if dt != "fp32" else y32
    src = y32 if mode == "ck" else y
    amax = np.max(np.abs(src), axis=1)
    xs = np.maximum((amax / np.float32(127.0)).astype(np.float32), EPS_SCALE)  # qlinear.py:288
    s = _to_dt(xs, dt) if dt != "fp32" else xs  # qlinear.py:289
    s = np.where(s == 0, _TINY[dt], s).astype(np.float32)  # qlinear.py:290
    with np.errstate(invalid="ignore", over="ignore", divide="ignore"):
        qv = (y / s[:, None]).astype(np.float32)  # fp32 quotient of dt values
        qv = _to_dt(qv, dt) if dt != "fp32" else qv  # the quotient lives in a dt tensor
        qv = np.clip(np.rint(qv), -128, 127)  # round_() half-to-even, clamp_ (qlinear.py:291)
        q = np.where(np.isnan(qv), 0, qv).astype(np.int8)
    return q, xs


# ----------------------------------------------------------------------------------------------------------- weights
def check_weight(q: np.ndarray, s_rel: np.ndarray, s_ch: np.ndarray, codebook: np.ndarray, group: int, convrot: int) -> Tuple[int, int]:
    """`_check_weight` (qlinear.py:140-154)."""
    if q.ndim != 2 or q.dtype not in (np.int8, np.uint8):
        raise ValueError(f"W4A8 q must be a 2D int8 tensor, got {q.shape} {q.dtype}")
    n, k = q.shape[0], q.shape[1] * 2
    gs, cr = group, convrot
    if gs < 4 or k % 16 or k % gs or k % cr or (16 % gs and gs % 16):
        raise ValueError(f"K={k} must be divisible by 16, group_size={gs} and convrot={cr}; group_size >= 4 dividing 16 or a multiple of 16")
    if tuple(s_rel.shape) != (n, k // gs):
        raise ValueError(f"s_rel must have shape {(n, k // gs)}, got {tuple(s_rel.shape)}")
    if tuple(s_ch.shape) != (n,):
        raise ValueError(f"s_ch must have shape {(n,)}, got {tuple(s_ch.shape)}")
    if tuple(codebook.shape) != (16,):
        raise ValueError(f"codebook must have shape (16,), got {tuple(codebook.shape)}")
    return n, k


def scale_values(s_rel: np.ndarray, s_kind: str) -> np.ndarray:
    """Group scales as fp32.  s_kind: "fp8" (raw E4M3FN bytes, uint8), "fp16", "bf16" (uint16 bits) or "fp32"."""
    if s_kind == "fp8":
        return _FP8[np.asarray(s_rel, dtype=np.uint8)]
    if s_kind == "bf16":
        return f32_from_bf16_bits(s_rel)
    return np.asarray(s_rel).astype(np.float32)


def decode_int8_grid(q: np.ndarray, s_rel: np.ndarray, s_kind: str, codebook: np.ndarray, group: int) -> np.ndarray:
    """int4 codebook indices -> the exact int8 grid (qlinear.py:157-204): nibble 2j is the LOW nibble of byte j
    (types.py:14-16); level = clamp(rint(fp32(codebook[nibble]) * fp32(scale)), -127, 127), half-to-even.
    A NaN product decodes to 0 (the fp8 table's nan_to_num, qlinear.py:162)."""
    qb = np.asarray(q).view(np.uint8)
    n, kh = qb.shape
    k = kh * 2
    code = np.empty((n, k), dtype=np.int64)
    code[:, 0::2] = qb & 0xF
    code[:, 1::2] = qb >> 4
    cb = np.asarray(codebook, dtype=np.float32)
    sv = scale_values(s_rel, s_kind).reshape(n, k // group, 1)
    with np.errstate(invalid="ignore", over="ignore"):
        prod = (cb[code].reshape(n, k // group, group) * sv).astype(np.float32)
        lv = np.clip(np.rint(prod), -127, 127)
    lv = np.where(np.isnan(lv), 0, lv)
    return lv.reshape(n, k).astype(np.int8)


# ----------------------------------------------------------------------------------------------------------- GEMM
def int8_mm(a: np.ndarray, w8: np.ndarray) -> np.ndarray:
    """Exact int32 a[M, K] @ w8[N, K]^T, restating the reference's CPU emulation (qlinear.py:236-254): fp32 GEMMs over
    K chunks of 1024, where every partial sum is an integer below 2^24, accumulated in int32."""
    m, k = a.shape
    n = w8.shape[0]
    acc = np.zeros((m, n), dtype=np.int32)
    if m == 0 or n == 0 or k == 0:
        return acc
    for k0 in range(0, k, EXACT_K):
        part = np.matmul(a[:, k0:k0 + EXACT_K].astype(np.float32), w8[:, k0:k0 + EXACT_K].astype(np.float32).T)
        acc += part.astype(np.int32)
    return acc


def epilogue(acc: np.ndarray, xs: np.ndarray, s_ch: np.ndarray, bias: Optional[np.ndarray], out_dt: str,
             mode: str = "ck", bias_dt: Optional[str] = None) -> np.ndarray:
    """`_TorchRunner._a8` epilogue (qlinear.py:396-405).  "ck": out = dt((fp32(acc) * xs) * s_ch); "eager":
    dt(fp32(acc) * (xs * s_ch)).  The bias is cast to out_dtype first and added after the output rounding (a second
    rounding).  Returns the output in out_dt's storage form."""
    accf = acc.astype(np.float32)
    xs = np.asarray(xs, dtype=np.float32).reshape(-1, 1)
    ws = np.asarray(s_ch, dtype=np.float32).reshape(1, -1)
    with np.errstate(over="ignore", invalid="ignore"):
        if mode == "ck":
            o = ((accf * xs).astype(np.float32) * ws).astype(np.float32)
        else:
            o = (accf * (xs * ws).astype(np.float32)).astype(np.float32)
        o = _to_dt(o, out_dt) if out_dt != "fp32" else o
        if bias is not None:
            b = to_f32(bias, bias_dt or out_dt)
            b = _to_dt(b, out_dt) if out_dt != "fp32" else b  # bias.to(out_dtype), qlinear.py:405
            o = (o + b.reshape(1, -1)).astype(np.float32)
            o = _to_dt(o, out_dt) if out_dt != "fp32" else o
    return from_f32(o, out_dt)


def swiglu(x: np.ndarray, dt: str) -> np.ndarray:
    """silu(gate) * up on [gate | up] halves in `dt` (qlinear.py:376-379): silu computed in fp32 and rounded to dt, then
    the product of the two dt values rounded to dt.  (silu's exp comes from the host libm; it can differ from torch's
    vectorised exp in the last fp32 bit, which the dt rounding almost always hides.)"""
    xf = to_f32(x, dt)
    k = xf.shape[1] // 2
    g, u = xf[:, :k], xf[:, k:]
    with np.errstate(over="ignore"):
        sl = (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)
    sl = _to_dt(sl, dt) if dt != "fp32" else sl
    return from_f32((sl * u).astype(np.float32), dt)


def linear(x: np.ndarray, dt: str, q: np.ndarray, s_rel: np.ndarray, s_kind: str, s_ch: np.ndarray, codebook: np.ndarray,
           group: int, convrot: int = CONVROT, bias: Optional[np.ndarray] = None, bias_dt: Optional[str] = None,
           out_dt: Optional[str] = None, input_act: Optional[str] = None, mode: str = "ck") -> np.ndarray:
    """`linear(..., precision="a8")` for a W4A8 weight (qlinear.py:466-507 -> _linear_w4a8 :433-463 -> _TorchRunner._a8):
    optional SwiGLU, rotate+quantise, exact int8 GEMM on the decoded grid, epilogue.  x is [M, K] (or [M, 2K] with
    input_act="swiglu"); returns [M, N] in out_dt's storage form."""
    out_dt = out_dt or dt
    n, k = check_weight(q, s_rel, s_ch, codebook, group, convrot)
    if input_act == "swiglu":
        x = swiglu(x, dt)
    if x.shape[1] != k:
        raise ValueError(f"input features {x.shape[1]} do not match the weight's K={k}")
    xq, xs = quantize_rows(x, dt, convrot, mode)
    acc = int8_mm(xq, decode_int8_grid(q, s_rel, s_kind, codebook, group))
    return epilogue(acc, xs, s_ch, bias, out_dt, mode, bias_dt)


# ----------------------------------------------------------------------------------------------------------- inputs
def synth_weight_int4_g128(n: int, k: int, seed: int = 0, group: int = 128, convrot: int = CONVROT):
    """The seeded synthetic layer of the benchmark configs: W ~ N(0, 0.02) rotated into the ConvRot basis, symmetric int4
    per (row, 128-group) with integer codebook cb[i] = i - 8, fp16 relative group scales and an fp32 per-channel scale.
    Returns (q int8 [n, k/2], s_rel fp16 [n, k/group], s_ch fp32 [n], codebook fp32 [16])."""
    rng = np.random.default_rng(seed)
    w = rng.standard_normal((n, k), dtype=np.float32) * np.float32(0.02)
    h = hadamard_regular(convrot)
    w_rot = (w.astype(np.float64).reshape(n, k // convrot, convrot) @ h).reshape(n, k)
    g = w_rot.reshape(n, k // group, group)
    a = np.abs(g).max(axis=2)
    sc = np.maximum(a / 7.0, 1e-12)
    code = np.clip(np.rint(g / sc[:, :, None]), -7, 7).astype(np.int64)
    nib = (code + 8).reshape(n, k)
    s_ch = (sc.max(axis=1) * 7.0 / 127.0).astype(np.float32)
    s_rel = (sc / s_ch.astype(np.float64)[:, None]).astype(np.float16)
    q = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8).view(np.int8)
    codebook = (np.arange(16, dtype=np.float32) - 8.0)
    return q, s_rel, s_ch, codebook


def synth_activation(m: int, k: int, seed: int = 0, outlier_frac: Optional[float] = None, n_outliers: Optional[int] = None,
                     dt: str = "bf16") -> np.ndarray:
    """x ~ N(0, 1) with a few outlier channels scaled x20, rounded to `dt` (the benchmark configs' activations)."""
    rng = np.random.default_rng(seed + 1000)
    x = rng.standard_normal((m, k), dtype=np.float32)
    cnt = n_outliers if n_outliers is not None else max(1, round((outlier_frac or 0.0) * k))
    if cnt:
        ch = rng.permutation(k)[:cnt]
        x[:, ch] *= np.float32(20.0)
    return from_f32(x, dt)
