"""CPU proofs of the numerical shortcuts the kernels take, done with exact rational arithmetic.

1. The rotate+quantise kernel divides by the per-row bf16 scale s with r = RN(1/s) and one Markstein correction step
   (q0 = RN(b r); e = b - q0 s, exact; q1 = RN(q0 + e r)).  For bf16 operands this equals the IEEE quotient RN(b / s)
   for every significand pair; rounding to nearest is invariant under scaling by powers of two, so one binade of b per
   divisor covers every normal pair.
2. The decode level rint(cb * s) clamped to +-127 is what cvt.rni.sat.s8 followed by max(., -127) computes.
3. For bf16, the quotient only matters after it is rounded to bf16, and RNbf16(RN(b * RN(1/s))) = RNbf16(RN(b / s)) for
   every pair of bf16 significands: the kernel multiplies by the per-row reciprocal without a correction step.
"""
import math
from fractions import Fraction as Fr

import numpy as np

from oracle import qlinear_oracle as orc


def rn32(x: Fr) -> Fr:
    if x == 0:
        return Fr(0)
    sgn = -1 if x < 0 else 1
    a = abs(x)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while Fr(2) ** e > a:
        e -= 1
    while Fr(2) ** (e + 1) <= a:
        e += 1
    ulp = Fr(2) ** (e - 23)
    n = a / ulp
    fl = n.numerator // n.denominator
    rem = n - fl
    if rem > Fr(1, 2) or (rem == Fr(1, 2) and fl % 2 == 1):
        fl += 1
    return sgn * fl * ulp


def test_markstein_division_is_correctly_rounded_for_all_bf16_significands():
    bad = 0
    for ms in range(128):
        s = Fr(128 + ms, 128)
        r = rn32(1 / s)
        for mb in range(128):
            b = Fr(128 + mb, 128)
            q0 = rn32(b * r)
            e = b - q0 * s
            assert rn32(e) == e  # the residual is exactly representable, so the FMA computes it exactly
            bad += rn32(q0 + e * r) != rn32(b / s)
    assert bad == 0


def test_decode_level_rule_matches_the_oracle_on_every_fp8_byte():
    """level = clamp(rint(cb * s), -127, 127) with NaN -> 0, for every fp8 scale byte and a codebook spanning the clamp."""
    cb = np.array([-1.0, -0.75, -0.5, -0.3, -0.1, -0.01, 0.0, 0.01, 0.1, 0.3, 0.5, 0.6, 0.75, 0.9, 0.99, 1.0], np.float32)
    s = orc.fp8_e4m3fn_table()
    prod = (cb[None, :] * s[:, None]).astype(np.float32)
    with np.errstate(invalid="ignore"):
        sat = np.clip(np.where(np.isnan(prod), 0, np.rint(prod)), -128, 127)  # cvt.rni.sat.s8 (NaN -> 0)
    kernel = np.maximum(sat, -127)
    q = np.broadcast_to((np.arange(16, dtype=np.uint8) | (np.arange(16, dtype=np.uint8) << 4))[None, :], (256, 16))
    grid = orc.decode_int8_grid(np.ascontiguousarray(q).view(np.int8), np.repeat(np.arange(256, dtype=np.uint8)[:, None], 2, 1),
                                "fp8", cb, 16)
    assert np.array_equal(grid[:, 0::2], kernel.astype(np.int8))
    assert kernel.min() == -127 and kernel.max() == 127


def _rne_bf16(y: np.ndarray) -> np.ndarray:
    u = y.view(np.uint32)
    with np.errstate(over="ignore"):
        return ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)).view(np.float32)


def test_reciprocal_product_gives_the_same_bf16_quotient_for_all_bf16_pairs():
    mb = (np.arange(128, dtype=np.uint32) | 128).astype(np.float32) / np.float32(128.0)
    r = (np.float32(1.0) / mb).astype(np.float32)
    for e in range(-3, 9):  # quotients from 2^-4 (code 0) to 2^8 (beyond the clamp)
        b = (mb * np.float32(2.0 ** e)).astype(np.float32)
        exact = np.ascontiguousarray((b[:, None] / mb[None, :]).astype(np.float32))
        fast = np.ascontiguousarray((b[:, None] * r[None, :]).astype(np.float32))
        assert np.array_equal(_rne_bf16(exact), _rne_bf16(fast)), e
