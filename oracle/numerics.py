"""Bit-exact scalar formats for the oracle (test infrastructure only).

numpy has IEEE float32 and float16 with round-to-nearest-even; bfloat16 and
float8_e4m3fn are restated here from their definitions:
  bf16  = the top 16 bits of an fp32 (RNE on the dropped 16 bits);
  e4m3fn = 1 sign, 4 exponent (bias 7), 3 mantissa bits, subnormals at 2^-9 steps, no
          infinities, max finite 448 (OCP FP8 spec), round to nearest even.
These are the conversions torch performs in the reference's ``.to(dtype)`` calls.
"""

from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even (NaN stays NaN)."""
    u = np.array(x, dtype=np.float32).view(np.uint32).astype(np.uint64)  # keeps 0-d shape
    lsb = (u >> 16) & 1
    r = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def round_f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def rounder(dtype: str):
    """Returns the fp32 -> fp32 function that rounds to ``dtype`` ('f32', 'f16', 'bf16')."""
    if dtype == "f32":
        return lambda v: np.asarray(v, dtype=np.float32)
    if dtype == "f16":
        return round_f16
    if dtype == "bf16":
        return round_bf16
    raise ValueError(dtype)


# ------------------------------------------------------------------ float8 e4m3fn
def _e4m3_table() -> np.ndarray:
    vals = np.zeros(256, dtype=np.float32)
    for code in range(256):
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        if e == 15 and m == 7:
            vals[code] = np.nan
        elif e == 0:
            vals[code] = s * m * 2.0 ** -9
        else:
            vals[code] = s * (1.0 + m / 8.0) * 2.0 ** (e - 7)
    return vals


E4M3_VALUES = _e4m3_table()


def e4m3_to_f32(codes: np.ndarray) -> np.ndarray:
    return E4M3_VALUES[np.asarray(codes, dtype=np.uint8)]


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fn codes, round to nearest even, saturating at +-448 (inputs are
    clamped to +-448 before every conversion on this path, so saturation never rounds)."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    sign = np.signbit(x).astype(np.uint8) << 7
    code = np.zeros(x.shape, dtype=np.int64)
    sub = a < 2.0 ** -6
    # subnormals (and the rounding up into the smallest normal): q = rne(a * 2^9) in 0..8
    q_sub = np.rint(a * 2.0 ** 9).astype(np.int64)
    code = np.where(sub, q_sub, code)
    # normals: a = f * 2^e with f in [0.5, 1) -> mantissa steps rne(f * 16) in [8, 16]
    f, e = np.frexp(np.where(sub, 1.0, a))
    q = np.rint(f * 16.0).astype(np.int64)
    E = e.astype(np.int64) - 1
    carry = q == 16
    q = np.where(carry, 8, q)
    E = np.where(carry, E + 1, E)
    normal_code = ((E + 7) << 3) | (q - 8)
    normal_code = np.minimum(normal_code, 0x7E)  # 448
    code = np.where(sub, code, normal_code)
    out = (code.astype(np.uint8) | sign).astype(np.uint8)
    nan = np.isnan(x)
    if nan.any():
        out = np.where(nan, np.uint8(0x7F), out)
    return out


# ------------------------------------------------------------------ float8 e4m3fnuz
def _e4m3fnuz_table() -> np.ndarray:
    """Values of the 256 e4m3fnuz codes: exponent bias 8, subnormals m * 2^-10, no infinities,
    no negative zero; 0x80 is the only NaN and 0x7F / 0xFF are +-240."""
    vals = np.zeros(256, dtype=np.float32)
    for code in range(256):
        if code == 0x80:
            vals[code] = np.nan
            continue
        s = -1.0 if code & 0x80 else 1.0
        e = (code >> 3) & 0xF
        m = code & 0x7
        vals[code] = s * (m * 2.0 ** -10 if e == 0 else (1.0 + m / 8.0) * 2.0 ** (e - 8))
    return vals


E4M3FNUZ_VALUES = _e4m3fnuz_table()


def e4m3fnuz_to_f32(codes: np.ndarray) -> np.ndarray:
    return E4M3FNUZ_VALUES[np.asarray(codes, dtype=np.uint8)]


def f32_to_e4m3fnuz(x: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fnuz codes by round to nearest even over the code values (|x| <= 240 on
    this path, every input is clamped first): the two neighbouring codes of |x|, the nearer
    one, on a tie the even code; a result of zero is +0 (the encoding has no -0); NaN -> 0x80.
    torch's CPU cast gives the same codes (pinned in the tests)."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    pos = E4M3FNUZ_VALUES[:128].astype(np.float64)  # ascending with the code
    hi = np.clip(np.searchsorted(pos, a, side="left"), 1, 127)
    lo = hi - 1
    d_lo, d_hi = a - pos[lo], pos[hi] - a
    code = np.where((d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0)), hi, lo).astype(np.int64)
    sign = np.where(np.signbit(x) & (code != 0), 0x80, 0)
    out = (code | sign).astype(np.uint8)
    return np.where(np.isnan(x), np.uint8(0x80), out).astype(np.uint8)


def log2_f32(x: np.ndarray) -> np.ndarray:
    """log2 rounded to fp32 (evaluated in float64, then rounded once)."""
    return np.log2(np.asarray(x, dtype=np.float64)).astype(np.float32)
