"""FP8 e4m3 oracle (test infrastructure only) -- restates tileops/quant_fp8.py."""

from __future__ import annotations

import numpy as np

from .numerics import (e4m3_to_f32, e4m3fnuz_to_f32, f32_to_e4m3, f32_to_e4m3fnuz, log2_f32,
                       rounder)

FP8_MAX = 448.0  # torch.finfo(torch.float8_e4m3fn).max (quant_fp8.py:39-45)
FNUZ_MAX = 240.0  # torch.finfo(torch.float8_e4m3fnuz).max: input_to_float8's bound
FNUZ_GROUP_MAX = 224.0  # get_fp8_min_max's override for e4m3fnuz (quant_fp8.py:42-43)


def ue8m0(scale: np.ndarray) -> np.ndarray:
    """quant_fp8.py:48-49: exp2(ceil(log2(max(s, 1e-30)))) with log2 rounded to fp32. NaN and
    inf scales pass through unchanged, as they do through torch's clamp, log2, ceil and exp2."""
    s = np.maximum(np.asarray(scale, np.float32), np.float32(1e-30))
    keep = ~np.isfinite(s)
    with np.errstate(invalid="ignore"):
        e = np.ceil(log2_f32(np.where(keep, np.float32(1), s))).astype(np.int32)
    return np.where(keep, s, np.ldexp(np.float32(1.0), e)).astype(np.float32)


def input_to_float8(x_f32: np.ndarray, dtype: str, fnuz: bool = False):
    """quant_fp8.py:52-63 in ``dtype``: amax = T(max(amax, 1e-12)); s = T(T(1/amax) * 448);
    q = e4m3(clamp(T(x * s), -448, 448)); returns (codes, float32(1 / s)).

    NaN products keep their NaN through the clamp, and the e4m3 cast keeps the NaN's sign:
    0x7F or 0xFF. Which sign the reference's x86 run gives them (single-threaded torch):
      * bfloat16: torch's vectorised bf16 rounding writes NaN as 0xFFFF (sign set) for every
        element in whole 32-element blocks from the start of the tensor; the scalar tail
        rounds NaN to the sign-clear 0x7FC0;
      * float32 / float16: a NaN in the tensor makes amax, s and every product a sign-clear NaN
        (0x7F); with a numeric s, a NaN product is 0 * inf, x86's sign-set default NaN (0xFF).
        In float16, 1e-12 rounds to 0, so an all-zero tensor has s = inf and every product is
        0 * inf.
    With fnuz (dtype=torch.float8_e4m3fnuz) the bound is 240 and every NaN code is 0x80."""
    rnd = rounder(dtype)
    fmax = np.float32(FNUZ_MAX if fnuz else FP8_MAX)
    x = rnd(np.asarray(x_f32, dtype=np.float32)).reshape(-1)
    amax = np.float32(np.max(np.abs(x)))  # NaN if any element is NaN, as aminmax
    with np.errstate(divide="ignore", over="ignore", invalid="ignore"):
        amax = rnd(np.maximum(amax, np.float32(1e-12)))
        r = rnd(np.float32(1.0) / amax)
        s = rnd(np.float32(r) * fmax)
        y = rnd(x * np.float32(s))
        nan = np.isnan(y)
        enc = f32_to_e4m3fnuz if fnuz else f32_to_e4m3
        codes = enc(np.clip(np.where(nan, np.float32(0), y), -fmax, fmax))
        if fnuz:
            nan_code = np.uint8(0x80)
        elif dtype == "bf16":
            blocked = np.arange(x.size) < (x.size // 32) * 32
            nan_code = np.where(blocked, np.uint8(0xFF), np.uint8(0x7F))
        else:
            nan_code = np.uint8(0x7F) if np.isnan(s) else np.uint8(0xFF)
        codes = np.where(nan, nan_code, codes).astype(np.uint8)
        return codes.reshape(np.shape(x_f32)), np.float32(np.float32(1.0) / np.float32(s))


def group_quant(x_f32: np.ndarray, group_size: int, eps: float = 1e-10, use_ue8m0: bool = False,
                column_major: bool = False, fnuz: bool = False):
    """quant_fp8.py:66-140: scale = max(absmax, eps) / 448 [-> ue8m0];
    q = e4m3(clamp(x / scale, +-448)). Returns (codes shaped like x, scales [..., K/G]; with
    column_major, the reference's reshape-then-transpose of the flat scales).

    A NaN in a group makes its absmax and scale NaN (sign clear). A NaN quotient x / scale keeps
    the sign the reference's x86 run gives it: with a NaN scale, x's own sign when x is NaN,
    else clear (0x7F); with a numeric scale (inf / inf, 0 / 0) the sign-set default NaN
    (0xFF). With fnuz (dtype=torch.float8_e4m3fnuz) the bound is 224 and every NaN code 0x80."""
    fmax = np.float32(FNUZ_GROUP_MAX if fnuz else FP8_MAX)
    x = np.asarray(x_f32, dtype=np.float32)
    lead, k = x.shape[:-1], x.shape[-1]
    flat = x.reshape(-1, group_size)
    absmax = np.maximum(np.max(np.abs(flat), axis=-1), np.float32(eps))
    scale = (absmax / fmax).astype(np.float32)
    if use_ue8m0:
        scale = ue8m0(scale)
    with np.errstate(divide="ignore", invalid="ignore"):
        y = np.clip(flat / scale[:, None], -fmax, fmax).astype(np.float32)
    nan = np.isnan(y)
    codes = (f32_to_e4m3fnuz if fnuz else f32_to_e4m3)(np.where(nan, np.float32(0), y))
    nan_scale = np.isnan(scale)[:, None]
    neg_nan_x = np.isnan(flat) & np.signbit(flat)
    nan_code = np.where(nan_scale & ~neg_nan_x, np.uint8(0x7F), np.uint8(0xFF))
    if fnuz:
        nan_code = np.uint8(0x80)
    q = np.where(nan, nan_code, codes).astype(np.uint8).reshape(*lead, k)
    if column_major:
        # quant_fp8.py:134-136: s_flat.reshape(..., G_, M).transpose(-2, -1).contiguous()
        m = x.shape[-2]
        s = np.ascontiguousarray(np.swapaxes(scale.reshape(*x.shape[:-2], k // group_size, m), -1, -2))
    else:
        s = scale.reshape(*lead, k // group_size)
    return q, s


def block_dequant(codes: np.ndarray, s: np.ndarray, block_size, fnuz: bool = False) -> np.ndarray:
    """quant_fp8.py:143-168: y[n, k] = float32(q[n, k]) * s[n // bn, k // bk]."""
    bn, bk = block_size
    n, k = codes.shape
    rows = np.arange(n) // bn
    cols = np.arange(k) // bk
    dec = e4m3fnuz_to_f32 if fnuz else e4m3_to_f32
    return (dec(codes) * np.asarray(s, np.float32)[rows][:, cols]).astype(np.float32)


def block_matmul(a_codes, b_codes, a_s, b_s, block_size, out_dtype: str) -> np.ndarray:
    """quant_fp8.py:188-236 with per-k-block sums in float64 (e4m3 products are exact), then
    scaled: the fp32-accumulated reference of the tolerance."""
    bn, bk = block_size
    a = e4m3_to_f32(a_codes).astype(np.float64)
    b = e4m3_to_f32(b_codes).astype(np.float64)
    m, k = a.shape
    n = b.shape[0]
    kt = -(-k // bk)
    rows_b = np.arange(n) // bn
    acc = np.zeros((m, n), dtype=np.float64)
    for kb in range(kt):
        sl = slice(kb * bk, min(k, (kb + 1) * bk))
        acc += (a[:, sl] @ b[:, sl].T) * a_s[:, kb].astype(np.float64)[:, None] * \
            b_s[rows_b, kb].astype(np.float64)[None, :]
    return rounder(out_dtype)(acc.astype(np.float32))


def block_matmul_reference_cpu(a_codes, b_codes, a_s, b_s, block_size, out_dtype: str):
    """The reference's CPU algorithm as it runs (fp32 dequant, fp32 GEMM)."""
    bn, bk = block_size
    k = a_codes.shape[1]
    cols = np.arange(k) // bk
    a_f = e4m3_to_f32(a_codes) * np.asarray(a_s, np.float32)[:, cols]
    b_f = block_dequant(b_codes, b_s, block_size)
    return rounder(out_dtype)(a_f @ b_f.T)


def layer_reference_cpu_torch(A, B):
    """The reference algorithm of the dynamic-FP8 layer on torch CPU tensors, timed as the CPU
    baseline: per-token quantisation of A (quant_fp8.py:66-80), tensor-wide quantisation of B
    (quant_fp8.py:52-63), then fp32 dequant of both and an fp32 GEMM cast to bf16
    (quant_fp8.py:231-236)."""
    import torch

    fp8 = torch.float8_e4m3fn
    a_f = A.float()
    a_scale = a_f.abs().amax(dim=-1, keepdim=True).clamp(min=1e-10) / FP8_MAX
    qa = (a_f / a_scale).clamp(-FP8_MAX, FP8_MAX).to(fp8)
    amax = B.abs().amax().clamp(min=1e-12)
    b_scale = amax.reciprocal() * FP8_MAX
    qb = (B * b_scale).clamp(-FP8_MAX, FP8_MAX).to(fp8)
    a_deq = qa.float() * a_scale
    b_deq = qb.float() * b_scale.float().reciprocal()
    return (a_deq @ b_deq.T).to(torch.bfloat16)
