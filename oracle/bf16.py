"""bfloat16 helpers for the oracle (test infrastructure only).

bfloat16 values are carried as ``uint16`` bit patterns or as the ``float32``
values they denote.  Every rounding is round-to-nearest-even, the rounding the
reference's Metal ``bfloat`` arithmetic and the CUDA ``__float2bfloat16_rn``
intrinsic both use.
"""
from __future__ import annotations

import numpy as np

BF16_NAN = np.uint16(0x7FC0)


def bits_to_f32(bits) -> np.ndarray:
    """bfloat16 bit patterns -> float32 values (exact)."""
    b = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return b.view(np.float32)


def f32_to_bits(values) -> np.ndarray:
    """float32 -> bfloat16 bits, round to nearest even (NaN -> 0x7FC0|sign)."""
    a = np.ascontiguousarray(values, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    out = ((u + 0x7FFF + lsb) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        out = np.where(nan, ((u >> 16).astype(np.uint16) & 0x8000) | BF16_NAN, out)
    return out.astype(np.uint16)


def round_f32(values) -> np.ndarray:
    """Round float32 values to bfloat16 precision, returned as float32."""
    return bits_to_f32(f32_to_bits(values))


def f64_to_bits(values) -> np.ndarray:
    """float64 -> bfloat16 bits with ONE rounding (nearest even).

    Used where the oracle defines a bfloat16 result as the correctly rounded
    value of an exactly known real (``exp`` of a bfloat16 input).  Handles
    overflow to infinity and the bfloat16 subnormal range.
    """
    a = np.asarray(values, dtype=np.float64)
    out = np.zeros(a.shape, dtype=np.float64)
    finite = np.isfinite(a) & (a != 0)
    m, e = np.frexp(np.where(finite, a, 1.0))
    # bfloat16 keeps 8 significant bits for normal values; subnormals keep
    # fewer (the smallest normal exponent of bfloat16 is -126).
    keep = np.where(e - 1 >= -126, 8, 8 - (-126 - (e - 1)))
    keep = np.maximum(keep, 0)
    r = np.rint(np.ldexp(m, keep))  # rint = round half to even
    val = np.ldexp(r, e - keep)
    out = np.where(finite, val, a)
    with np.errstate(over="ignore"):
        f32 = out.astype(np.float32)
    bits = f32_to_bits(f32)  # exact: val already has bfloat16 precision
    big = finite & (np.abs(val) > 3.3895313892515355e38)
    if big.any():
        bits = np.where(big, np.where(a > 0, 0x7F80, 0xFF80), bits).astype(np.uint16)
    return bits.astype(np.uint16)


def op(fn, *args) -> np.ndarray:
    """Apply a float32 operation to bfloat16 values and round the result.

    This is how the reference's Metal ``bfloat`` arithmetic behaves: each
    operation is evaluated in float32 and rounded back to bfloat16.
    """
    with np.errstate(all="ignore"):
        r = fn(*[np.asarray(a, dtype=np.float32) for a in args]).astype(np.float32)
    return round_f32(r)
