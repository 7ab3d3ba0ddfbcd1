"""Bit-level number formats used by the reference, restated in numpy.

Values of a narrow format are carried in ``float32`` arrays holding exactly
representable values; ``*_bits`` functions give the stored bit patterns.
TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
BF16_EPS = F32(2.0**-7)  # torch.finfo(torch.bfloat16).eps, CT/quantization/utils/helpers.py:364-372
BF16_TINY = F32(2.0**-126)  # torch.finfo(torch.bfloat16).tiny
FP8_MAX = F32(448.0)  # CT/quantization/quant_args.py FP8_E4M3_DATA.max
FP8_EPS = F32(0.125)  # CT/quantization/utils/helpers.py:365-366
FP4_MAX = F32(6.0)  # CT/quantization/quant_args.py FP4_E2M1_DATA.max


# ---------------------------------------------------------------- bfloat16
def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bits (torch's conversion)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        rounded = np.where(nan, np.uint16(0x7FC0), rounded)
    return rounded


def rb(x) -> np.ndarray:
    """Round float32 values to the bfloat16 grid (result kept as float32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(x, dtype=np.float32)))


# ---------------------------------------------------------------- fp8 e4m3fn
def round_fp8_e4m3(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest float8_e4m3fn value, ties to even.

    Inputs are already clamped to +-448 by the callers (as in
    ``CT/quantization/quant_args.py:411-436,439-475``), so no overflow path.
    """
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x).astype(np.float64)
    _, e = np.frexp(a)  # a = m * 2**e, m in [0.5, 1)
    exp = np.maximum(e - 1, -6)  # unbiased exponent, subnormals share 2**-6
    quantum = np.ldexp(1.0, exp - 3)
    q = np.rint(a / quantum) * quantum
    q = np.where(a == 0, 0.0, q)
    return (np.copysign(q, x)).astype(np.float32)


def fp8_e4m3_bits(v: np.ndarray) -> np.ndarray:
    """Bit pattern of float32 values that are exact e4m3fn values."""
    v = np.asarray(v, dtype=np.float64)
    sign = (np.signbit(v)).astype(np.uint8) << 7
    a = np.abs(v)
    _, e = np.frexp(a)
    exp = e - 1
    normal = exp >= -6
    mant_n = np.where(normal, np.rint(np.ldexp(a, -exp) * 8) - 8, 0)
    bits_n = ((exp + 7).astype(np.int64) << 3) + mant_n.astype(np.int64)
    bits_s = np.rint(a / 2.0**-9).astype(np.int64)
    bits = np.where(a == 0, 0, np.where(normal, bits_n, bits_s))
    return (bits.astype(np.uint8) | sign).astype(np.uint8)


def fp8_e4m3_bits_to_f32(b: np.ndarray) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    sign = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 7
    val = np.where(e == 0, m * 2.0**-9, (1 + m / 8.0) * np.ldexp(1.0, e - 7))
    val = np.where((b & 0x7F) == 0x7F, np.nan, val)
    return (sign * val).astype(np.float32)


# ---------------------------------------------------------------- fp4 e2m1
E2M1_GRID = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)


def cast_to_fp4(x: np.ndarray) -> np.ndarray:
    """``FP4_E2M1_DATA.cast_to_fp4`` (CT/quantization/quant_args.py:46-66).

    Thresholds with the reference's closed/open ends; the sign comes from
    ``torch.sign`` so a negative input that rounds to zero gives -0.0, and
    +-0.0 inputs give +0.0 (sign(0) == 0).
    """
    x = np.asarray(x, dtype=np.float32)
    s = np.sign(x)
    a = np.abs(x)
    out = np.select(
        [a <= 0.25, a < 0.75, a <= 1.25, a < 1.75, a <= 2.5, a < 3.5, a <= 5.0],
        [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0],
        default=6.0,
    ).astype(np.float32)
    return (out * s).astype(np.float32)


def fp4_codes(v: np.ndarray) -> np.ndarray:
    """E2M1 magnitude index with sign bit 8 (CT/compressors/nvfp4/helpers.py:34-74)."""
    v = np.asarray(v, dtype=np.float32)
    idx = np.argmin(np.abs(np.abs(v)[..., None] - E2M1_GRID), axis=-1)
    return (idx + (np.signbit(v).astype(np.int64) << 3)).astype(np.uint8)


def pack_nibbles_u8(codes: np.ndarray) -> np.ndarray:
    """Two 4-bit codes per byte, even column in the low nibble."""
    c = np.asarray(codes, dtype=np.uint8)
    return (c[..., 0::2] | (c[..., 1::2] << 4)).astype(np.uint8)
