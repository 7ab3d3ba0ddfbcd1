"""Min-max observers and quantization-parameter arithmetic, restated in numpy.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

Arithmetic follows torch's dtype rules exactly: statistics of a bf16 weight
are bf16, every op on them is computed in float32 and rounded to bf16
(``rb``); a float32 global scale promotes the product to float32.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from .numerics import (
    BF16_EPS,
    BF16_TINY,
    FP8_EPS,
    FP8_MAX,
    bf16_bits_to_f32,
    f32_to_bf16_bits,
    rb,
    round_fp8_e4m3,
)

F32 = np.float32


@dataclass
class QArgs:
    """The fields of ``CT QuantizationArgs`` the hot path reads."""

    num_bits: int = 4
    type: str = "int"  # "int" | "float"
    symmetric: bool = True
    strategy: str = "group"  # tensor | channel | group | tensor_group | block
    group_size: int | None = 128
    block_structure: tuple[int, int] | None = None
    scale_dtype: str | None = None  # None | "fp8" | "uint8" | "f32"
    zp_dtype: str = "int8"  # "int8" | "fp8" | "uint8"
    extra: dict = field(default_factory=dict)

    @property
    def is_mx(self) -> bool:
        """``should_generate_mx_scales`` (CT/quantization/utils/mxfp_utils.py:33-39)."""
        return (
            self.num_bits in (4, 8)
            and self.type == "float"
            and self.group_size == 32
            and self.scale_dtype == "uint8"
        )


def calculate_range(args: QArgs) -> tuple[float, float]:
    """``calculate_range`` (CT/quantization/utils/helpers.py:199-226)."""
    if args.type == "int":
        r = 2.0**args.num_bits
        return -r / 2, r / 2 - 1
    if args.num_bits == 8:
        return -448.0, 448.0
    if args.num_bits == 4:
        return -6.0, 6.0
    raise NotImplementedError(args)


# ---------------------------------------------------------------- statistics
def pad_for_block(w: np.ndarray, block: tuple[int, int]) -> np.ndarray:
    """``maybe_pad_tensor_for_block_quant`` (CT/quantization/utils/helpers.py:375-429)."""
    bh, bw = block
    r, c = w.shape
    pr, pc = (bh - r % bh) % bh, (bw - c % bw) % bw
    if pr == 0 and pc == 0:
        return w
    return np.pad(w, ((0, pr), (0, pc)))


def flatten_weight(w: np.ndarray, args: QArgs) -> np.ndarray:
    """``_flatten_weight`` (S/observers/helpers.py:63-102) without the leading 1."""
    r, c = w.shape
    s = args.strategy
    if s == "tensor":
        return w.reshape(1, -1)
    if s == "channel":
        return w.reshape(r, 1, c)
    if s in ("group", "tensor_group"):
        if c % args.group_size:
            raise ValueError(f"columns {c} not divisible by group_size {args.group_size}")
        return w.reshape(r, c // args.group_size, args.group_size)
    if s == "block":
        bh, bw = args.block_structure
        p = pad_for_block(w, (bh, bw))
        pr, pc = p.shape
        return p.reshape(pr // bh, bh, pc // bw, bw).transpose(0, 2, 1, 3).reshape(pr // bh, pc // bw, bh * bw)
    raise ValueError(s)


def minmax(w: np.ndarray, args: QArgs) -> tuple[np.ndarray, np.ndarray]:
    """``MemorylessMinMaxObserver`` -> ``_get_min_max`` (S/observers/min_max.py:16-25,106-110).

    ``w`` holds bf16 (or float32) values as float32; min/max are exact.
    Returns shapes: tensor (1,), channel (r, 1), group (r, G), block (R, C).
    """
    f = flatten_weight(np.asarray(w, dtype=F32), args)
    return f.min(axis=-1), f.max(axis=-1)


# ---------------------------------------------------------------- qparams
def _round_half_even(x):
    return np.rint(x)


def _to_int_dtype(x: np.ndarray, lo: int, hi: int, np_dtype) -> np.ndarray:
    """``round_to_quantized_type_dtype`` for an integer dtype
    (CT/quantization/quant_args.py:411-436): clamp, round half-even, cast.
    NaN converts to 0, as the x86 conversion the reference runs on does."""
    y = _round_half_even(np.clip(x, lo, hi))
    y = np.where(np.isnan(y), 0, y)
    return y.astype(np_dtype)


def round_to_power_2_bf16(x_bf16_vals: np.ndarray) -> np.ndarray:
    """``round_to_power_2`` on bf16 bits (CT/quantization/utils/mxfp_utils.py:67-108)."""
    bits = f32_to_bf16_bits(x_bf16_vals).astype(np.int32)
    out = ((bits + (1 << 5)) & 0xFF80).astype(np.uint16)
    return bf16_bits_to_f32(out)


def generate_mx_scales(mvp: np.ndarray, num_bits: int) -> np.ndarray:
    """``generate_mx_scales`` (CT/quantization/utils/mxfp_utils.py:111-128), bf16 arithmetic."""
    offset = 2 if num_bits == 4 else 8
    p2 = round_to_power_2_bf16(mvp)
    with np.errstate(divide="ignore"):
        lg = rb(np.log2(p2.astype(np.float32)))
    return rb(rb(F32(127) + np.floor(lg)) - F32(offset))


def calculate_qparams(mn, mx, args: QArgs, global_scale=None, dtype: str = "bf16"):
    """``calculate_qparams`` (CT/quantization/utils/helpers.py:50-137).

    ``dtype`` is the dtype of the statistics (the observed weight's dtype).
    Returns ``(scale, zero_point)``: scale as float32 values (on the grid of
    the returned ``scale_dtype`` name), zero point as an integer/float array.
    """
    R = rb if dtype == "bf16" else (lambda v: np.asarray(v, dtype=F32))
    mn = np.minimum(np.asarray(mn, F32), F32(0))
    mx = np.maximum(np.asarray(mx, F32), F32(0))
    qmin, qmax = calculate_range(args)
    bit_range = qmax - qmin
    with np.errstate(divide="ignore", invalid="ignore"):
        if args.symmetric:
            mvp = np.maximum(np.abs(mn), np.abs(mx))
            if args.is_mx:
                scales = generate_mx_scales(mvp, args.num_bits)
            else:
                scales = R(mvp / F32(bit_range / 2))
            zp = np.zeros_like(scales)
        else:
            if args.num_bits == 4 and args.type == "float":
                raise NotImplementedError("Asymmetric Quantization is not supported for FP4")
            scales = R(R(mx - mn) / F32(bit_range))
            zp = R(F32(qmin) - R(mn / scales))
            zp = np.clip(zp, qmin, qmax)  # NaN propagates, as torch.clamp
    cur = dtype
    if global_scale is not None:
        scales = (np.float32(global_scale) * scales.astype(F32)).astype(F32)
        cur = "f32"
        R = lambda v: np.asarray(v, dtype=F32)  # noqa: E731
    if args.scale_dtype == "fp8":
        scales = R(round_fp8_e4m3(np.clip(scales, -FP8_MAX, FP8_MAX)))
    elif args.scale_dtype == "uint8":
        scales = R(np.where(np.isnan(scales), 0, _round_half_even(np.clip(scales, 0, 255))).astype(F32))
    if args.is_mx:
        scales = R(np.exp2(scales.astype(np.int32) - 127).astype(F32))
    if args.scale_dtype == "fp8":
        eps = FP8_EPS
    elif args.scale_dtype == "uint8":
        eps = F32(1)
    elif args.scale_dtype == "f32" or cur == "f32":
        eps = F32(np.finfo(np.float32).eps)
    else:
        eps = BF16_EPS
    scales = np.where(scales == 0, eps, scales).astype(F32)
    if args.zp_dtype == "int8":
        zp = _to_int_dtype(zp, -128, 127, np.int8)
    elif args.zp_dtype == "uint8":
        zp = _to_int_dtype(zp, 0, 255, np.uint8)
    else:  # fp8 zero points (always zero for the symmetric float schemes)
        zp = np.asarray(zp, dtype=F32)
    return scales, zp


def generate_gparam(absmax) -> np.float32:
    """Global scale for TENSOR_GROUP (``Observer.get_global_scale``,
    S/observers/base.py:78-96 -> ``generate_gparam``,
    CT/quantization/utils/helpers.py:309-338).

    ``448 * 6 / a`` with ``a`` a bf16 scalar runs as ``a.reciprocal() * 2688``
    (``Tensor.__rtruediv__``): two bf16 roundings, then NaN/Inf -> 1, then
    float32.
    """
    a = F32(absmax)
    a = np.maximum(a, BF16_TINY)
    with np.errstate(divide="ignore", over="ignore"):
        recip = rb(F32(1.0) / a)
        gs = rb(recip * F32(448.0 * 6.0))
    gs = np.nan_to_num(gs, nan=1.0, posinf=1.0, neginf=1.0)
    return F32(gs)


def fused_absmax(stats: list[tuple[np.ndarray, np.ndarray]]) -> np.float32:
    """Absmax over a fused set's statistics (S/observers/base.py:90-94)."""
    a = F32(stats[0][1].max())
    for mn, mx in stats:
        a = max(a, F32(-mn.min()))
        a = max(a, F32(mx.max()))
    return F32(a)


# ---------------------------------------------------------------- MSE grid search
def fake_quant_groups(x: np.ndarray, scale: np.ndarray, zp, args: QArgs, dtype: str = "bf16") -> np.ndarray:
    """``fake_quantize`` of grouped values ``x`` (..., n) with per-group scale
    / zero point (...,) as ``_quantize_dequantize`` evaluates it
    (CT/quantization/lifecycle/forward_helpers.py ``_quantize_dequantize``):
    quotient and every later op rounded to the tensor's dtype."""
    from .numerics import cast_to_fp4

    R = rb if dtype == "bf16" else (lambda v: np.asarray(v, dtype=F32))
    s = np.asarray(scale, F32)[..., None]
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        q = R(x / s)
        if zp is not None:
            z = np.asarray(zp, F32)[..., None]
            q = R(q + z)
        qmin, qmax = calculate_range(args)
        q = np.clip(q, qmin, qmax)
        if args.type == "int":
            q = np.rint(q)
        elif args.num_bits == 8:
            q = round_fp8_e4m3(q)
        else:
            q = cast_to_fp4(q)
        if zp is not None:
            q = R(q - z)
        return R(q * s)


def mse_minmax(w: np.ndarray, args: QArgs, maxshrink: float = 0.2, patience: int = 5, grid: float = 100.0,
               norm: float = 2.4, dtype: str = "bf16"):
    """``memoryless_mse`` observer statistics: the eager grid search of
    ``_grid_search_eager`` (S/observers/mse_quant.py:90-141) with
    ``_calculate_error`` (:235-273).

    Per group: candidates (min, max) * p, p = 1 - i/grid for i < int(maxshrink *
    grid); error = sum(|fake_quant(x) - x| ** norm) in the tensor's dtype
    (the exponent itself rounded to that dtype, as torch's ``pow`` with a
    Python scalar does; each power rounded to the dtype, summed in float64
    here, then rounded);
    a candidate replaces the best when its error is strictly lower; the search
    stops for the whole tensor after ``patience`` consecutive steps in which no
    group improved.  Returns (min_vals, max_vals) like ``minmax``.
    """
    R = rb if dtype == "bf16" else (lambda v: np.asarray(v, dtype=F32))
    f = flatten_weight(np.asarray(w, dtype=F32), args)
    mn0, mx0 = f.min(axis=-1), f.max(axis=-1)
    best = np.full(mn0.shape, F32(3.3895313892515355e38 if dtype == "bf16" else np.finfo(F32).max), F32)
    bmn, bmx = mn0.copy(), mx0.copy()
    steps = int(maxshrink * grid)
    no_improve = 0
    for i in range(steps):
        p = F32(1 - i / grid)
        smn, smx = R(mn0 * p), R(mx0 * p)
        scale, zp = calculate_qparams(smn, smx, args, dtype=dtype)
        zpv = None if zp is None else np.asarray(zp, F32)
        q = fake_quant_groups(f, scale, zpv, args, dtype)
        with np.errstate(over="ignore", invalid="ignore"):
            d = np.abs(R(q - f)).astype(F32)
            # torch casts the exponent to the tensor's dtype: bf16(2.4) = 2.40625
            e = R(np.power(d, R(F32(norm))).astype(F32))
            err = R(e.astype(np.float64).sum(axis=-1).astype(F32))
        improved = err < best
        if improved.any():
            best = np.where(improved, err, best)
            bmn = np.where(improved, smn, bmn)
            bmx = np.where(improved, smx, bmx)
            no_improve = 0
        else:
            no_improve += 1
            if no_improve >= patience:
                break
    return bmn.astype(F32), bmx.astype(F32)


# ---------------------------------------------------------------- activation observers
def activation_minmax(x: np.ndarray, args: QArgs) -> tuple[np.ndarray, np.ndarray]:
    """``_get_min_max`` (S/observers/min_max.py:106-110) over the activation
    layouts of ``flatten_for_calibration`` (S/observers/helpers.py:104-153):
    TENSOR -> one value; GROUP / TENSOR_GROUP -> one value per feature group
    over all tokens.  ``x``: (..., features) values as float32."""
    x = np.asarray(x, F32)
    if args.strategy == "tensor":
        return np.array([x.min()], F32), np.array([x.max()], F32)
    gs = args.group_size
    v = x.reshape(-1, x.shape[-1] // gs, gs)
    return v.min(axis=(0, 2)).astype(F32), v.max(axis=(0, 2)).astype(F32)


def update_activation_minmax(prev_min, prev_max, new_min, new_max, observer: str,
                             averaging_constant: float = 0.01, dtype: str = "bf16"):
    """One observer update of (min_vals, max_vals); ``prev_*`` None before the
    first batch."""
    R = rb if dtype == "bf16" else (lambda v: np.asarray(v, F32))
    if prev_min is None or observer == "memoryless_minmax" or (
            observer == "minmax" and float(averaging_constant) == 1.0):
        return R(new_min), R(new_max)
    if observer == "static_minmax":
        return np.minimum(prev_min, new_min).astype(F32), np.maximum(prev_max, new_max).astype(F32)
    w0, w1 = F32(1.0 - averaging_constant), F32(averaging_constant)

    def lerp(a, b):
        return R(R(np.asarray(a, F32) * w0) + R(np.asarray(b, F32) * w1))

    return lerp(prev_min, new_min), lerp(prev_max, new_max)
