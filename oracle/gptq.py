"""GPTQ Hessian accumulation and block solve, restated in numpy/scipy.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).
"""
from __future__ import annotations

import math

import numpy as np
import scipy.linalg as sla

from .numerics import rb
from .observers import QArgs, calculate_qparams, calculate_range, minmax

F32 = np.float32


def accumulate_hessian(x: np.ndarray, H: np.ndarray, num_samples: float) -> tuple[np.ndarray, float]:
    """``accumulate_hessian`` (S/modifiers/gptq/gptq_quantize.py:63-97) for a Linear.

    ``x`` is (batch, tokens, d) or (tokens, d) of bf16 values as float32; a
    2-D input counts as one sample (``:70-73``).  ``H += (sqrt2 x)^T (sqrt2 x)``
    in float32 (``:29-32``).
    """
    x = np.asarray(x, dtype=F32)
    if x.ndim == 2:
        x = x[None]
    num_samples += x.shape[0]
    xs = F32(math.sqrt(2)) * x.reshape(-1, x.shape[-1])
    H += np.ascontiguousarray(xs.T) @ xs
    return H, num_samples


def fake_quantize_column(w: np.ndarray, s: np.ndarray, zp: np.ndarray, args: QArgs, f32_scale: bool = False) -> np.ndarray:
    """``fake_quantize`` of one float32 column with per-row scale
    (CT/quantization/lifecycle/forward_helpers.py ``_quantize_dequantize``):
    float32 quotient, + zp, clamp, round (half-even for int, RNE cast for
    FP8, ``cast_to_fp4`` thresholds for FP4), back to the scale dtype, - zp,
    times the scale.  The scale dtype is bf16 (products rounded to bf16)
    unless ``f32_scale`` (NVFP4's effective scale ``scale / global_scale``,
    float32 throughout)."""
    from .numerics import cast_to_fp4, round_fp8_e4m3

    lo, hi = calculate_range(args)
    R = (lambda v: np.asarray(v, F32)) if f32_scale else rb
    zpf = np.asarray(zp, F32)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        q = (w / s).astype(F32) + zpf
        q = np.clip(q, lo, hi).astype(F32)
        if args.type == "int":
            q = np.rint(q).astype(F32)
        elif args.num_bits == 8:
            q = round_fp8_e4m3(q)
        else:
            q = cast_to_fp4(q)
        deq = R(q - zpf)
        return R(deq * s)


def hinv_upper(H: np.ndarray, percdamp: float) -> tuple[np.ndarray, bool]:
    """Damping + inverse (S/modifiers/gptq/gptq_quantize.py:181-196): returns the
    upper Cholesky factor of (H + damp I)^-1, or identity on failure."""
    d = H.shape[0]
    damp = F32(percdamp) * F32(np.mean(np.diag(H), dtype=F32))
    H = H.copy()
    H[np.arange(d), np.arange(d)] += damp
    try:
        L = sla.cholesky(H, lower=True, check_finite=False)
        inv, info = sla.lapack.spotri(L, lower=1)
        if info != 0:
            raise np.linalg.LinAlgError("spotri")
        inv = np.tril(inv) + np.tril(inv, -1).T
        U = sla.cholesky(inv.astype(F32), lower=False, check_finite=False)
        return U.astype(F32), True
    except np.linalg.LinAlgError:
        return np.eye(d, dtype=F32), False


def resolve_actorder(actorder) -> str | None:
    """``ActivationOrdering`` value as ``quantize_weight`` compares it: STATIC is
    an alias of WEIGHT and DYNAMIC of GROUP (CT/quantization/quant_args.py)."""
    a = getattr(actorder, "value", actorder)
    return {None: None, "static": "weight", "weight": "weight", "dynamic": "group", "group": "group"}[a]


def actorder_perm(H: np.ndarray) -> np.ndarray:
    """``_apply_activation_ordering`` (S/modifiers/gptq/gptq_quantize.py:299-310):
    columns by descending diag(H).  Ties keep index order (a stable sort)."""
    return np.argsort(-np.diag(H).astype(F32), kind="stable")


def quantize_weight(
    w_bf16: np.ndarray,
    H: np.ndarray,
    args: QArgs,
    blocksize: int = 128,
    percdamp: float = 0.01,
    hinv: np.ndarray | None = None,
    actorder=None,
    global_scale=None,
):
    """``quantize_weight`` (S/modifiers/gptq/gptq_quantize.py:100-296).

    ``w_bf16``: (rows, cols) bf16 values as float32.  ``H``: the averaged
    Hessian (H / num_samples, ``S/modifiers/gptq/base.py:594``).
    ``hinv`` (optional): a precomputed inverse factor for this H (of the
    permuted H when ``actorder`` is set), so that the block loop can be
    timed apart from the factorisation.  ``actorder``: None / "weight"
    ("static") / "group" ("dynamic").  ``global_scale`` (TENSOR_GROUP): the
    fused set's global scale; by default the weight's own.

    Returns ``(loss, weight_bf16_values, scale, zero_point, ok)`` and, when
    present, ``extra`` = {"g_idx": ..., "global_scale": ...} as a 6th item.
    """
    r, c = w_bf16.shape
    strategy = args.strategy
    order = resolve_actorder(actorder)
    if order == "group" and strategy not in ("group", "tensor_group"):
        order = None  # (:126-134): falls back with a warning
    if strategy not in ("tensor", "channel", "group", "tensor_group", "block"):
        raise ValueError(f"Quantization strategy is not supported for GPTQ: {strategy}")

    W = w_bf16.astype(F32).copy()
    H = np.array(H, dtype=F32, copy=True)
    perm = None
    if order:
        perm = actorder_perm(H)
        W = W[:, perm]
        H = H[perm][:, perm]
    # the observer's statistics: the original weight, or the permuted one for
    # GROUP ordering (:141-145); min/max of bf16 values
    mn, mx = minmax(W if order == "group" else w_bf16.astype(F32), args)
    gs = None
    if strategy == "tensor_group":
        from .observers import fused_absmax, generate_gparam

        gs = F32(global_scale) if global_scale is not None else generate_gparam(fused_absmax([(mn, mx)]))
    # GROUP re-observes the permuted float32 W: float32 qparams (:120-123,141-145)
    scale, zp = calculate_qparams(mn, mx, args, global_scale=gs, dtype="f32" if order == "group" else "bf16")
    f32_scale = gs is not None or order == "group"
    zp = np.asarray(zp)
    g_idx = None
    if strategy in ("group", "tensor_group", "block"):
        div = args.group_size if strategy != "block" else args.block_structure[1]
        g_idx = np.arange(c) // div
        if order == "weight":
            g_idx = g_idx[perm]
    eff = scale.astype(F32) if gs is None else (scale.astype(F32) / F32(gs)).astype(F32)
    zpf = zp.astype(F32) if zp.dtype != np.float32 else zp
    if strategy == "tensor":
        col = lambda j: (np.full(r, eff.reshape(-1)[0], F32), np.full(r, zpf.reshape(-1)[0], F32))  # noqa: E731
    elif strategy == "channel":
        col = lambda j: (eff[:, 0], zpf[:, 0])  # noqa: E731
    elif strategy in ("group", "tensor_group"):
        col = lambda j: (eff[:, g_idx[j]], zpf[:, g_idx[j]])  # noqa: E731
    else:
        bh = args.block_structure[0]
        rb_idx = np.arange(r) // bh
        col = lambda j: (eff[rb_idx, g_idx[j]], zpf[rb_idx, g_idx[j]])  # noqa: E731

    dead = np.diag(H) == 0  # _mask_dead_hessian (:35-38), after the permutation
    H[dead, dead] = 1
    W[:, dead] = 0
    if hinv is None:
        Hinv, ok = hinv_upper(H, percdamp)
    else:
        Hinv, ok = hinv, True

    losses = np.zeros(r, dtype=F32)
    for i1 in range(0, c, blocksize):
        i2 = min(i1 + blocksize, c)
        count = i2 - i1
        W1 = W[:, i1:i2].copy()
        Q1 = np.zeros_like(W1)
        Err1 = np.zeros_like(W1)
        losses1 = np.zeros_like(W1)
        Hinv1 = Hinv[i1:i2, i1:i2]
        for i in range(count):
            w = W1[:, i]
            d = Hinv1[i, i]
            s_col, z_col = col(i1 + i)
            q = fake_quantize_column(w, s_col, z_col, args, f32_scale=f32_scale)
            Q1[:, i] = q
            losses1[:, i] = (w - q) ** 2 / d**2
            err1 = (w - q) / d
            W1[:, i:] -= np.outer(err1, Hinv1[i, i:]).astype(F32)
            Err1[:, i] = err1
        W[:, i1:i2] = Q1
        losses += np.sum(losses1, 1) / 2
        W[:, i2:] -= Err1 @ Hinv[i1:i2, i2:]
    extra = {}
    if order:
        invperm = np.argsort(perm)
        W = W[:, invperm]
        if order == "group":
            extra["g_idx"] = g_idx[invperm].astype(np.int32)
    if gs is not None:
        extra["global_scale"] = gs
    out = (float(np.sum(losses)), rb(W), scale, zp, ok)
    return out + (extra,) if extra else out


def codes_from_weight(wq: np.ndarray, scale: np.ndarray, zp, args: QArgs, g_idx=None, global_scale=None) -> np.ndarray:
    """Codes a compressed-tensors save would store for a GPTQ weight
    (CT forward_helpers.py ``_quantize``): bf16 quotient (float32 with a
    global scale), + zp, clamp, round -- integer codes for int args, the FP8 /
    FP4 grid values for float args.  ``g_idx``: the group of each column
    (activation ordering GROUP)."""
    from .casts import expand_scale
    from .numerics import cast_to_fp4, round_fp8_e4m3

    lo, hi = calculate_range(args)
    if g_idx is not None:
        s = np.asarray(scale, F32)[:, np.asarray(g_idx)]
        z = None if zp is None or args.symmetric else np.asarray(zp, F32)[:, np.asarray(g_idx)]
    else:
        s = expand_scale(scale, args, wq.shape)
        z = None if zp is None or args.symmetric else expand_scale(np.asarray(zp, F32), args, wq.shape)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        if global_scale is not None:
            q = (wq / (s.astype(F32) / F32(global_scale)).astype(F32)).astype(F32)
        else:
            q = rb(wq / s)
        if z is not None:
            q = rb(q + z)
        q = np.clip(q, lo, hi)
        if args.type == "int":
            return np.rint(q).astype(np.int32)
        return round_fp8_e4m3(q) if args.num_bits == 8 else cast_to_fp4(q)


def layer_output_error(w: np.ndarray, q: np.ndarray, x: np.ndarray) -> float:
    """||(W - Q) X||^2 / ||W X||^2 with X the layer's calibration inputs (tokens, d)."""
    w = w.astype(np.float64)
    q = q.astype(np.float64)
    x = x.reshape(-1, x.shape[-1]).astype(np.float64)
    return float(np.sum(((w - q) @ x.T) ** 2) / np.sum((w @ x.T) ** 2))
