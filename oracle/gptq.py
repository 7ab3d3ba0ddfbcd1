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


def fake_quantize_column(w: np.ndarray, s: np.ndarray, zp: np.ndarray, args: QArgs) -> np.ndarray:
    """``fake_quantize`` of one float32 column with per-row bf16 scale
    (CT/quantization/lifecycle/forward_helpers.py:175-210): float32 quotient,
    + zp, clamp, round half-even, back to the scale dtype (bf16), - zp, times
    scale rounded to bf16."""
    lo, hi = calculate_range(args)
    q = (w / s).astype(F32)
    zpf = zp.astype(F32)
    q = q + zpf
    q = np.rint(np.clip(q, lo, hi)).astype(F32)
    deq = rb(q - zpf)
    return rb(deq * s)


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


def quantize_weight(
    w_bf16: np.ndarray,
    H: np.ndarray,
    args: QArgs,
    blocksize: int = 128,
    percdamp: float = 0.01,
    hinv: np.ndarray | None = None,
):
    """``quantize_weight`` (S/modifiers/gptq/gptq_quantize.py:100-296), actorder off.

    ``hinv`` (optional): a precomputed inverse factor for this H, so that the
    block loop can be timed apart from the factorisation.

    ``w_bf16``: (rows, cols) bf16 values as float32.  ``H``: the averaged
    Hessian (H / num_samples, ``S/modifiers/gptq/base.py:594``).
    Returns ``(loss, weight_bf16_values, scale, zero_point, ok)``.
    """
    r, c = w_bf16.shape
    mn, mx = minmax(w_bf16, args)  # observer on the original weight (:168-173)
    scale, zp = calculate_qparams(mn, mx, args)
    if args.strategy == "tensor":
        col_scale = lambda j: np.full(r, scale.reshape(-1)[0], F32)  # noqa: E731
        col_zp = lambda j: np.full(r, np.asarray(zp).reshape(-1)[0], F32)  # noqa: E731
    elif args.strategy == "channel":
        col_scale = lambda j: scale[:, 0]  # noqa: E731
        col_zp = lambda j: np.asarray(zp)[:, 0]  # noqa: E731
    elif args.strategy == "group":
        gs = args.group_size
        col_scale = lambda j: scale[:, j // gs]  # noqa: E731
        col_zp = lambda j: np.asarray(zp)[:, j // gs]  # noqa: E731
    else:
        raise ValueError(f"Quantization strategy is not supported for GPTQ: {args.strategy}")

    W = w_bf16.astype(F32).copy()
    H = np.array(H, dtype=F32, copy=True)
    dead = np.diag(H) == 0  # _mask_dead_hessian (:35-38)
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
            q = fake_quantize_column(w, col_scale(i1 + i), col_zp(i1 + i), args)
            Q1[:, i] = q
            losses1[:, i] = (w - q) ** 2 / d**2
            err1 = (w - q) / d
            W1[:, i:] -= np.outer(err1, Hinv1[i, i:]).astype(F32)
            Err1[:, i] = err1
        W[:, i1:i2] = Q1
        losses += np.sum(losses1, 1) / 2
        W[:, i2:] -= Err1 @ Hinv[i1:i2, i2:]
    return float(np.sum(losses)), rb(W), scale, zp, ok


def codes_from_weight(wq: np.ndarray, scale: np.ndarray, zp, args: QArgs) -> np.ndarray:
    """Integer codes a compressed-tensors save would pack for a GPTQ weight
    (bf16 quotient, + zp, clamp, round), CT forward_helpers.py:213-242."""
    from .casts import expand_scale

    lo, hi = calculate_range(args)
    q = rb(wq / expand_scale(scale, args, wq.shape))
    if not args.symmetric:
        q = rb(q + expand_scale(np.asarray(zp, F32), args, wq.shape))
    return np.rint(np.clip(q, lo, hi)).astype(np.int32)


def layer_output_error(w: np.ndarray, q: np.ndarray, x: np.ndarray) -> float:
    """||(W - Q) X||^2 / ||W X||^2 with X the layer's calibration inputs (tokens, d)."""
    w = w.astype(np.float64)
    q = q.astype(np.float64)
    x = x.reshape(-1, x.shape[-1]).astype(np.float64)
    return float(np.sum(((w - q) @ x.T) ** 2) / np.sum((w @ x.T) ** 2))
