"""compressed-tensors casts and packers, restated in numpy.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``).

``modelfree_tensor`` restates the per-tensor model-free path
(S/entrypoints/model_free/lifecycle.py:38-60 then ``compress_module``,
CT/compressors/base.py:145-166) for the weight-only preset schemes.
"""
from __future__ import annotations

import numpy as np

from .numerics import (
    FP4_MAX,
    FP8_MAX,
    cast_to_fp4,
    fp4_codes,
    fp8_e4m3_bits,
    pack_nibbles_u8,
    rb,
    round_fp8_e4m3,
)
from .observers import (
    QArgs,
    calculate_qparams,
    calculate_range,
    fused_absmax,
    generate_gparam,
    minmax,
    pad_for_block,
)

F32 = np.float32

SCHEMES: dict[str, QArgs] = {
    # CT/quantization/quant_scheme.py presets (weights only)
    "W4A16": QArgs(4, "int", True, "group", 128),
    "W4A16_ASYM": QArgs(4, "int", False, "group", 128),
    "W8A16": QArgs(8, "int", True, "channel", None),
    "FP8_DYNAMIC": QArgs(8, "float", True, "channel", None, zp_dtype="fp8"),
    "FP8": QArgs(8, "float", True, "tensor", None, zp_dtype="fp8"),
    "FP8_BLOCK": QArgs(8, "float", True, "block", None, (128, 128), zp_dtype="fp8"),
    "NVFP4A16": QArgs(4, "float", True, "tensor_group", 16, scale_dtype="fp8", zp_dtype="fp8"),
    "MXFP4A16": QArgs(4, "float", True, "group", 32, scale_dtype="uint8", zp_dtype="uint8"),
}


def expand_scale(scale: np.ndarray, args: QArgs, shape) -> np.ndarray:
    """Broadcast per-group/channel/block parameters to the weight's shape."""
    r, c = shape
    s = np.asarray(scale)
    if args.strategy == "tensor":
        return np.broadcast_to(s.reshape(1, 1), (r, c))
    if args.strategy == "channel":
        return np.broadcast_to(s.reshape(r, 1), (r, c))
    if args.strategy in ("group", "tensor_group"):
        return np.repeat(s.reshape(r, -1), args.group_size, axis=1)
    if args.strategy == "block":
        bh, bw = args.block_structure
        return np.repeat(np.repeat(s, bh, axis=0), bw, axis=1)[:r, :c]
    raise ValueError(args.strategy)


def quantize_int(w: np.ndarray, scale: np.ndarray, zp, args: QArgs, scale_f32: bool = False) -> np.ndarray:
    """``quantize(..., dtype=int8)`` for INT args (CT/quantization/lifecycle/forward_helpers.py:213-242).

    bf16 weight / bf16 scale is a bf16 quotient; with a float32 scale the
    quotient stays float32.  Zero point (if any) is added in the same dtype,
    then clamp to the integer range and round half-even.
    """
    R = (lambda v: np.asarray(v, F32)) if scale_f32 else rb
    s = expand_scale(scale, args, w.shape)
    q = R(w / s)
    if zp is not None:
        q = R(q + expand_scale(np.asarray(zp, F32), args, w.shape))
    lo, hi = calculate_range(args)
    return np.rint(np.clip(q, lo, hi)).astype(np.int8)


def pack_to_int32(codes: np.ndarray, num_bits: int, packed_dim: int = 1) -> np.ndarray:
    """``pack_to_int32`` (CT/compressors/pack_quantized/helpers.py:20-89)."""
    v = (codes.astype(np.int32) + (1 << (num_bits - 1))).astype(np.uint32) & ((1 << num_bits) - 1)
    if packed_dim == 0:
        v = v.T
    r, c = v.shape
    pf = 32 // num_bits
    pc = -(-c // pf) * pf
    if pc != c:
        v = np.pad(v, ((0, 0), (0, pc - c)))
    v = v.reshape(r, pc // pf, pf)
    packed = np.zeros((r, pc // pf), dtype=np.uint32)
    for j in range(pf):
        packed |= v[:, :, j] << np.uint32(num_bits * j)
    packed = packed.view(np.int32)
    return packed.T.copy() if packed_dim == 0 else packed


def quantize_fp8(w: np.ndarray, scale: np.ndarray, args: QArgs) -> np.ndarray:
    """FP8 ``quantize`` (CT forward_helpers.py:213-242 via round_to_quantized_type_args,
    CT/quantization/quant_args.py:439-475): bf16 quotient, clamp +-448, cast RNE."""
    if args.strategy == "block":
        p = pad_for_block(w, args.block_structure)
        s = expand_scale(scale, args, p.shape)
        q = rb(p / s)
        v = round_fp8_e4m3(np.clip(q, -FP8_MAX, FP8_MAX))
        return fp8_e4m3_bits(v[: w.shape[0], : w.shape[1]])
    s = expand_scale(scale, args, w.shape)
    q = rb(w / s)
    return fp8_e4m3_bits(round_fp8_e4m3(np.clip(q, -FP8_MAX, FP8_MAX)))


def quantize_nvfp4(w: np.ndarray, scale_f32: np.ndarray, global_scale: np.float32, args: QArgs) -> np.ndarray:
    """NVFP4 ``quantize`` + ``pack_fp4_to_uint8`` (CT/compressors/nvfp4/base.py:40-73).

    Effective scale ``scale / global_scale`` in float32; float32 quotient;
    ``+= zero_point`` (0.0, so -0.0 becomes +0.0); clamp +-6; E2M1 cast.
    """
    eff = (scale_f32.astype(F32) / F32(global_scale)).astype(F32)
    s = expand_scale(eff, args, w.shape)
    q = (w.astype(F32) / s).astype(F32) + F32(0.0)
    v = cast_to_fp4(np.clip(q, -FP4_MAX, FP4_MAX))
    return pack_nibbles_u8(fp4_codes(v))


def quantize_mxfp4(w: np.ndarray, scale_bf16: np.ndarray, args: QArgs) -> np.ndarray:
    """MXFP4 ``quantize`` + pack (CT/compressors/mxfp4/base.py:20-34 inheriting
    nvfp4/base.py:40-73) with the scale held in bf16: bf16 quotient."""
    s = expand_scale(scale_bf16, args, w.shape)
    q = rb(w / s) + F32(0.0)
    v = cast_to_fp4(np.clip(q, -FP4_MAX, FP4_MAX))
    return pack_nibbles_u8(fp4_codes(v))


def mx_scale_to_e8m0(scale: np.ndarray) -> np.ndarray:
    """``compress_mx_scale`` (CT/compressors/mx_utils.py:18-30)."""
    with np.errstate(divide="ignore"):
        e = 127 + np.floor(np.log2(scale.astype(F32))).astype(np.int32)
    return e.astype(np.uint8)


def modelfree_tensor(w: np.ndarray, scheme: str, global_scale=None) -> dict:
    """One tensor through the model-free path; keys as compressed-tensors writes them.

    ``w`` holds bf16 values as float32.  For NVFP4 the caller may pass the
    fused set's global scale (see ``nvfp4_global_scale``).
    """
    args = SCHEMES[scheme]
    mn, mx = minmax(w, args)
    out: dict[str, np.ndarray] = {}
    if args.strategy == "tensor_group":
        if global_scale is None:
            global_scale = generate_gparam(fused_absmax([(mn, mx)]))
        scale, _ = calculate_qparams(mn, mx, args, global_scale=global_scale)
        out["weight_packed"] = quantize_nvfp4(w, scale, global_scale, args)
        out["weight_scale"] = fp8_e4m3_bits(scale)
        out["weight_global_scale"] = np.array([global_scale], dtype=F32)
        return out
    scale, zp = calculate_qparams(mn, mx, args)
    if args.is_mx:
        out["weight_packed"] = quantize_mxfp4(w, scale, args)
        out["weight_scale"] = mx_scale_to_e8m0(scale)
        return out
    if args.type == "float":
        out["weight"] = quantize_fp8(w, scale, args)
        out["weight_scale"] = scale
        return out
    codes = quantize_int(w, scale, None if args.symmetric else zp, args)
    out["weight_packed"] = pack_to_int32(codes, args.num_bits)
    out["weight_scale"] = scale
    out["weight_shape"] = np.array(w.shape, dtype=np.int64)
    if not args.symmetric:
        out["weight_zero_point"] = pack_to_int32(zp, args.num_bits, packed_dim=0)
    return out


def nvfp4_global_scale(weights: list[np.ndarray]) -> np.float32:
    """Shared global scale of a fused set (q/k/v, gate/up): S/observers/base.py:78-96."""
    args = SCHEMES["NVFP4A16"]
    return generate_gparam(fused_absmax([minmax(w, args) for w in weights]))


def pack_int4_to_int8(t: np.ndarray) -> np.ndarray:
    """``_pack_int4_to_int8`` (S/utils/pack_int4_to_int8.py:13-28): int8 (rows,
    cols) -> int8 (rows, cols/2), low nibble = even column, high = odd."""
    t = np.asarray(t, dtype=np.int8)
    lo = t[:, 0::2].astype(np.int16) & 0x0F
    hi = t[:, 1::2].astype(np.int16) & 0x0F
    return ((hi << 4) | lo).astype(np.uint8).view(np.int8)
