"""compressed-tensors compressors backed by the cast kernels.

Same classmethod interface as ``CT/compressors/base.py`` (``compress(state_dict,
scheme)`` on a per-module state dict with local names) and the same output
keys, dtypes and layouts as ``PackedQuantizationCompressor``
(CT/compressors/pack_quantized/base.py:29-78), ``NaiveQuantizationCompressor``
(CT/compressors/naive_quantized/base.py), ``NVFP4PackedCompressor``
(CT/compressors/nvfp4/base.py:23-73) and ``MXFP4PackedCompressor``
(CT/compressors/mxfp4/base.py:20-34).  Tensors must be on a CUDA device.

``register_with_compressed_tensors()`` routes compressed-tensors' registry
entries to these classes, so its ``compress_module`` and
``ModelCompressor.compress_model`` (the save path of ``oneshot``,
S/transformers/compression/compressed_tensors_utils.py:172-191) run them.
"""
from __future__ import annotations

import torch

from . import _lib, ops


def _remove_symmetric_zp(sd: dict, scheme) -> dict:
    """``BaseCompressor._remove_symmetric_zp`` (CT/compressors/base.py)."""
    for name, args in (("input", getattr(scheme, "input_activations", None)), ("weight", scheme.weights),
                       ("output", getattr(scheme, "output_activations", None))):
        if args is not None and args.symmetric:
            sd.pop(f"{name}_zero_point", None)
    return sd


class PackedQuantizationCompressor:
    """int4/int8 weights packed into int32 (``pack-quantized``)."""

    format = "pack-quantized"

    @classmethod
    def compress(cls, state_dict: dict, scheme) -> dict:
        sd = dict(state_dict)
        weight = sd.pop("weight")
        scale = sd.get("weight_scale")
        zp = sd.get("weight_zero_point", None)
        args = scheme.weights
        g_idx = sd.get("weight_g_idx")
        if g_idx is not None and g_idx.device.type != "meta" and getattr(args, "group_size", None):
            sd["weight_packed"] = _pack_with_g_idx(weight, args, scale, zp, g_idx)
        else:
            sd["weight_packed"] = ops.quantize_pack(weight, args, scale, zp, fmt=_lib.FMT_PACK_INT32)
        sd["weight_shape"] = torch.tensor(weight.shape)
        strategy = getattr(args.strategy, "value", args.strategy)
        if not args.symmetric and strategy in ("group", "channel"):
            sd["weight_zero_point"] = ops.pack_zero_point(zp, args.num_bits)
        return _remove_symmetric_zp(sd, scheme)


def _pack_with_g_idx(weight, args, scale, zp, g_idx):
    """Packed codes when column j belongs to group ``g_idx[j]`` (activation
    ordering GROUP; -1 means the column's own group j // group_size, the
    placeholder compressed-tensors initialises g_idx with): the group scales
    are expanded to one scale per column on the device (no host sync) and the
    columns quantized as groups of one -- the same per-element arithmetic as
    ``quantize`` with ``g_idx``."""
    rows, cols = weight.shape
    own = torch.arange(cols, device=weight.device) // int(args.group_size)
    gi = torch.where(g_idx.to(torch.int64) < 0, own, g_idx.to(torch.int64))
    idx = gi.unsqueeze(0).expand(rows, cols)
    scale_cols = scale.gather(1, idx).contiguous()
    zp_cols = zp.gather(1, idx).contiguous() if (zp is not None and not args.symmetric) else None
    args1 = args.model_copy(update={"group_size": 1, "actorder": None})
    # one code per byte (a packed word may not straddle parameter groups), then
    # pack_to_int32's layout: code j of a word at bits j * num_bits, offset 2^(num_bits-1)
    codes = ops.quantize_pack(weight, args1, scale_cols, zp_cols, fmt=_lib.FMT_INT8)
    bits = int(args.num_bits)
    per = 32 // bits
    if cols % per:
        codes = torch.nn.functional.pad(codes, (0, per - cols % per))
    u = (codes.to(torch.int32) + (1 << (bits - 1))) & ((1 << bits) - 1)
    shifts = torch.arange(per, device=weight.device, dtype=torch.int32) * bits
    return (u.reshape(rows, -1, per) << shifts).sum(dim=-1, dtype=torch.int32)


class NaiveQuantizationCompressor:
    """Weights cast to the narrow dtype (float8_e4m3fn or int8), ``naive-quantized``."""

    format = "naive-quantized"

    @classmethod
    def compress(cls, state_dict: dict, scheme) -> dict:
        sd = dict(state_dict)
        weight = sd.pop("weight")
        scale = sd.get("weight_scale")
        zp = sd.get("weight_zero_point", None)
        args = scheme.weights
        fmt = _lib.FMT_FP8 if getattr(args.type, "value", args.type) == "float" else _lib.FMT_INT8
        sd["weight"] = ops.quantize_pack(weight, args, scale, zp, fmt=fmt)
        return _remove_symmetric_zp(sd, scheme)


class FloatQuantizationCompressor(NaiveQuantizationCompressor):
    format = "float-quantized"


class IntQuantizationCompressor(NaiveQuantizationCompressor):
    format = "int-quantized"


class NVFP4PackedCompressor:
    """E2M1 pairs per byte + fp8 scales + float32 global scale (``nvfp4-pack-quantized``)."""

    format = "nvfp4-pack-quantized"

    @classmethod
    def _compress_scale(cls, scale: torch.Tensor, args) -> torch.Tensor:
        return scale.to(args.scale_dtype or torch.float8_e4m3fn)

    @classmethod
    def compress(cls, state_dict: dict, scheme) -> dict:
        sd = dict(state_dict)
        weight = sd.pop("weight")
        scale = sd.pop("weight_scale")
        gs = sd.get("weight_global_scale", None)
        args = scheme.weights
        fmt = _lib.FMT_MXFP4 if args.group_size == 32 else _lib.FMT_NVFP4
        sd["weight_packed"] = ops.quantize_pack(weight, args, scale, None, global_scale=gs, fmt=fmt)
        sd["weight_scale"] = cls._compress_scale(scale, args)
        return _remove_symmetric_zp(sd, scheme)


class MXFP4PackedCompressor(NVFP4PackedCompressor):
    """E2M1 pairs per byte + E8M0 scales (``mxfp4-pack-quantized``)."""

    format = "mxfp4-pack-quantized"

    @classmethod
    def _compress_scale(cls, scale: torch.Tensor, args) -> torch.Tensor:
        # compress_mx_scale (CT/compressors/mx_utils.py:18-30) step for step, in
        # the scale's own dtype (the log2 rounds there) -- the same value for
        # every input, powers of two or not, subnormals and zeros included.
        # The model-free kernels write E8M0 directly; this is the save path's
        # small per-group tensor.
        return (127 + torch.floor(torch.log2(scale)).to(torch.int32)).to(args.scale_dtype or torch.uint8)


COMPRESSORS = {
    c.format: c
    for c in (PackedQuantizationCompressor, NaiveQuantizationCompressor, FloatQuantizationCompressor,
              IntQuantizationCompressor, NVFP4PackedCompressor, MXFP4PackedCompressor)
}


def infer_format(scheme) -> str:
    """``infer_module_format`` priority (CT/compressors/format.py:16-25) for Linear modules."""
    w = scheme.weights
    typ = getattr(w.type, "value", w.type)
    if w.num_bits == 4 and typ == "float":
        return "mxfp4-pack-quantized" if w.group_size == 32 else "nvfp4-pack-quantized"
    if typ == "int" and w.num_bits in (4, 8) and getattr(scheme, "input_activations", None) is None:
        return "pack-quantized"
    if getattr(scheme, "input_activations", None) is not None:
        return "int-quantized" if typ == "int" else "float-quantized"
    return "naive-quantized"


def compress_module(module: torch.nn.Module, format: str | None = None) -> None:
    """``compress_module`` (CT/compressors/base.py:145-166) with these compressors."""
    scheme = getattr(module, "quantization_scheme", None)
    if scheme is None or scheme.weights is None:
        return
    fmt = format or getattr(getattr(scheme, "format", None), "value", None) or infer_format(scheme)
    comp = COMPRESSORS[fmt]
    sd = {k: v.data for k, v in module.named_parameters(recurse=False)}
    sd.update({k: v for k, v in module.named_buffers(recurse=False)})
    out = comp.compress(sd, scheme)
    for k in list(sd):
        module._parameters.pop(k, None)
        module._buffers.pop(k, None)
    for k, v in out.items():
        module.register_parameter(k, torch.nn.Parameter(v, requires_grad=False))


_ORIGINAL: dict = {}


def register_with_compressed_tensors() -> None:
    """Route compressed-tensors' ``compress`` classmethods for every format
    covered here to these kernels (the save-path plug-in point).
    ``unregister_from_compressed_tensors`` restores the originals."""
    from compressed_tensors.compressors import BaseCompressor

    for fmt, cls in COMPRESSORS.items():
        ct_cls = BaseCompressor.get_value_from_registry(fmt)
        if fmt not in _ORIGINAL:
            _ORIGINAL[fmt] = (ct_cls, ct_cls.__dict__.get("compress"))
        ct_cls.compress = classmethod(lambda _c, state_dict, scheme, _impl=cls: _impl.compress(state_dict, scheme))


def unregister_from_compressed_tensors() -> None:
    for fmt, (ct_cls, orig) in list(_ORIGINAL.items()):
        if orig is None:
            if "compress" in ct_cls.__dict__:
                delattr(ct_cls, "compress")
        else:
            ct_cls.compress = orig
        del _ORIGINAL[fmt]
