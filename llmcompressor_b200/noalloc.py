"""Python binding of ``llmc_gptq_quantize_noalloc``: the GPTQ block loop for
callers that cannot allocate device memory (see include/llmc_b200.h).  The
scratch is a fixed 32 MiB array inside the library; weights whose workspace
does not fit are rejected with ValueError.  Calls that overlap on the GPU
share that array and race."""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_ptr

_P, _I64 = ctypes.c_void_p, ctypes.c_int64
_lib.extend_signatures(
    {"llmc_gptq_quantize_noalloc": [_P, _I64, _I64, _P, _P, _P, ctypes.POINTER(_lib.QuantArgs), _P, _P, _I64, _P, _P,
                                    _P, _P]}
)

SCRATCH_BYTES = 32 << 20


def _require(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def quantize_with_inverse_noalloc(weight: torch.Tensor, quant_args, hinv, scale: torch.Tensor,
                                  zero_point: torch.Tensor | None, out: torch.Tensor, loss: torch.Tensor,
                                  blocksize: int = 128) -> None:
    """Fill ``out`` (bf16, weight-shaped) and ``loss`` (float32, 1 element) --
    both provided by the caller -- without allocating anything on the device.

    Nothing is converted here (a conversion would allocate), so the inputs
    must already be what the kernels read: ``weight``, ``out`` and ``scale``
    contiguous CUDA bf16 tensors on one device (integer types with bf16
    scales, as ``ops.calculate_qparams`` returns for them), ``loss`` one
    float32 element, and for asymmetric schemes an int8 ``zero_point``.
    Anything else raises ValueError before any launch."""
    if getattr(hinv, "perm", None) is not None:
        raise ValueError("the no-allocation entry point takes factors without activation ordering")
    qtype = getattr(quant_args.type, "value", quant_args.type)
    _require(qtype == "int", "the no-allocation entry point takes integer quantization types")
    _require(weight.ndim == 2, "weight must be 2-D")
    rows, cols = weight.shape
    dev = weight.device
    for name, t in (("weight", weight), ("out", out), ("scale", scale)):
        _require(t.is_cuda and t.device == dev, f"{name} must be a CUDA tensor on {dev}")
        _require(t.dtype == torch.bfloat16, f"{name} must be bfloat16, got {t.dtype}")
        _require(t.is_contiguous(), f"{name} must be contiguous")
    _require(tuple(out.shape) == (rows, cols), f"out must have the weight's shape {(rows, cols)}")
    _require(loss.is_cuda and loss.device == dev and loss.dtype == torch.float32 and loss.numel() == 1,
             "loss must be a one-element float32 CUDA tensor on the weight's device")
    _require(hinv.hinv.shape[0] == cols, f"Hessian size {hinv.hinv.shape[0]} != weight columns {cols}")
    zp = None
    if not quant_args.symmetric:
        _require(zero_point is not None, "asymmetric schemes need a zero point")
        _require(zero_point.is_cuda and zero_point.device == dev and zero_point.dtype == torch.int8
                 and zero_point.is_contiguous(), "zero_point must be a contiguous int8 CUDA tensor")
        _require(zero_point.numel() == scale.numel(), "zero_point must have the scale's shape")
        zp = zero_point
    qa = _lib.qargs_struct(quant_args)
    check(lib().llmc_gptq_quantize_noalloc(ptr(weight), rows, cols, ptr(hinv.hinv), ptr(hinv.hinv_t), ptr(hinv.dead),
                                           ctypes.byref(qa),
                                           ptr(scale), ptr(zp), int(blocksize), ptr(out), ptr(loss),
                                           ptr(hinv.status), stream_ptr(dev)),
          "gptq_quantize_noalloc")
