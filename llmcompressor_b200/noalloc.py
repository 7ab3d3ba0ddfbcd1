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


def quantize_with_inverse_noalloc(weight: torch.Tensor, quant_args, hinv, scale: torch.Tensor,
                                  zero_point: torch.Tensor | None, out: torch.Tensor, loss: torch.Tensor,
                                  blocksize: int = 128) -> None:
    """Fill ``out`` (bf16, weight-shaped) and ``loss`` (float32, 1 element) --
    both provided by the caller -- without allocating anything on the device."""
    if getattr(hinv, "perm", None) is not None:
        raise ValueError("the no-allocation entry point takes factors without activation ordering")
    rows, cols = weight.shape
    qa = _lib.qargs_struct(quant_args)
    zp = None if quant_args.symmetric else zero_point
    check(lib().llmc_gptq_quantize_noalloc(ptr(weight), rows, cols, ptr(hinv.hinv), ptr(hinv.hinv_t), ptr(hinv.dead),
                                           ctypes.byref(qa),
                                           ptr(scale), ptr(zp), int(blocksize), ptr(out), ptr(loss),
                                           ptr(hinv.status), stream_ptr(weight.device)),
          "gptq_quantize_noalloc")
