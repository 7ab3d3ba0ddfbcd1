"""GPTQ drop-ins: ``make_empty_hessian``, ``accumulate_hessian``, ``quantize_weight``.

Same signatures, argument meaning, return values and error behaviour as
``S/modifiers/gptq/gptq_quantize.py:54-296``; the arithmetic runs in
libllmc_b200.so:

* ``accumulate_hessian``: H += 2 X^T X on tcgen05 tensor cores (bf16 in,
  float32 accumulate in TMEM, TMA reduce-add into H), no host sync.
* ``quantize_weight``: damped Cholesky/inverse, then the 128-column GPTQ block
  loop with per-column fake-quant and error propagation, on the GPU.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, lib, ptr, require_cuda, stream_ptr

_P, _I64, _I32, _F32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float

_lib.extend_signatures(
    {
        "llmc_hessian_accumulate": [_P, _I64, _I64, _I64, _P, _F32, _P, _F32, _P, _P],
        "llmc_hessian_tiles": [_I64],
    }
)

GPTQ_PRECISION = torch.float32

__all__ = ["make_empty_hessian", "accumulate_hessian", "quantize_weight"]


def make_empty_hessian(module: torch.nn.Module, device: torch.device | None = None) -> torch.Tensor:
    """``make_empty_hessian`` (S/modifiers/gptq/gptq_quantize.py:54-60)."""
    weight = module.weight
    num_columns = weight.shape[1]
    device = device if device is not None else weight.device
    return torch.zeros((num_columns, num_columns), device=device, dtype=GPTQ_PRECISION)


def hessian_update_(H: torch.Tensor, x2d: torch.Tensor, alpha: float = 2.0,
                    num_samples: torch.Tensor | None = None, num_add: float = 0.0) -> torch.Tensor:
    """H += alpha * x^T x for x (tokens, d) bf16 on the tensor cores; optionally
    num_samples += num_add in the same launch."""
    require_cuda(H, x2d)
    if x2d.dtype != torch.bfloat16:
        raise NotImplementedError(f"Hessian inputs of dtype {x2d.dtype}: the tensor-core path takes bf16")
    if H.dtype != torch.float32 or not H.is_contiguous() or H.ndim != 2 or H.shape[0] != H.shape[1]:
        raise ValueError("H must be a contiguous float32 (d, d) tensor")
    d = H.shape[0]
    if x2d.shape[-1] != d:
        raise ValueError(f"input feature size {x2d.shape[-1]} != Hessian size {d}")
    if x2d.stride(-1) != 1:
        x2d = x2d.contiguous()
    n = x2d.shape[0]
    ld = x2d.stride(0) if n > 1 else d
    ns = None
    if num_samples is not None:
        require_cuda(num_samples)
        if num_samples.dtype != torch.float32:
            raise ValueError("num_samples must be a float32 tensor")
        ns = num_samples
    check(lib().llmc_hessian_accumulate(ptr(x2d), n, d, ld, ptr(H), float(alpha), ptr(ns), float(num_add), None,
                                        stream_ptr(H.device)), "hessian_accumulate")
    return H


def accumulate_hessian(
    inp: torch.Tensor,
    module: torch.nn.Module,
    H: torch.Tensor,
    num_samples: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``accumulate_hessian`` (S/modifiers/gptq/gptq_quantize.py:63-97).

    ``num_samples`` counts the batch dimension (a 2-D input counts as one
    sample) and is updated in place on the device, as is ``H``.
    """
    inp = inp.to(device=H.device)
    if len(inp.shape) == 2:
        inp = inp.unsqueeze(0)
    num_added = inp.shape[0]
    if not isinstance(module, torch.nn.Linear) and type(module).__name__ != "Conv1D":
        raise NotImplementedError(f"GPTQ Hessian for {type(module).__name__}: only Linear / Conv1D inputs")
    x = inp.reshape((-1, inp.shape[-1]))
    if num_samples.device != H.device or num_samples.dtype != torch.float32:
        num_samples += num_added
        hessian_update_(H, x, 2.0)
    else:
        hessian_update_(H, x, 2.0, num_samples, float(num_added))
    return H, num_samples
