"""ctypes binding of ``libllmc_b200.so`` (the C ABI declared in include/llmc_b200.h).

There is no fallback: if the library is missing or cannot load, every call
raises.  Status codes map to the exceptions the reference raises on the same
conditions (ValueError for shapes/dtypes, NotImplementedError for unsupported
combinations).
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libllmc_b200.so")

OK, EINVAL_SHAPE, EINVAL_DTYPE, ENOT_PD, ETIMEOUT, ECUDA, EINVAL_ARG, ENOSUPPORT = range(8)

STRAT = {"tensor": 0, "channel": 1, "group": 2, "tensor_group": 3, "block": 4}
SCALE_NONE, SCALE_FP8, SCALE_U8, SCALE_F32 = range(4)
ZP_INT8, ZP_FP8, ZP_UINT8 = range(3)
FMT_PACK_INT32, FMT_FP8, FMT_NVFP4, FMT_MXFP4, FMT_INT8 = range(5)


class LlmcError(RuntimeError):
    """A CUDA-side failure reported by libllmc_b200 (status code attached)."""

    def __init__(self, status: int, msg: str):
        super().__init__(msg)
        self.status = status


class NotPositiveDefinite(LlmcError):
    """The damped Hessian has no Cholesky factor (``torch._C._LinAlgError`` in the reference)."""


class DeviceTimeout(LlmcError):
    """A bounded wait inside a tensor-core kernel ran out; the kernel stopped
    early and its outputs are unusable (the GPU context stays usable)."""


class QuantArgs(ctypes.Structure):
    _fields_ = [
        ("num_bits", ctypes.c_int32),
        ("type", ctypes.c_int32),
        ("symmetric", ctypes.c_int32),
        ("strategy", ctypes.c_int32),
        ("group_size", ctypes.c_int64),
        ("block_rows", ctypes.c_int64),
        ("block_cols", ctypes.c_int64),
        ("scale_dtype", ctypes.c_int32),
        ("zp_dtype", ctypes.c_int32),
    ]


_lib = None
_lock = threading.Lock()

class CastJob(ctypes.Structure):
    """``LlmcCastJob`` (include/llmc_b200.h)."""

    _fields_ = [
        ("w", ctypes.c_void_p),
        ("rows", ctypes.c_int64),
        ("cols", ctypes.c_int64),
        ("global_scale", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("scale_out", ctypes.c_void_p),
        ("zp_out", ctypes.c_void_p),
    ]


_P = ctypes.c_void_p
_I64 = ctypes.c_int64
_I32 = ctypes.c_int
_QA = ctypes.POINTER(QuantArgs)

# name -> argtypes (all return int status unless listed in _RESTYPES)
_SIGS = {
    "llmc_version": [],
    "llmc_kernel_launches": [],
    "llmc_status_string": [_I32],
    "llmc_last_cuda_error": [],
    "llmc_device_status": [_I32, ctypes.POINTER(ctypes.c_int)],
    "llmc_observe_minmax": [_P, _I64, _I64, _QA, _P, _P, _P],
    "llmc_observe_mse_workspace_size": [_I64, _I64, _QA, _P],
    "llmc_modelfree_quantize_batch": [ctypes.POINTER(CastJob), _I32, _QA, _I32, _P],
    "llmc_pack_int4_to_int8": [_P, _I64, _I64, _P, _P],
    "llmc_observe_mse": [_P, _I64, _I64, _QA, ctypes.c_float, _I32, ctypes.c_float, ctypes.c_float, _P, _P, _P, _P],
    "llmc_absmax_accumulate": [_P, _I64, _P, _P],
    "llmc_global_scale": [_P, _P, _P],
    "llmc_calculate_qparams": [_P, _P, _I64, _QA, _P, _P, _P, _P],
    "llmc_calculate_qparams_ex": [_P, _P, _I64, _QA, _P, ctypes.c_int, _P, _P, _P],
    "llmc_quantize_pack": [_P, _I64, _I64, _QA, _P, _I32, _P, _P, _I32, _P, _P],
    "llmc_modelfree_quantize": [_P, _I64, _I64, _QA, _P, _I32, _P, _P, _P, _P],
    "llmc_pack_zero_point": [_P, _I64, _I64, _I32, _P, _P],
}
_RESTYPES = {"llmc_status_string": ctypes.c_char_p, "llmc_kernel_launches": ctypes.c_int64,
             "llmc_last_cuda_error": ctypes.c_char_p}


def _register(lib, name, argtypes, restype=ctypes.c_int):
    fn = getattr(lib, name)
    fn.argtypes = argtypes
    fn.restype = restype
    return fn


def lib():
    """The loaded library; raises if it has not been built (no CPU fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m llmcompressor_b200.build` "
                    "(there is no CPU fallback)"
                )
            l = ctypes.CDLL(LIB_PATH)
            for name, at in _SIGS.items():
                _register(l, name, at, _RESTYPES.get(name, ctypes.c_int))
            _lib = l
    return _lib


def extend_signatures(sigs: dict, restypes: dict | None = None) -> None:
    """Register more entry points (used by the modules that own them)."""
    _SIGS.update(sigs)
    if restypes:
        _RESTYPES.update(restypes)
    if _lib is not None:
        for name, at in sigs.items():
            _register(_lib, name, at, (restypes or {}).get(name, ctypes.c_int))


def check(status: int, what: str = "") -> None:
    if status == OK:
        return
    msg = lib().llmc_status_string(status).decode()
    msg = f"{what}: {msg}" if what else msg
    if status in (EINVAL_SHAPE, EINVAL_DTYPE):
        raise ValueError(msg)
    if status == ENOSUPPORT:
        raise NotImplementedError(msg)
    if status == ENOT_PD:
        raise NotPositiveDefinite(status, msg)
    if status == ECUDA:
        detail = (lib().llmc_last_cuda_error() or b"").decode()
        if detail:
            msg = f"{msg} ({detail})"
    raise LlmcError(status, msg)


_error_words: dict = {}


def error_word(device: torch.device | int | str | None = None) -> torch.Tensor:
    """The per-device int32 status word the tensor-core kernels raise to
    ``ETIMEOUT`` when a bounded wait runs out.  Launches never read it, so
    passing it costs no host sync; ``check_device_errors`` reads it."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if dev.index is None:
        dev = torch.device("cuda", torch.cuda.current_device())
    w = _error_words.get(dev.index)
    if w is None:
        w = torch.zeros(1, dtype=torch.int32, device=dev)
        _error_words[dev.index] = w
    return w


def check_device_errors(device: torch.device | int | str | None = None, what: str = "") -> None:
    """Read the device's status word (one host sync); if a kernel reported a
    timeout since the last check, clear the word and raise ``DeviceTimeout``."""
    w = error_word(device)
    code = int(w.item())
    if code != OK:
        w.zero_()
        raise_status(code, what or "device kernel")
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        v = ctypes.c_int(0)
        check(lib().llmc_device_status(1, ctypes.byref(v)), "llmc_device_status")
    if v.value != OK:
        raise_status(v.value, what or "device kernel")


def raise_status(code: int, what: str) -> None:
    """Raise the exception for a status read back from the device."""
    if code == OK:
        return
    msg = f"{what}: {lib().llmc_status_string(code).decode()}"
    if code == ETIMEOUT:
        raise DeviceTimeout(code, msg)
    if code == ENOT_PD:
        raise NotPositiveDefinite(code, msg)
    raise LlmcError(code, msg)


def stream_ptr(device: torch.device | None = None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise ValueError("llmcompressor_b200 kernels run on CUDA tensors only (no CPU fallback)")


# ------------------------------------------------------------ quant args
def _enum_val(v):
    return getattr(v, "value", v)


def qargs_struct(args) -> QuantArgs:
    """``compressed_tensors.QuantizationArgs`` (or any object with its fields) -> C struct."""
    strategy = _enum_val(args.strategy)
    typ = _enum_val(args.type)
    block = getattr(args, "block_structure", None) or (0, 0)
    sd = getattr(args, "scale_dtype", None)
    zd = getattr(args, "zp_dtype", None)
    if sd is None:
        scale_dtype = SCALE_NONE
    elif sd == torch.float8_e4m3fn:
        scale_dtype = SCALE_FP8
    elif sd == torch.uint8:
        scale_dtype = SCALE_U8
    elif sd == torch.float32:
        scale_dtype = SCALE_F32
    elif sd in (torch.bfloat16,):
        scale_dtype = SCALE_NONE
    else:
        raise NotImplementedError(f"scale_dtype {sd}")
    if zd is None or zd == torch.int8:
        zp_dtype = ZP_INT8
    elif zd == torch.float8_e4m3fn:
        zp_dtype = ZP_FP8
    elif zd == torch.uint8:
        zp_dtype = ZP_UINT8
    else:
        raise NotImplementedError(f"zp_dtype {zd}")
    return QuantArgs(
        int(args.num_bits),
        1 if typ == "float" else 0,
        1 if args.symmetric else 0,
        STRAT[strategy],
        int(getattr(args, "group_size", None) or 0),
        int(block[0]),
        int(block[1]),
        scale_dtype,
        zp_dtype,
    )


def kernel_launches() -> int:
    """Kernels launched by libllmc_b200 in this process so far."""
    return int(lib().llmc_kernel_launches())
