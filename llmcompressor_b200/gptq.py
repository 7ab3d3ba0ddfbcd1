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
        "llmc_hessian_accumulate_grouped": [_P, _I64, _I64, _I64, _I64, _P, _F32, _P, _F32, _P, _P, _P],
        "llmc_hessian_tiles": [_I64],
        "llmc_gemm_f32_nt": [_I64, _I64, _I64, _P, _I64, _P, _I64, _P, _I64, _I32, _P],
    }
)


class HessianOpts(ctypes.Structure):
    """LlmcHessianOpts (include/llmc_b200.h)."""

    _fields_ = [
        ("fold_tokens", ctypes.c_int64),
        ("wait_ns", ctypes.c_int64),
        ("test_stall", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
    ]


GPTQ_PRECISION = torch.float32

__all__ = ["make_empty_hessian", "accumulate_hessian", "quantize_weight", "BatchedHessian"]


def make_empty_hessian(module: torch.nn.Module, device: torch.device | None = None) -> torch.Tensor:
    """``make_empty_hessian`` (S/modifiers/gptq/gptq_quantize.py:54-60)."""
    weight = module.weight
    num_columns = weight.shape[1]
    device = device if device is not None else weight.device
    return torch.zeros((num_columns, num_columns), device=device, dtype=GPTQ_PRECISION)


# Optional instrumentation: when a list, every Hessian launch appends
# (start event, end event, useful flops) recorded on its stream, so a caller
# (the benchmark) can time the kernel inside a larger pipeline.
TIMING_EVENTS: list | None = None


def hessian_update_(H: torch.Tensor, x2d: torch.Tensor, alpha: float = 2.0,
                    num_samples: torch.Tensor | None = None, num_add: float = 0.0,
                    groups: int = 1, fold_tokens: int = 0, wait_ns: int = 0,
                    status: torch.Tensor | None = None, _test_stall: bool = False) -> torch.Tensor:
    """H += alpha * x^T x for x (tokens, d) bf16 on the tensor cores; optionally
    num_samples += num_add in the same launch.  Any number of tokens per call:
    the kernel folds its tensor-core accumulators into float32 sums every
    ``fold_tokens`` tokens (0: the library default, 1024), so H stays within
    the Hessian bar of the exact sum however long the call.

    ``groups`` > 1: block-diagonal Hessians -- x is (tokens, groups * d) and
    H is (groups * d, d); group g accumulates columns [g*d, (g+1)*d) of x into
    rows [g*d, (g+1)*d) of H (one Hessian per MoE expert).

    A bounded wait that runs out inside the kernel raises ``status`` (default:
    the device's error word, read by ``_lib.check_device_errors``) to ETIMEOUT;
    this call itself never synchronises.  ``wait_ns`` / ``_test_stall`` exist
    for the tests of that path."""
    require_cuda(H, x2d)
    if x2d.dtype != torch.bfloat16:
        raise NotImplementedError(f"Hessian inputs of dtype {x2d.dtype}: the tensor-core path takes bf16")
    groups = int(groups)
    if H.dtype != torch.float32 or not H.is_contiguous() or H.ndim != 2 or H.shape[0] != groups * H.shape[1]:
        raise ValueError("H must be a contiguous float32 (groups * d, d) tensor")
    d = H.shape[1]
    if x2d.shape[-1] != groups * d:
        raise ValueError(f"input feature size {x2d.shape[-1]} != Hessian size {groups} x {d}")
    if x2d.stride(-1) != 1:
        x2d = x2d.contiguous()
    n = x2d.shape[0]
    ld = x2d.stride(0) if n > 1 else groups * d
    ns = None
    if num_samples is not None:
        require_cuda(num_samples)
        if num_samples.dtype != torch.float32:
            raise ValueError("num_samples must be a float32 tensor")
        ns = num_samples
    st = status if status is not None else _lib.error_word(H.device)
    opts = HessianOpts(int(fold_tokens), int(wait_ns), 1 if _test_stall else 0, 0)
    ev = TIMING_EVENTS
    if ev is not None:
        e0 = torch.cuda.Event(enable_timing=True)
        e0.record()
    check(lib().llmc_hessian_accumulate_grouped(ptr(x2d), n, groups, d, ld, ptr(H), float(alpha), ptr(ns),
                                                float(num_add), ptr(st), ctypes.byref(opts), stream_ptr(H.device)),
          "hessian_accumulate")
    if ev is not None:
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record()
        ev.append((e0, e1, float(n) * d * (d + 1) * groups))
    return H


def accumulate_hessian(
    inp: torch.Tensor,
    module: torch.nn.Module,
    H: torch.Tensor,
    num_samples: torch.Tensor,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``accumulate_hessian`` (S/modifiers/gptq/gptq_quantize.py:63-97).

    ``num_samples`` counts the batch dimension (a 2-D input counts as one
    sample) and is updated in place on the device, as is ``H``; one launch per
    call, with no host sync.
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


class BatchedHessian:
    """H += 2 X^T X for callers that see a few thousand tokens per call.

    The reference accumulates each Linear's Hessian once per calibration
    sample from its forward hook (S/modifiers/gptq/base.py:255-289 ->
    ``accumulate_hessian``, S/modifiers/gptq/gptq_quantize.py:63-97): 2048
    tokens per call, too few to keep every SM pair busy for long.  This class
    keeps the calls' inputs in a device buffer of ``chunk_tokens`` rows and
    folds a full buffer into H with one launch (an input at least that long
    goes straight to the kernel), so the hook pays only a device-to-device
    copy.  ``num_samples`` counts as the reference does: the batch dimension,
    a 2-D input counting as one.  The kernel's in-launch folding keeps the
    accuracy of the per-call drop-in at any chunk size.

    Call ``finalize()`` (or ``flush()``) before reading H: up to
    ``chunk_tokens - 1`` tokens may still sit in the buffer.  Calls must come
    from one stream (the buffer is reused in stream order).
    """

    def __init__(self, d: int, device: torch.device | str = "cuda", chunk_tokens: int = 16384,
                 H: torch.Tensor | None = None):
        self.d = int(d)
        self.device = torch.device(device)
        self.H = H if H is not None else torch.zeros(self.d, self.d, dtype=GPTQ_PRECISION, device=self.device)
        self.chunk = int(chunk_tokens)
        self._buf = None  # allocated when a call shorter than the chunk arrives
        self._fill = 0
        self.samples = 0

    def add(self, inp: torch.Tensor) -> None:
        if inp.shape[-1] != self.d:
            raise ValueError(f"input feature size {inp.shape[-1]} != Hessian size {self.d}")
        self.samples += inp.shape[0] if inp.ndim > 2 else 1
        x = inp.to(device=self.device).reshape(-1, self.d)
        if x.dtype != torch.bfloat16:
            raise NotImplementedError(f"Hessian inputs of dtype {x.dtype}: the tensor-core path takes bf16")
        pos, n = 0, x.shape[0]
        while pos < n:
            if self._fill == 0 and n - pos >= self.chunk:
                take = n - pos - (n - pos) % self.chunk  # whole chunks go straight to the kernel
                hessian_update_(self.H, x[pos:pos + take], 2.0)
                pos += take
                continue
            take = min(self.chunk - self._fill, n - pos)
            if self._buf is None:
                self._buf = torch.empty(self.chunk, self.d, dtype=torch.bfloat16, device=self.device)
            self._buf[self._fill:self._fill + take].copy_(x[pos:pos + take])
            self._fill += take
            pos += take
            if self._fill == self.chunk:
                self.flush()

    def flush(self) -> None:
        if self._fill:
            hessian_update_(self.H, self._buf[:self._fill], 2.0)
            self._fill = 0

    def finalize(self) -> tuple[torch.Tensor, torch.Tensor]:
        """Flush and return (H, num_samples) as ``accumulate_hessian`` leaves them."""
        self.flush()
        # a fill kernel, not a host-to-device copy (which would wait for the stream)
        return self.H, torch.full((), float(self.samples), dtype=torch.float32, device=self.device)


_I64P = ctypes.POINTER(ctypes.c_int64)
_lib.extend_signatures(
    {
        "llmc_gptq_prepare_hessian": [_P, _I64, _F32, _P, _P],
        "llmc_gptq_hinv_workspace_size": [_I64, _I64P],
        "llmc_gptq_hinv": [_P, _I64, _P, _P, _P, _P, _P],
        "llmc_gptq_quantize_workspace_size": [_I64, _I64, _I64P],
        "llmc_gptq_quantize": [_P, _I64, _I64, _P, _P, _P, ctypes.POINTER(_lib.QuantArgs), _P, _P, _I64, _P, _P, _P,
                               _P, _P],
    }
)


class GptqColumns(ctypes.Structure):
    """LlmcGptqColumns (include/llmc_b200.h)."""

    _fields_ = [
        ("perm", ctypes.c_void_p),
        ("order", ctypes.c_int32),
        ("scale_is_f32", ctypes.c_int32),
        ("global_scale", ctypes.c_void_p),
        ("g_idx_out", ctypes.c_void_p),
        ("row_loss_out", ctypes.c_void_p),
    ]


_lib.extend_signatures(
    {
        "llmc_gptq_actorder_perm": [_P, _I64, _P, _P],
        "llmc_gptq_permute_hessian": [_P, _I64, _P, _P, _P],
        "llmc_permute_columns_bf16": [_P, _I64, _I64, _P, _P, _P],
        "llmc_gptq_quantize_ex": [_P, _I64, _I64, _P, _P, _P, ctypes.POINTER(_lib.QuantArgs), _P, _P,
                                  ctypes.POINTER(GptqColumns), _I64, _P, _P, _P, _P, _P],
    }
)

_ORDER_CODE = {None: 0, "weight": 1, "group": 2}


def resolve_actorder(actorder) -> str | None:
    """The ordering ``quantize_weight`` applies (S/modifiers/gptq/gptq_quantize.py:120-166):
    None, "weight" (WEIGHT, and STATIC -- its alias) or "group" (GROUP, and
    DYNAMIC -- its alias)."""
    a = getattr(actorder, "value", actorder)
    table = {None: None, "static": "weight", "weight": "weight", "dynamic": "group", "group": "group"}
    if a not in table:
        raise ValueError(f"unknown activation ordering {actorder!r}")
    return table[a]


def actorder_perm(H: torch.Tensor) -> torch.Tensor:
    """``torch.argsort(torch.diag(H), descending=True)``
    (S/modifiers/gptq/gptq_quantize.py:299-310) on the GPU; equal diagonal
    values keep index order.  int32 (d,)."""
    require_cuda(H)
    d = H.shape[0]
    perm = torch.empty(d, dtype=torch.int32, device=H.device)
    check(lib().llmc_gptq_actorder_perm(ptr(H), d, ptr(perm), stream_ptr(H.device)), "gptq_actorder_perm")
    return perm


def permute_hessian(H: torch.Tensor, perm: torch.Tensor) -> torch.Tensor:
    """``H[perm][:, perm]`` into a new tensor."""
    require_cuda(H, perm)
    d = H.shape[0]
    out = torch.empty_like(H)
    check(lib().llmc_gptq_permute_hessian(ptr(H), d, ptr(perm), ptr(out), stream_ptr(H.device)),
          "gptq_permute_hessian")
    return out


def permute_columns(w: torch.Tensor, perm: torch.Tensor) -> torch.Tensor:
    """``w[:, perm]`` of a bf16 weight into a new tensor."""
    require_cuda(w, perm)
    if w.dtype != torch.bfloat16:
        raise NotImplementedError(f"weights of dtype {w.dtype}: the GPTQ kernels take bf16 weights")
    w = w.contiguous()
    out = torch.empty_like(w)
    check(lib().llmc_permute_columns_bf16(ptr(w), w.shape[0], w.shape[1], ptr(perm), ptr(out),
                                          stream_ptr(w.device)), "permute_columns")
    return out


def _ws_bytes(fn, *args) -> int:
    out = ctypes.c_int64(0)
    check(fn(*args, ctypes.byref(out)), fn.__name__)
    return int(out.value)


class InverseHessian:
    """Damped, dead-masked inverse-Hessian factor shared by every module that
    consumes the same Hessian (q/k/v, gate/up).  ``status`` stays on the
    device; ``ok()`` reads it (one host sync).  ``perm``: the activation
    order the factor was built in (None: column order)."""

    def __init__(self, hinv: torch.Tensor, dead: torch.Tensor, status: torch.Tensor,
                 hinv_t: torch.Tensor | None = None, perm: torch.Tensor | None = None):
        self.hinv, self.dead, self.status, self.hinv_t, self.perm = hinv, dead, status, hinv_t, perm

    def ok(self) -> bool:
        """False when the factorisation fell back to the identity (ENOT_PD);
        raises ``DeviceTimeout`` if a kernel of the solve timed out."""
        code = int(self.status.item())
        if code == _lib.ETIMEOUT:
            _lib.raise_status(code, "gptq solve")
        return code != _lib.ENOT_PD


def inverse_hessian(H: torch.Tensor, percdamp: float = 0.01, actorder=None) -> InverseHessian:
    """Dead-column mask, damping and the upper Cholesky factor of H^-1
    (S/modifiers/gptq/gptq_quantize.py:35-38,177-196).  ``H`` is clobbered.
    With an activation ordering the factor is built for H[perm][:, perm],
    perm = argsort(diag(H), descending) (:148-149,299-310)."""
    require_cuda(H)
    if H.dtype != torch.float32 or H.ndim != 2 or H.shape[0] != H.shape[1]:
        raise ValueError("hessian must be a float32 (d, d) tensor")
    H = H.contiguous()
    perm = None
    if resolve_actorder(actorder):
        perm = actorder_perm(H)
        H = permute_hessian(H, perm)
    d = H.shape[0]
    dev = H.device
    st = stream_ptr(dev)
    dead = torch.empty(d, dtype=torch.uint8, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    check(lib().llmc_gptq_prepare_hessian(ptr(H), d, float(percdamp), ptr(dead), st), "gptq_prepare_hessian")
    ws = torch.empty(_ws_bytes(lib().llmc_gptq_hinv_workspace_size, d), dtype=torch.uint8, device=dev)
    hinv = torch.empty(d, d, dtype=torch.float32, device=dev)
    hinv_t = torch.empty(d, d, dtype=torch.float32, device=dev)
    check(lib().llmc_gptq_hinv(ptr(H), d, ptr(hinv), ptr(hinv_t), ptr(ws), ptr(status), st), "gptq_hinv")
    return InverseHessian(hinv, dead, status, hinv_t, perm)


def _strategy(args) -> str:
    return getattr(args.strategy, "value", args.strategy)


def _qtype(args) -> str:
    return getattr(args.type, "value", args.type)


def _fused_weights(module: torch.nn.Module) -> list[torch.Tensor]:
    """The weights that share this module's NVFP4 global scale: its own and
    those of the modules its observer is fused with (S/observers/fusion.py,
    ``FusionHandler``)."""
    ws = [module.weight]
    obs = getattr(module, "weight_observer", None)
    handler = getattr(obs, "fusion_handler", None)
    for h in getattr(handler, "_group", None) or []:
        mod = getattr(h, "module", None)
        if mod is not None and mod is not module:
            ws.append(mod.weight)
    return ws


def weight_qparams(module: torch.nn.Module, quant_args, weight: torch.Tensor | None = None,
                   stats_dtype: torch.dtype = torch.bfloat16):
    """The weight observer's qparams (S/modifiers/gptq/gptq_quantize.py:168-173).

    Weights are always observed memorylessly (S/modifiers/quantization/calibration.py:64-78);
    the statistics of the unmodified weight (or of ``weight``, the permuted
    float32 weight under activation ordering GROUP, with ``stats_dtype``
    float32) are recomputed on the GPU: min-max, or the MSE grid search when
    the attached observer is an MSE observer.  TENSOR_GROUP: the global scale
    from the absmax over the observer's fused set (S/observers/base.py:78-96).
    An attached observer's statistics are released as ``get_qparams`` does.
    Returns ``(scale, zero_point, global_scale or None)``.
    """
    from . import ops

    w = module.weight if weight is None else weight
    obs = getattr(module, "weight_observer", None)
    if obs is not None and "mse" in type(obs).__name__.lower():
        if stats_dtype != torch.bfloat16:
            raise NotImplementedError("MSE observer statistics of a float32 weight (activation ordering GROUP)")
        # S/observers/mse.py: the grid search on the GPU with the observer's knobs
        mn, mx = ops.observe_mse(w, quant_args, getattr(obs, "maxshrink", None),
                                 getattr(obs, "patience", None), getattr(obs, "grid", None),
                                 getattr(obs, "norm", None))
    else:
        mn, mx = ops.observe_minmax(w, quant_args)
    gs = None
    if _strategy(quant_args) == "tensor_group":
        gs = ops.fused_global_scale(_fused_weights(module))
    scale, zp = ops.calculate_qparams(mn, mx, quant_args, gs, stats_dtype=stats_dtype)
    if obs is not None and hasattr(obs, "delete_statistics"):
        try:
            obs.delete_statistics()
        except Exception:  # an observer without statistics: nothing to release
            pass
    return scale, zp, gs


def quantize_with_inverse(weight: torch.Tensor, quant_args, hinv: InverseHessian, scale: torch.Tensor,
                          zero_point: torch.Tensor | None, blocksize: int = 128, actorder=None,
                          global_scale: torch.Tensor | None = None,
                          g_idx_out: torch.Tensor | None = None,
                          row_loss_out: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """GPTQ block loop for one bf16 weight with a prepared inverse factor.
    Returns (fake-quantized bf16 weight, loss as a float32 device scalar).

    ``actorder`` must match the ordering ``hinv`` was built with; with GROUP
    ordering ``scale`` holds the groups of the permuted weight (float32) and
    ``g_idx_out`` (int32, cols) receives each column's group.  ``global_scale``:
    TENSOR_GROUP; ``scale`` is then float32.  ``row_loss_out`` (float32,
    rows): each row's share of the loss."""
    require_cuda(weight, scale)
    if weight.dtype != torch.bfloat16:
        raise NotImplementedError(f"weights of dtype {weight.dtype}: the GPTQ kernels take bf16 weights")
    w = weight.contiguous()
    rows, cols = w.shape
    if hinv.hinv.shape[0] != cols:
        raise ValueError(f"Hessian size {hinv.hinv.shape[0]} != weight columns {cols}")
    order = resolve_actorder(actorder)
    if bool(order) != (hinv.perm is not None):
        raise ValueError("the inverse factor was built for a different activation ordering")
    if order == "group" and g_idx_out is None:
        raise ValueError("activation ordering GROUP needs g_idx_out")
    dev = w.device
    qa = _lib.qargs_struct(quant_args)
    zp = None
    if not quant_args.symmetric and _qtype(quant_args) == "int":
        zp = zero_point.to(torch.int8).contiguous()
    scale_f32 = scale.dtype == torch.float32
    sc = scale.contiguous() if scale_f32 else scale.to(torch.bfloat16).contiguous()
    gsc = global_scale.to(torch.float32).contiguous() if global_scale is not None else None
    if row_loss_out is not None and (row_loss_out.dtype != torch.float32 or row_loss_out.numel() != rows
                                     or not row_loss_out.is_contiguous()):
        raise ValueError("row_loss_out must be a contiguous float32 tensor of one value per row")
    cx = GptqColumns(ptr(hinv.perm), _ORDER_CODE[order], int(scale_f32), ptr(gsc), ptr(g_idx_out),
                     ptr(row_loss_out))
    ws = torch.empty(_ws_bytes(lib().llmc_gptq_quantize_workspace_size, rows, cols), dtype=torch.uint8, device=dev)
    out = torch.empty_like(w)
    loss = torch.empty(1, dtype=torch.float32, device=dev)
    check(lib().llmc_gptq_quantize_ex(ptr(w), rows, cols, ptr(hinv.hinv), ptr(hinv.hinv_t), ptr(hinv.dead),
                                      ctypes.byref(qa), ptr(sc), ptr(zp), ctypes.byref(cx), int(blocksize),
                                      ptr(out), ptr(loss), ptr(ws), ptr(hinv.status), stream_ptr(dev)),
          "gptq_quantize")
    return out, loss


def _warn_fallback():
    from loguru import logger

    logger.warning(
        "Failed to invert hessian due to numerical instability. Consider "
        "increasing GPTQModifier.dampening_frac, increasing the number "
        "of calibration samples, or shuffling the calibration dataset. "
        "Falling back to round-to-nearest for this module."
    )


def quantize_modules_shared(
    modules: list[torch.nn.Module],
    quant_args,
    hessian: torch.Tensor,
    blocksize: int = 128,
    percdamp: float = 0.01,
) -> tuple[InverseHessian, list[tuple[torch.Tensor, dict]]]:
    """``quantize_weight`` for several modules that read the same input (q/k/v,
    gate/up, the experts of an all-expert MoE layer): the Hessian is factored
    once and every module runs its block loop against the shared factor.
    ``quant_args`` is one QuantizationArgs for all modules or a list, one per
    module (the activation ordering must agree).  No host sync: returns the
    factor (``ok()`` reads its status) and, per module, (loss as a float32
    device scalar, q_param_dict as ``quantize_weight`` returns it)."""
    args_list = list(quant_args) if isinstance(quant_args, (list, tuple)) else [quant_args] * len(modules)
    orders = []
    for qa in args_list:
        strategy = _strategy(qa)
        order = resolve_actorder(getattr(qa, "actorder", None))
        if order == "group" and strategy not in ("group", "tensor_group"):
            from loguru import logger

            logger.warning(
                "ActivationOrdering.GROUP requires a grouped quantization strategy; "
                "falling back to actorder=None for this module."
            )
            order = None
        if strategy not in ("tensor", "channel", "group", "tensor_group", "block"):
            raise ValueError(f"Quantization strategy is not supported for GPTQ: {strategy}")
        if order == "group" and (strategy == "tensor_group" or _qtype(qa) == "float"):
            raise NotImplementedError("activation ordering GROUP with float types: scales from float32 statistics "
                                      "are only built for integer types")
        orders.append(order)
    if len({bool(o) for o in orders}) > 1:
        raise ValueError("modules sharing a Hessian must agree on whether activation ordering is used")
    hinv = inverse_hessian(hessian, percdamp, orders[0] if orders else None)
    if len(modules) > 1 and _stackable(modules, args_list, orders):
        return hinv, _quantize_stacked(modules, args_list[0], orders[0], hinv, blocksize)
    results = []
    for module, qa, order in zip(modules, args_list, orders):
        final_dtype = module.weight.dtype
        g_idx = None
        if order == "group":
            # re-observe the permuted (float32) weight for the groups of the new order (:141-145)
            wp = permute_columns(module.weight, hinv.perm)
            scale, zp, gs = weight_qparams(module, qa, weight=wp, stats_dtype=torch.float32)
            g_idx = torch.empty(module.weight.shape[1], dtype=torch.int32, device=module.weight.device)
        else:
            scale, zp, gs = weight_qparams(module, qa)
        wq, loss = quantize_with_inverse(module.weight, qa, hinv, scale, zp, blocksize, order, gs, g_idx)
        zp_dtype = getattr(qa, "zp_dtype", None) or torch.int8
        q_param_dict = {
            "weight": wq.reshape(module.weight.shape).to(final_dtype),
            "weight_scale": scale.to(dtype=final_dtype),
            "weight_zero_point": zp.to(dtype=zp_dtype),
        }
        if gs is not None:
            q_param_dict["weight_global_scale"] = gs.to(dtype=final_dtype)
        if g_idx is not None:
            q_param_dict["weight_g_idx"] = g_idx
        results.append((loss, q_param_dict))
    return hinv, results


def _stackable(modules, args_list, orders) -> bool:
    """Modules whose rows can go through one block-loop call: the same
    per-row-scaled scheme (GROUP or CHANNEL, bf16 weights of one width) and
    the same ordering -- GPTQ rows are independent given the factor, so
    stacking them changes nothing but the number of launches."""
    qa0 = args_list[0]
    if _strategy(qa0) not in ("group", "channel") or orders[0] == "group":
        return False
    cols = modules[0].weight.shape[1]
    for m, qa in zip(modules, args_list):
        if m.weight.dtype != torch.bfloat16 or m.weight.shape[1] != cols or qa != qa0:
            return False
        if getattr(m, "weight_observer", None) is not None and "mse" in type(m.weight_observer).__name__.lower():
            return False
    return True


def _quantize_stacked(modules, qa, order, hinv, blocksize) -> list[tuple[torch.Tensor, dict]]:
    """One block-loop call over the stacked rows of several modules; each
    module gets its rows back, its own scales and its own loss (the sum of
    its rows' losses)."""
    from . import ops

    w = torch.cat([m.weight.detach() for m in modules])
    # GROUP / CHANNEL statistics are per row: one pass over the stacked rows
    # gives each module's own min-max qparams
    mn, mx = ops.observe_minmax(w, qa)
    scale, zp = ops.calculate_qparams(mn, mx, qa)
    for m in modules:
        obs = getattr(m, "weight_observer", None)
        if obs is not None and hasattr(obs, "delete_statistics"):
            try:
                obs.delete_statistics()
            except Exception:  # an observer without statistics: nothing to release
                pass
    row_loss = torch.empty(w.shape[0], dtype=torch.float32, device=w.device)
    wq, _ = quantize_with_inverse(w, qa, hinv, scale, zp, blocksize, order, None, None, row_loss)
    zp_dtype = getattr(qa, "zp_dtype", None) or torch.int8
    out, r0 = [], 0
    for m in modules:
        r1 = r0 + m.weight.shape[0]
        q = {"weight": wq[r0:r1].to(m.weight.dtype), "weight_scale": scale[r0:r1].to(dtype=m.weight.dtype),
             "weight_zero_point": zp[r0:r1].to(dtype=zp_dtype)}
        out.append((row_loss[r0:r1].sum().reshape(1), q))
        r0 = r1
    return out


_lib.extend_signatures({
    "llmc_gptq_solve_batch_workspace_size": [_I64, _I64, _I64, ctypes.c_int, _P],
    "llmc_gptq_solve_batch": [_P, _I64, _I64, ctypes.c_float, _P, _I64, _P, _P, _P, _I64, _P, _P, _P, _P,
                              ctypes.c_int, _P],
})
SOLVE_BATCH_STREAMS = 16


class BatchStatus:
    """The status word of one expert of a batched solve (``ok()`` as
    ``InverseHessian.ok``)."""

    def __init__(self, status: torch.Tensor, e: int):
        self.status, self.e = status, e

    def ok(self) -> bool:
        code = int(self.status[self.e].item())
        if code == _lib.ETIMEOUT:
            _lib.raise_status(code, "gptq solve")
        return code != _lib.ENOT_PD


def batchable(modules, args_list, orders) -> bool:
    """Modules whose Hessians can go through one batched solve: one weight
    shape, bf16, the same per-row-scaled scheme (GROUP or CHANNEL, min-max
    observers) and column order."""
    if not modules or any(o is not None for o in orders):
        return False
    shape = modules[0].weight.shape
    return _stackable(modules, args_list, orders) and all(m.weight.shape == shape for m in modules)


def solve_batched(modules: list[torch.nn.Module], qa, H: torch.Tensor, blocksize: int = 128,
                  percdamp: float = 0.01):
    """The batched solve of E modules of one shape with E distinct Hessians
    H (E*d, d) float32 (averaged; clobbered), in one call
    (``llmc_gptq_solve_batch``).  The qparams come from one min-max pass over
    the stacked weights (per-row statistics: the same values as per module).
    Returns the stacked results: (weights (E, rows, d) bf16, scales
    (E*rows, ...), zero points (E*rows, ...), losses (E) float32, status (E)
    int32)."""
    from . import ops

    E = len(modules)
    rows, d = modules[0].weight.shape
    if H.dtype != torch.float32 or not H.is_contiguous() or tuple(H.shape) != (E * d, d):
        raise ValueError("H must be a contiguous float32 (E * d, d) tensor")
    dev = H.device
    w = torch.stack([m.weight.detach() for m in modules])  # (E, rows, d)
    mn, mx = ops.observe_minmax(w.view(E * rows, d), qa)
    scale, zp = ops.calculate_qparams(mn, mx, qa)
    for m in modules:
        obs = getattr(m, "weight_observer", None)
        if obs is not None and hasattr(obs, "delete_statistics"):
            try:
                obs.delete_statistics()
            except Exception:  # an observer without statistics: nothing to release
                pass
    zpk = zp.to(torch.int8).contiguous() if (not qa.symmetric and _qtype(qa) == "int") else None
    sc = scale.to(torch.bfloat16).contiguous()
    out = torch.empty_like(w)
    loss = torch.empty(E, dtype=torch.float32, device=dev)
    status = torch.empty(E, dtype=torch.int32, device=dev)
    nb = ctypes.c_int64(0)
    check(lib().llmc_gptq_solve_batch_workspace_size(E, rows, d, SOLVE_BATCH_STREAMS, ctypes.byref(nb)),
          "gptq_solve_batch_workspace_size")
    ws = torch.empty(nb.value + 256, dtype=torch.uint8, device=dev)
    wsp = (ws.data_ptr() + 255) // 256 * 256
    qs = _lib.qargs_struct(qa)
    check(lib().llmc_gptq_solve_batch(ptr(H), E, d, float(percdamp), ptr(w), rows, ctypes.byref(qs), ptr(sc),
                                      ptr(zpk), int(blocksize), ptr(out), ptr(loss), ptr(status), wsp,
                                      SOLVE_BATCH_STREAMS, stream_ptr(dev)), "gptq_solve_batch")
    return out, scale, zp, loss, status


def batched_param_dicts(modules, qa, out, scale, zp, loss) -> list[tuple[torch.Tensor, dict]]:
    """Per module (loss as a float32 device scalar, q_param_dict) from the
    stacked results of ``solve_batched``."""
    rows = modules[0].weight.shape[0]
    zp_dtype = getattr(qa, "zp_dtype", None) or torch.int8
    res = []
    for e, m in enumerate(modules):
        r0, r1 = e * rows, (e + 1) * rows
        res.append((loss[e:e + 1], {"weight": out[e].to(m.weight.dtype),
                                    "weight_scale": scale[r0:r1].to(dtype=m.weight.dtype),
                                    "weight_zero_point": zp[r0:r1].to(dtype=zp_dtype)}))
    return res


def quantize_batched(modules: list[torch.nn.Module], qa, H: torch.Tensor, blocksize: int = 128,
                     percdamp: float = 0.01) -> tuple[torch.Tensor, list[tuple[torch.Tensor, dict]]]:
    """``quantize_weight`` for E modules of one shape with E distinct
    Hessians (``solve_batched``).  Returns (status (E) int32, per module
    (loss as a float32 device scalar, q_param_dict));
    ``BatchStatus(status, e).ok()`` reads expert e."""
    out, scale, zp, loss, status = solve_batched(modules, qa, H, blocksize, percdamp)
    return status, batched_param_dicts(modules, qa, out, scale, zp, loss)


def quantize_weight(
    module: torch.nn.Module,
    quant_args,
    hessian: torch.Tensor,
    blocksize: int = 128,
    percdamp: float = 0.01,
):
    """``quantize_weight`` (S/modifiers/gptq/gptq_quantize.py:100-296).

    :return: (loss, q_param_dict) with ``weight`` (weight dtype),
        ``weight_scale`` (weight dtype), ``weight_zero_point`` (zp_dtype),
        ``weight_global_scale`` (TENSOR_GROUP) and ``weight_g_idx``
        (activation ordering GROUP).
    """
    hinv, [(loss, q_param_dict)] = quantize_modules_shared([module], quant_args, hessian, blocksize, percdamp)
    # one host sync: Hessian-accumulation timeouts since the last check, then the factor's status
    _lib.check_device_errors(module.weight.device, "hessian_accumulate")
    if not hinv.ok():
        _warn_fallback()
    return float(loss.item()), q_param_dict
