"""torch-facing wrappers of the observer / qparams / cast kernels.

Each function validates devices, dtypes and shapes, allocates its outputs
with torch (the C side never allocates caller-visible memory), and launches
on the current CUDA stream without synchronising.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, lib, ptr, qargs_struct, require_cuda, stream_ptr


def _strategy(args) -> str:
    return getattr(args.strategy, "value", args.strategy)


def _type(args) -> str:
    return getattr(args.type, "value", args.type)


def stats_shape(rows: int, cols: int, args) -> tuple[int, ...]:
    """Shape of min/max/scale for a (rows, cols) weight (S/observers/helpers.py:63-102)."""
    s = _strategy(args)
    if s == "tensor":
        return (1,)
    if s == "channel":
        return (rows, 1)
    if s in ("group", "tensor_group"):
        if cols % args.group_size:
            raise ValueError(
                f"group quantization strategy requires strict division of weight/activation "
                f"size {cols} and group/block size {args.group_size}"
            )
        return (rows, cols // args.group_size)
    if s == "block":
        bh, bw = args.block_structure
        return (-(-rows // bh), -(-cols // bw))
    raise ValueError(f"Unknown strategy {s}")


def _check_weight(w: torch.Tensor) -> torch.Tensor:
    require_cuda(w)
    if w.dtype != torch.bfloat16:
        raise NotImplementedError(f"weights of dtype {w.dtype}: the kernels take bf16 weights")
    if w.ndim != 2:
        raise ValueError(f"expected 2D linear weight, but got shape {tuple(w.shape)}")
    return w.contiguous()


def observe_minmax(w: torch.Tensor, args) -> tuple[torch.Tensor, torch.Tensor]:
    """Memoryless min-max statistics (S/observers/min_max.py:16-25,106-110)."""
    w = _check_weight(w)
    shape = stats_shape(w.shape[0], w.shape[1], args)
    mn = torch.empty(shape, dtype=torch.bfloat16, device=w.device)
    mx = torch.empty(shape, dtype=torch.bfloat16, device=w.device)
    qa = qargs_struct(args)
    check(lib().llmc_observe_minmax(ptr(w), w.shape[0], w.shape[1], ctypes.byref(qa), ptr(mn), ptr(mx),
                                    stream_ptr(w.device)), "observe_minmax")
    return mn, mx


MSE_DEFAULTS = {"maxshrink": 0.20, "patience": 5, "grid": 100.0, "norm": 2.4}


def observe_mse(w: torch.Tensor, args, maxshrink: float | None = None, patience: int | None = None,
                grid: float | None = None, norm: float | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """MSE grid-search statistics (``memoryless_mse``: S/observers/mse.py:12-45,
    S/observers/mse_quant.py:19-141).  Unset knobs come from
    ``args.observer_kwargs`` and then the reference's defaults."""
    w = _check_weight(w)
    kw = dict(MSE_DEFAULTS)
    kw.update(getattr(args, "observer_kwargs", None) or {})
    maxshrink = float(kw["maxshrink"] if maxshrink is None else maxshrink)
    patience = int(kw["patience"] if patience is None else patience)
    grid = float(kw["grid"] if grid is None else grid)
    norm = float(kw["norm"] if norm is None else norm)
    rows, cols = w.shape
    shape = stats_shape(rows, cols, args)
    mn = torch.empty(shape, dtype=torch.bfloat16, device=w.device)
    mx = torch.empty(shape, dtype=torch.bfloat16, device=w.device)
    qa = qargs_struct(args)
    nbytes = ctypes.c_int64(0)
    check(lib().llmc_observe_mse_workspace_size(rows, cols, ctypes.byref(qa), ctypes.byref(nbytes)), "observe_mse")
    ws = torch.empty(max(int(nbytes.value), 8), dtype=torch.uint8, device=w.device)
    check(lib().llmc_observe_mse(ptr(w), rows, cols, ctypes.byref(qa), maxshrink, patience, grid, norm, ptr(mn),
                                 ptr(mx), ptr(ws), stream_ptr(w.device)), "observe_mse")
    return mn, mx


def grid_search_mse(observed: torch.Tensor, args, token_args=None, maxshrink: float = 0.20, patience: int = 5,
                    grid: float = 100.0, norm: float = 2.4, chunk_size: int = 5):
    """Drop-in for the reference's ``_grid_search_mse`` (S/observers/mse_quant.py:19-87)
    on a bf16 *weight* view from ``flatten_for_calibration``: (1, r, G, gs) for
    group strategies, (1, r, 1, c) channel, (1, 1, n) tensor, (1, R, C, bh*bw)
    block (zero-padded).  Returns (min_vals, max_vals) shaped like the
    reference's.  ``token_args`` / ``chunk_size`` only steer the reference's
    evaluation order and are not needed here."""
    s = _strategy(args)
    if observed.dim() == 4 and observed.shape[0] == 1 and s in ("group", "tensor_group"):
        _, r, g, gs = observed.shape
        w2 = observed.reshape(r, g * gs)
    elif observed.dim() == 4 and observed.shape[0] == 1 and s == "channel":
        w2 = observed.reshape(observed.shape[1], observed.shape[3])
    elif observed.dim() == 3 and observed.shape[0] == 1 and s == "tensor":
        w2 = observed.reshape(1, observed.shape[2])
    elif observed.dim() == 4 and observed.shape[0] == 1 and s == "block":
        bh, bw = args.block_structure
        _, R, C, _ = observed.shape
        w2 = observed.reshape(R, C, bh, bw).transpose(1, 2).reshape(R * bh, C * bw)
    else:
        raise NotImplementedError(f"MSE search over an observed view of shape {tuple(observed.shape)} ({s})")
    mn, mx = observe_mse(w2.contiguous(), args, maxshrink, patience, grid, norm)
    lead = observed.shape[1:-1]
    return mn.reshape(lead), mx.reshape(lead)


class MemorylessMSEObserver:
    """GPU mirror of the reference's ``memoryless_mse`` weight observer
    (S/observers/mse.py:12-45): ``forward(weight)`` sets ``min_vals`` /
    ``max_vals``; ``get_qparams()`` returns scale / zero_point (and
    ``global_scale`` for TENSOR_GROUP) and drops the statistics, as
    ``Observer.get_qparams`` (S/observers/base.py:99-123) does."""

    def __init__(self, args, base_name: str = "weight", **_):
        self.args = args
        self.base_name = base_name
        kw = dict(MSE_DEFAULTS)
        kw.update(getattr(args, "observer_kwargs", None) or {})
        self.maxshrink, self.patience = float(kw["maxshrink"]), int(kw["patience"])
        self.grid, self.norm = float(kw["grid"]), float(kw["norm"])
        self.min_vals = self.max_vals = None
        self._global_scale = None

    def __call__(self, observed: torch.Tensor):
        return self.forward(observed)

    def forward(self, observed: torch.Tensor):
        self.min_vals, self.max_vals = observe_mse(observed, self.args, self.maxshrink, self.patience, self.grid,
                                                   self.norm)
        if _strategy(self.args) == "tensor_group":
            self._global_scale = fused_global_scale([observed])
        return self

    def get_qparams(self) -> dict:
        assert self.min_vals is not None, "No statistics available"
        scale, zp = calculate_qparams(self.min_vals, self.max_vals, self.args, global_scale=self._global_scale)
        out = {"scale": scale, "zero_point": zp, "global_scale": self._global_scale}
        self.min_vals = self.max_vals = None
        return out


def absmax_(w: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """Max-accumulate |w| into the float32 scalar ``out`` (initialise to 0)."""
    require_cuda(w, out)
    if w.dtype != torch.bfloat16:
        raise NotImplementedError(f"dtype {w.dtype}")
    w = w.contiguous()
    check(lib().llmc_absmax_accumulate(ptr(w), w.numel(), ptr(out), stream_ptr(w.device)), "absmax")
    return out


def global_scale_from_absmax(absmax: torch.Tensor) -> torch.Tensor:
    """generate_gparam (CT/quantization/utils/helpers.py:309-338): float32 (1,)."""
    gs = torch.empty(1, dtype=torch.float32, device=absmax.device)
    check(lib().llmc_global_scale(ptr(absmax), ptr(gs), stream_ptr(absmax.device)), "global_scale")
    return gs


def fused_global_scale(weights: list[torch.Tensor]) -> torch.Tensor:
    """Shared TENSOR_GROUP global scale of a fused set (q/k/v, gate/up): one
    absmax over all members, then generate_gparam (S/observers/base.py:78-96)."""
    acc = torch.zeros(1, dtype=torch.float32, device=weights[0].device)
    for w in weights:
        absmax_(w, acc)
    return global_scale_from_absmax(acc)


def calculate_qparams(mn: torch.Tensor, mx: torch.Tensor, args, global_scale: torch.Tensor | None = None,
                      stats_dtype: torch.dtype = torch.bfloat16):
    """calculate_qparams (CT/quantization/utils/helpers.py:50-137) on the GPU.

    ``stats_dtype``: the dtype of the observed tensor the statistics came
    from -- bf16 for weights; float32 for the permuted float32 weight that
    activation ordering GROUP re-observes (the values are passed as bf16,
    where they are exact; the arithmetic and the scale are float32)."""
    require_cuda(mn, mx)
    if mn.dtype != torch.bfloat16 or mx.dtype != torch.bfloat16:
        raise NotImplementedError("statistics must be bf16 (the observed weight's dtype)")
    mn, mx = mn.contiguous(), mx.contiguous()
    qa = qargs_struct(args)
    if global_scale is not None:
        global_scale = global_scale.to(torch.float32).contiguous()
    f32stats = stats_dtype == torch.float32
    scale = torch.empty(mn.shape, dtype=torch.float32 if (global_scale is not None or f32stats) else torch.bfloat16,
                        device=mn.device)
    zp_dtype = args.zp_dtype if getattr(args, "zp_dtype", None) is not None else torch.int8
    if zp_dtype == torch.float8_e4m3fn:
        zp = torch.zeros(mn.shape, dtype=zp_dtype, device=mn.device)
        zp_out = None
    else:
        zp = torch.empty(mn.shape, dtype=zp_dtype, device=mn.device)
        zp_out = zp
    check(lib().llmc_calculate_qparams_ex(ptr(mn), ptr(mx), mn.numel(), ctypes.byref(qa), ptr(global_scale),
                                          int(f32stats), ptr(scale), ptr(zp_out), stream_ptr(mn.device)),
          "calculate_qparams")
    if scale.ndim == 0:
        scale, zp = scale.reshape(1), zp.reshape(1)
    return scale, zp


def format_of(args) -> int:
    """compressed-tensors format for weight-only args (CT/compressors/format.py:16-25)."""
    if _type(args) == "float":
        if args.num_bits == 4:
            return _lib.FMT_MXFP4 if args.group_size == 32 else _lib.FMT_NVFP4
        return _lib.FMT_FP8
    return _lib.FMT_PACK_INT32


def packed_shape(rows: int, cols: int, args, fmt: int) -> tuple[tuple[int, ...], torch.dtype]:
    if fmt == _lib.FMT_PACK_INT32:
        pf = 32 // args.num_bits
        return (rows, -(-cols // pf)), torch.int32
    if fmt in (_lib.FMT_NVFP4, _lib.FMT_MXFP4):
        return (rows, cols // 2), torch.uint8
    if fmt == _lib.FMT_FP8:
        return (rows, cols), torch.float8_e4m3fn
    return (rows, cols), torch.int8


def quantize_pack(w: torch.Tensor, args, scale: torch.Tensor, zero_point: torch.Tensor | None = None,
                  global_scale: torch.Tensor | None = None, fmt: int | None = None) -> torch.Tensor:
    """``quantize`` + the compressor's packing with stored qparams
    (CT/compressors/{pack_quantized,naive_quantized,nvfp4,mxfp4}/base.py)."""
    w = _check_weight(w)
    fmt = format_of(args) if fmt is None else fmt
    rows, cols = w.shape
    stats_shape(rows, cols, args)
    require_cuda(scale)
    if scale.dtype == torch.float8_e4m3fn:
        scale = scale.to(torch.float32)
    if scale.dtype not in (torch.bfloat16, torch.float32):
        raise NotImplementedError(f"scale dtype {scale.dtype}")
    scale = scale.contiguous()
    zp = None
    if zero_point is not None and not args.symmetric:
        zp = zero_point.to(torch.int8).contiguous()
    if global_scale is not None:
        global_scale = global_scale.to(torch.float32).reshape(1).contiguous()
    shape, dtype = packed_shape(rows, cols, args, fmt)
    out = torch.empty(shape, dtype=dtype, device=w.device)
    qa = qargs_struct(args)
    check(lib().llmc_quantize_pack(ptr(w), rows, cols, ctypes.byref(qa), ptr(scale),
                                   1 if scale.dtype == torch.float32 else 0, ptr(zp), ptr(global_scale), fmt,
                                   ptr(out), stream_ptr(w.device)), "quantize_pack")
    return out


def pack_zero_point(zp: torch.Tensor, num_bits: int) -> torch.Tensor:
    """pack_to_int32(zero_point, num_bits, packed_dim=0)."""
    require_cuda(zp)
    zp = zp.to(torch.int8).contiguous()
    rows, groups = zp.shape
    pf = 32 // num_bits
    out = torch.empty((-(-rows // pf), groups), dtype=torch.int32, device=zp.device)
    check(lib().llmc_pack_zero_point(ptr(zp), rows, groups, num_bits, ptr(out), stream_ptr(zp.device)),
          "pack_zero_point")
    return out


def _modelfree_buffers(w: torch.Tensor, args, global_scale: torch.Tensor | None):
    rows, cols = w.shape
    fmt = format_of(args)
    sshape = stats_shape(rows, cols, args)
    shape, dtype = packed_shape(rows, cols, args, fmt)
    out = torch.empty(shape, dtype=dtype, device=w.device)
    if fmt == _lib.FMT_NVFP4:
        if global_scale is None:
            global_scale = fused_global_scale([w])
        global_scale = global_scale.to(torch.float32).reshape(1).contiguous()
        scale = torch.empty(sshape, dtype=torch.float8_e4m3fn, device=w.device)
    elif fmt == _lib.FMT_MXFP4:
        scale = torch.empty(sshape, dtype=torch.uint8, device=w.device)
    else:
        scale = torch.empty(sshape, dtype=torch.bfloat16, device=w.device)
    zp = None if args.symmetric else torch.empty(sshape, dtype=torch.int8, device=w.device)
    return fmt, out, scale, zp, global_scale


def _modelfree_state(fmt, args, rows, cols, out, scale, zp, global_scale) -> dict:
    res: dict[str, torch.Tensor] = {}
    if fmt == _lib.FMT_FP8:
        res["weight"] = out
        res["weight_scale"] = scale
        return res
    res["weight_packed"] = out
    res["weight_scale"] = scale
    if fmt == _lib.FMT_NVFP4:
        res["weight_global_scale"] = global_scale
    if fmt == _lib.FMT_PACK_INT32:
        res["weight_shape"] = torch.tensor([rows, cols], dtype=torch.int64)
        if zp is not None:
            res["weight_zero_point"] = pack_zero_point(zp, args.num_bits)
    return res


def modelfree_quantize(w: torch.Tensor, args, global_scale: torch.Tensor | None = None) -> dict:
    """One weight through observe -> qparams -> quantize -> pack in a single
    pass; returns the compressed-tensors state dict entries for it.

    Keys and dtypes follow the compressors: ``weight_packed`` (int32 or uint8)
    or ``weight`` (fp8), ``weight_scale`` (bf16 / fp8 / uint8 E8M0),
    ``weight_global_scale`` (NVFP4), ``weight_shape`` (pack_quantized),
    ``weight_zero_point`` (asymmetric pack_quantized, packed along rows).
    """
    w = _check_weight(w)
    rows, cols = w.shape
    fmt, out, scale, zp, global_scale = _modelfree_buffers(w, args, global_scale)
    qa = qargs_struct(args)
    check(lib().llmc_modelfree_quantize(ptr(w), rows, cols, ctypes.byref(qa), ptr(global_scale), fmt, ptr(out),
                                        ptr(scale), ptr(zp), stream_ptr(w.device)), "modelfree_quantize")
    return _modelfree_state(fmt, args, rows, cols, out, scale, zp, global_scale)


class ModelfreeBatch:
    """A prepared batched model-free pass over fixed weights: outputs and the
    job table are allocated once, ``run()`` only launches (a few microseconds
    of host work), ``results`` holds the compressed-tensors entries per weight.
    Use it when the same set of tensors is quantized repeatedly or when host
    overhead matters (many small expert tensors)."""

    def __init__(self, ws: list[torch.Tensor], args, global_scales: list[torch.Tensor | None] | None = None):
        gss = list(global_scales) if global_scales is not None else [None] * len(ws)
        self.ws = [_check_weight(w) for w in ws]
        self.dev = self.ws[0].device if self.ws else None
        self.jobs = (_lib.CastJob * max(1, len(self.ws)))()
        self.qa = qargs_struct(args)
        self.fmt = format_of(args)
        bufs = []
        for i, (w, gs) in enumerate(zip(self.ws, gss)):
            if w.device != self.dev:
                raise ValueError("all weights of a batch must be on one device")
            fmt, out, scale, zp, gs = _modelfree_buffers(w, args, gs)
            bufs.append((out, scale, zp, gs))
            j = self.jobs[i]
            j.w, j.rows, j.cols = ptr(w), w.shape[0], w.shape[1]
            j.global_scale, j.out, j.scale_out, j.zp_out = ptr(gs), ptr(out), ptr(scale), ptr(zp)
        self._bufs = bufs
        self._args = args

    def run(self) -> "ModelfreeBatch":
        if self.ws:
            check(lib().llmc_modelfree_quantize_batch(self.jobs, len(self.ws), ctypes.byref(self.qa), self.fmt,
                                                      stream_ptr(self.dev)), "modelfree_quantize_batch")
        return self

    @property
    def results(self) -> list[dict]:
        return [_modelfree_state(self.fmt, self._args, w.shape[0], w.shape[1], out, scale, zp, gs)
                for w, (out, scale, zp, gs) in zip(self.ws, self._bufs)]


def modelfree_quantize_batch(ws: list[torch.Tensor], args,
                             global_scales: list[torch.Tensor | None] | None = None) -> list[dict]:
    """``modelfree_quantize`` for many weights with the same args (MoE expert
    sets, the tensors of a shard) in as few launches as possible."""
    if not ws:
        return []
    return ModelfreeBatch(ws, args, global_scales).run().results
    res["weight_packed"] = out
    res["weight_scale"] = scale
    if fmt == _lib.FMT_NVFP4:
        res["weight_global_scale"] = global_scale
    if fmt == _lib.FMT_PACK_INT32:
        res["weight_shape"] = torch.tensor([rows, cols], dtype=torch.int64)
        if zp is not None:
            res["weight_zero_point"] = pack_zero_point(zp, args.num_bits)
    return res


def pack_int4_to_int8(t: torch.Tensor) -> torch.Tensor:
    """``_pack_int4_to_int8`` of the checkpoint repacker
    (S/utils/pack_int4_to_int8.py:13-28): int8 (rows, cols) holding int4
    values -> int8 (rows, cols/2), the even column in the low nibble."""
    require_cuda(t)
    if t.ndim != 2:
        raise ValueError(f"Expected 2D tensor, but got {t.ndim}D")
    rows, cols = t.shape
    if cols % 2 != 0:
        raise ValueError(f"Expected even number of columns for int4 packing, but got shape {t.shape}")
    if t.dtype != torch.int8:
        raise NotImplementedError(f"dtype {t.dtype}: the repacker takes int8")
    t = t.contiguous()
    out = torch.empty(rows, cols // 2, dtype=torch.int8, device=t.device)
    check(lib().llmc_pack_int4_to_int8(ptr(t), rows, cols, ptr(out), stream_ptr(t.device)), "pack_int4_to_int8")
    return out
