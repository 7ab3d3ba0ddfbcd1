"""Activation observers of static activation schemes on the GPU.

The min/max observers that static activation schemes (input / output
activations, KV-cache q/k/v states) accumulate over the calibration batches:
``MemorylessMinMaxObserver``, ``StaticMinMaxObserver`` and ``MinMaxObserver``
(S/observers/min_max.py:16-110) with the reference's statistics layout
(``flatten_for_calibration``, S/observers/helpers.py:104-153) and update
rules; ``get_qparams`` / ``get_global_scale`` / ``sync_activation_stats``
as ``Observer`` defines them (S/observers/base.py:78-165).

Each observation is one pass of ``llmc_observe_activation`` over the batch
(min/max reduction, then the update rule in the statistics' dtype), so the
statistics never leave the device and no host sync happens in the forward
hook (S/modifiers/quantization/calibration.py:160-183).

Layouts built: activations (``input`` / ``output``) with TENSOR, GROUP and
TENSOR_GROUP strategies; attention states (``q`` / ``k`` / ``v``) with TENSOR.
The other layouts raise ``ValueError`` where the reference does and
``NotImplementedError`` otherwise.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, lib, ptr, require_cuda, stream_ptr

_P, _I64, _I32, _F32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float
_lib.extend_signatures(
    {
        "llmc_observe_activation_workspace_size": [_I64, _I64, ctypes.POINTER(ctypes.c_int64)],
        "llmc_observe_activation": [_P, _I64, _I64, _I32, _I64, _I32, _F32, _F32, _I32, _P, _P, _P, _P],
    }
)

__all__ = [
    "observe_activation_",
    "ActivationObserver",
    "MemorylessMinMaxObserver",
    "StaticMinMaxObserver",
    "MinMaxObserver",
    "OBSERVERS",
]

_MEMORYLESS, _STATIC, _AVERAGE = 0, 1, 2


def _val(x):
    return getattr(x, "value", x)


def _layout(value: torch.Tensor, base_name: str, args) -> tuple[torch.Tensor, int]:
    """(tokens x features view, group) for the statistics layout of
    ``flatten_for_calibration`` (0: one statistic for the whole tensor)."""
    strategy = _val(args.strategy)
    if base_name in ("input", "output"):
        if strategy == "tensor":
            return value.reshape(-1, value.shape[-1]), 0
        if strategy in ("group", "tensor_group"):
            gs = int(args.group_size)
            if value.shape[-1] % gs:
                raise ValueError(f"activation size {value.shape[-1]} is not divisible by group_size {gs}")
            return value.reshape(-1, value.shape[-1]), gs
        if strategy == "token":
            raise NotImplementedError("token activation statistics (dynamic per-token scales are computed at run time)")
        if strategy == "channel":
            raise ValueError("Channel quantization cannot be applied to activations")
        if strategy == "block":
            raise ValueError("Block quantization cannot be applied to activations")
        if strategy == "attn_head":
            raise ValueError("Attention head quantization cannot be applied to activations")
    elif base_name in ("q", "k", "v"):
        if strategy == "tensor":
            return value.reshape(-1, value.shape[-1]), 0
        if strategy == "token":
            raise ValueError("Token quantization cannot be applied to attention")
        if strategy in ("group", "tensor_group"):
            raise ValueError("Group quantization cannot be applied to attention")
        if strategy == "block":
            raise ValueError("Block quantization cannot be applied to attention")
        raise NotImplementedError(f"attention statistics per {strategy}")
    elif base_name == "weight":
        raise ValueError("weights are observed memorylessly by the weight observers (ops.observe_minmax)")
    raise ValueError(f"Unknown quantization base name: {base_name}")


def observe_activation_(value: torch.Tensor, args, base_name: str, mode: int, averaging_constant: float,
                        min_vals: torch.Tensor | None, max_vals: torch.Tensor | None
                        ) -> tuple[torch.Tensor, torch.Tensor]:
    """Fold one observation into (min_vals, max_vals) -- updated in place when
    given, created otherwise -- and return them."""
    require_cuda(value)
    if value.dtype not in (torch.bfloat16, torch.float32):
        raise NotImplementedError(f"activations of dtype {value.dtype}: the observer takes bf16 or float32")
    x, group = _layout(value, base_name, args)
    x = x.contiguous()
    n_tok, hidden = x.shape
    ng = hidden // group if group else 1
    has_prev = min_vals is not None and max_vals is not None
    if not has_prev:
        min_vals = torch.empty(ng, dtype=value.dtype, device=value.device)
        max_vals = torch.empty(ng, dtype=value.dtype, device=value.device)
    elif min_vals.dtype != value.dtype or min_vals.numel() != ng or not min_vals.is_contiguous():
        raise ValueError("statistics do not match this observation's layout or dtype")
    ws_bytes = ctypes.c_int64(0)
    check(lib().llmc_observe_activation_workspace_size(hidden, group, ctypes.byref(ws_bytes)),
          "observe_activation_workspace_size")
    ws = torch.empty(int(ws_bytes.value), dtype=torch.uint8, device=value.device)
    c = float(averaging_constant)
    check(lib().llmc_observe_activation(ptr(x), n_tok, hidden, 0 if value.dtype == torch.bfloat16 else 1, group,
                                        int(mode), float(1.0 - c), c, int(has_prev), ptr(min_vals), ptr(max_vals),
                                        ptr(ws), stream_ptr(value.device)), "observe_activation")
    return min_vals, max_vals


class ActivationObserver:
    """The ``Observer`` interface (S/observers/base.py) for activation
    statistics: call it on each batch, then ``get_qparams()``."""

    _mode = _STATIC
    _sync_ops: dict = {}
    _stats_attrs = ("min_vals", "max_vals")

    def __init__(self, base_name: str, args, **observer_kwargs):
        self.base_name = base_name
        self.args = args
        kw = dict(getattr(args, "observer_kwargs", None) or {})
        kw.update(observer_kwargs)
        self.observer_kwargs = kw

    # -- statistics --------------------------------------------------------
    @property
    def has_statistics(self) -> bool:
        return all(hasattr(self, a) for a in self._stats_attrs)

    def get_statistics(self) -> dict[str, torch.Tensor]:
        assert self.has_statistics, "No statistics available. Call observer(value) first."
        return {a: getattr(self, a) for a in self._stats_attrs}

    def delete_statistics(self, check_fused: bool = True) -> None:
        for a in self._stats_attrs:
            if hasattr(self, a):
                delattr(self, a)

    def _mode_now(self) -> int:
        return self._mode

    @torch.no_grad()
    def forward(self, observed: torch.Tensor) -> "ActivationObserver":
        """S/observers/base.py:126-145 for activations: every batch updates."""
        if observed.numel() == 0:
            return self
        prev = self.has_statistics
        mn, mx = observe_activation_(observed, self.args, self.base_name, self._mode_now(),
                                     self.observer_kwargs.get("averaging_constant", 0.01),
                                     self.min_vals if prev else None, self.max_vals if prev else None)
        self.min_vals, self.max_vals = mn, mx
        return self

    __call__ = forward

    # -- qparams -----------------------------------------------------------
    def get_global_scale(self) -> torch.Tensor | None:
        """TENSOR_GROUP: generate_gparam from the absmax of the statistics
        (S/observers/base.py:78-96)."""
        from . import ops

        if _val(self.args.strategy) != "tensor_group":
            return None
        assert self.has_statistics, "No statistics available. Call observer(value) first."
        if self.min_vals.dtype != torch.bfloat16:
            raise NotImplementedError("global scales from float32 statistics")
        absmax = torch.zeros(1, dtype=torch.float32, device=self.min_vals.device)
        ops.absmax_(self.min_vals, absmax)
        ops.absmax_(self.max_vals, absmax)
        return ops.global_scale_from_absmax(absmax)

    @torch.no_grad()
    def get_qparams(self) -> dict:
        """S/observers/base.py:99-123: calculate_qparams on the statistics,
        which are then released."""
        from . import ops

        assert self.has_statistics, "No statistics available. Call observer(value) first."
        if self.min_vals.dtype != torch.bfloat16:
            raise NotImplementedError("qparams from float32 statistics: observe bf16 activations")
        gs = self.get_global_scale()
        scale, zp = ops.calculate_qparams(self.min_vals, self.max_vals, self.args, gs)
        self.delete_statistics()
        return {"scale": scale, "zero_point": zp, "global_scale": gs}

    def sync_activation_stats(self) -> list:
        """All-reduce the statistics across ranks (S/observers/base.py:146-165)."""
        import torch.distributed as dist

        works = []
        for name, op in self._sync_ops.items():
            val = getattr(self, name, None)
            if val is not None:
                works.append(dist.all_reduce(val, op=getattr(dist.ReduceOp, op), async_op=True))
        return works


class MemorylessMinMaxObserver(ActivationObserver):
    """``memoryless_minmax``: the last batch's min / max."""

    _mode = _MEMORYLESS
    _sync_ops: dict = {}


class StaticMinMaxObserver(ActivationObserver):
    """``static_minmax``: min / max over all batches."""

    _mode = _STATIC
    _sync_ops = {"min_vals": "MIN", "max_vals": "MAX"}


class MinMaxObserver(ActivationObserver):
    """``minmax``: moving average of the batch min / max,
    ``prev * (1 - c) + new * c`` with c = ``averaging_constant`` (0.01)."""

    _mode = _AVERAGE
    _sync_ops = {"min_vals": "AVG", "max_vals": "AVG"}

    def _mode_now(self) -> int:
        # S/observers/min_max.py:95-103: c == 1 keeps the new values as they are
        return _MEMORYLESS if float(self.observer_kwargs.get("averaging_constant", 0.01)) == 1.0 else _AVERAGE


OBSERVERS = {
    "memoryless_minmax": MemorylessMinMaxObserver,
    "static_minmax": StaticMinMaxObserver,
    "minmax": MinMaxObserver,
}


# ------------------------------------------------------------------ reference registry seam
_REGISTERED: dict = {}


def register_with_llmcompressor() -> list[str]:
    """Make the reference's observer registry (``Observer.register`` /
    ``load_from_registry``, S/observers/base.py:29,
    S/modifiers/quantization/calibration.py:80-83) build observers whose
    activation statistics come from the GPU kernels.

    Each registry name (``memoryless_minmax``, ``static_minmax``, ``minmax``)
    is pointed at a subclass of the reference's own observer class, so
    ``initialize_observer`` attaches it as before (an ``nn.Module`` with the
    fusion handler, ``get_qparams``, ``sync_activation_stats`` ...); only its
    ``forward`` on a CUDA activation is replaced by the kernel update above
    (bit-identical statistics).  Weight observations and CPU tensors keep the
    reference's path.  Returns the names routed; ``unregister_from_llmcompressor``
    restores the registry.  Needs the reference package importable."""
    from compressed_tensors.registry.registry import _REGISTRY, standardize_lookup_name
    from llmcompressor.observers.base import Observer as RefObserver

    table = _REGISTRY[RefObserver]
    modes = {"memoryless_minmax": _MEMORYLESS, "static_minmax": _STATIC, "minmax": _AVERAGE}
    for name, mode in modes.items():
        key = standardize_lookup_name(name)  # the registry's own key form
        ref_cls = _REGISTERED.get(name, (table.get(key), key))[0]
        if ref_cls is None:
            continue
        _REGISTERED.setdefault(name, (ref_cls, key))
        table[key] = _gpu_subclass(ref_cls, mode)
    return sorted(n for n in modes if n in _REGISTERED)


def unregister_from_llmcompressor() -> None:
    from compressed_tensors.registry.registry import _REGISTRY
    from llmcompressor.observers.base import Observer as RefObserver

    table = _REGISTRY[RefObserver]
    for name, (ref_cls, key) in list(_REGISTERED.items()):
        table[key] = ref_cls
        del _REGISTERED[name]


def _gpu_subclass(ref_cls, mode: int):
    class GpuActivationObserver(ref_cls):
        @torch.no_grad()
        def forward(self, observed: torch.Tensor):
            if self.is_weight_obs or not observed.is_cuda or observed.dtype not in (torch.bfloat16, torch.float32):
                return super().forward(observed)
            if observed.numel() == 0:
                return self
            c = float((self.args.observer_kwargs or {}).get("averaging_constant", 0.01))
            m = _MEMORYLESS if (mode == _AVERAGE and c == 1.0) else mode
            prev = self.has_statistics
            mn, mx = observe_activation_(observed, self.args, self.base_name, m, c,
                                         self.min_vals if prev else None, self.max_vals if prev else None)
            self.min_vals, self.max_vals = mn, mx
            self.fusion_handler.get_fused_statistics()
            return self

    GpuActivationObserver.__name__ = f"Gpu{ref_cls.__name__}"
    GpuActivationObserver.__qualname__ = GpuActivationObserver.__name__
    return GpuActivationObserver
