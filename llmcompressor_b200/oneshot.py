"""``oneshot`` with ``GPTQModifier`` / ``QuantizationModifier`` on the GPU.

Drop-in for the reference's entry point and modifiers on the
post-training-quantization path:

* ``oneshot(model, dataset, recipe=GPTQModifier(...))``
  (S/entrypoints/oneshot.py:285) with the sequential pipeline
  (S/pipelines/sequential/pipeline.py:55-178): the model is processed one
  decoder layer at a time; each layer sees the calibration data twice --
  a calibration pass whose forward hooks accumulate the GPTQ Hessians
  (S/modifiers/gptq/base.py:255-289), then, after the layer's weights are
  quantized (``on_sequential_epoch_end``, :239-321), a propagation pass whose
  outputs, computed with the quantized weights, become the next layer's
  inputs.
* ``GPTQModifier``: same arguments and scheme resolution as
  S/modifiers/gptq/base.py:44-193 (``actorder`` defaults to STATIC for
  schemes that leave it unset).
* ``QuantizationModifier``: round-to-nearest weight qparams
  (S/modifiers/quantization/quantization/base.py:85-137), no calibration
  data needed for weight-only schemes.

What is structured differently (the results are not):

* Layer inputs live on the GPU between layers (the reference offloads them
  to the CPU per batch, S/pipelines/cache.py), and calibration samples of
  equal length are stacked into batches of up to
  ``calibration_batch_tokens`` tokens per forward call; the Hessian counts
  samples (the batch dimension), as the reference does.
* Modules that read the same tensor in a forward pass (q/k/v, gate/up, the
  experts of an all-expert MoE layer) share one Hessian accumulation and one
  factorisation (the reference accumulates and factors identical copies).
* Layers are found as the reference's default sequential targets do: the
  model's ``_no_split_modules`` classes, in module order.

The arithmetic is the library's CUDA kernels (Hessians, factorisation, block
loop, observers); the decoder forward passes are the model's own torch code.
"""
from __future__ import annotations

import contextlib
import math
import time
from dataclasses import dataclass, field

import torch

from . import _lib, gptq, moe, ops
from .layer_forward import deferrable_down, defer_down, finish_deferred, fused_layer_ops

__all__ = ["oneshot", "GPTQModifier", "QuantizationModifier", "OneshotStats"]


class _Static:
    """The modifier-level ``actorder`` default: STATIC where the scheme
    leaves it unset (S/modifiers/gptq/base.py:142-160)."""

    def __repr__(self):
        return "Sentinel('static')"


_STATIC_DEFAULT = _Static()


def _schemes(targets, scheme, config_groups):
    """QuantizationSchemes of a modifier, in the precedence the reference's
    ``QuantizationMixin.resolve_quantization_config`` gives them."""
    from compressed_tensors.quantization import QuantizationScheme
    from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme

    targets = [targets] if isinstance(targets, str) else list(targets or ["Linear"])
    out = []
    if config_groups:
        for g in config_groups.values():
            out.append(g if isinstance(g, QuantizationScheme) else QuantizationScheme(**g))
        return out
    if scheme is None:
        raise ValueError("a scheme or config_groups is required")
    if isinstance(scheme, str):
        return [preset_name_to_scheme(scheme, targets)]
    if isinstance(scheme, QuantizationScheme):
        return [scheme]
    if isinstance(scheme, dict):
        if all(isinstance(k, str) and k.isupper() for k in scheme):  # {"W4A16": ["Linear"], ...}
            for name, tg in scheme.items():
                out.append(preset_name_to_scheme(name, [tg] if isinstance(tg, str) else list(tg)))
            return out
        return [QuantizationScheme(targets=targets, **scheme)]
    raise ValueError(f"unsupported scheme {scheme!r}")


class _Modifier:
    kind = ""

    def __init__(self, targets="Linear", scheme=None, config_groups=None, ignore=None, **kwargs):
        self.targets = targets
        self.scheme = scheme
        self.config_groups = config_groups
        self.ignore = list(ignore or [])
        self.extra = kwargs

    def resolve(self, model: torch.nn.Module) -> dict[str, tuple[torch.nn.Module, object]]:
        """name -> (module, QuantizationScheme) for every module to quantize."""
        from compressed_tensors.utils import match_named_modules

        found: dict[str, tuple[torch.nn.Module, object]] = {}
        for sch in self._resolved_schemes():
            for name, mod in match_named_modules(model, sch.targets, self.ignore):
                if name in found or sch.weights is None or isinstance(mod, torch.nn.Embedding):
                    continue
                found[name] = (mod, sch)
        if not found:
            raise ValueError(f"{type(self).__name__} was unable to find any modules to quantize. Please check "
                             "quantization `config_groups` and `targets` in recipe")
        return found

    def _resolved_schemes(self):
        return _schemes(self.targets, self.scheme, self.config_groups)


class GPTQModifier(_Modifier):
    """``GPTQModifier`` (S/modifiers/gptq/base.py:44-140): ``block_size``,
    ``dampening_frac``, ``actorder`` (default: STATIC unless the scheme sets
    one), ``offload_hessians`` (accepted; Hessians stay on the GPU),
    ``targets`` / ``scheme`` / ``config_groups`` / ``ignore``."""

    kind = "gptq"

    def __init__(self, targets="Linear", scheme=None, config_groups=None, ignore=None, block_size: int = 128,
                 dampening_frac: float | None = 0.01, actorder=_STATIC_DEFAULT, offload_hessians: bool = False,
                 **kwargs):
        super().__init__(targets, scheme, config_groups, ignore, **kwargs)
        self.block_size = int(block_size)
        self.dampening_frac = 0.01 if dampening_frac is None else float(dampening_frac)
        self.actorder = actorder
        self.offload_hessians = offload_hessians

    def _resolved_schemes(self):
        from compressed_tensors.quantization import QuantizationStrategy
        from compressed_tensors.quantization.quant_args import ActivationOrdering

        out = []
        for sch in super()._resolved_schemes():
            sch = sch.model_copy(deep=True)
            w = sch.weights
            if w is not None and w.strategy in (QuantizationStrategy.GROUP, QuantizationStrategy.TENSOR_GROUP,
                                                QuantizationStrategy.CHANNEL, QuantizationStrategy.TENSOR,
                                                QuantizationStrategy.BLOCK):
                existing = w.actorder
                if self.actorder is _STATIC_DEFAULT:
                    w.actorder = ActivationOrdering.STATIC if existing is None else existing
                elif existing is None or self.actorder == existing:
                    w.actorder = self.actorder
                else:
                    raise ValueError(
                        "Cannot resolve activation ordering when both `GPTQModifier.actorder` and "
                        f"`QuantizationScheme.actorder` are provided and differ ({self.actorder}, {existing}). "
                        "Either unset `GPTQModifier.actorder` or remove `actorder` from config groups.")
                if w.actorder == ActivationOrdering.GROUP and w.strategy not in (
                        QuantizationStrategy.GROUP, QuantizationStrategy.TENSOR_GROUP):
                    from loguru import logger

                    logger.warning(f"ActivationOrdering.GROUP is not compatible with strategy={w.strategy}; "
                                   "falling back to actorder=None for this scheme.")
                    w.actorder = None
            out.append(sch)
        return out


class QuantizationModifier(_Modifier):
    """``QuantizationModifier`` (S/modifiers/quantization/quantization/base.py):
    round-to-nearest weight qparams from the memoryless min-max observer.
    Weight-only schemes (and schemes whose activations are dynamic) need no
    calibration data; static activation schemes are not taken here."""

    kind = "rtn"


@dataclass
class OneshotStats:
    """Where the time of the last ``oneshot`` call went (wall seconds, host
    clock around synchronised phases) and the per-module GPTQ losses."""

    seconds: dict = field(default_factory=dict)
    losses: dict = field(default_factory=dict)
    samples: int = 0
    tokens: int = 0


LAST_STATS = OneshotStats()


# ------------------------------------------------------------------ data
def _calibration_batches(dataset, num_samples: int, batch_tokens: int, device) -> list[dict]:
    """Calibration samples as forward-call batches on ``device``: samples of
    equal length are stacked up to ``batch_tokens`` tokens per call."""
    samples: list[tuple[torch.Tensor, torch.Tensor | None]] = []

    def add(ids, mask=None):
        ids = torch.as_tensor(ids)
        if ids.ndim == 1:
            ids = ids.unsqueeze(0)
        mask = None if mask is None else torch.as_tensor(mask).reshape(ids.shape)
        for i in range(ids.shape[0]):
            samples.append((ids[i], None if mask is None else mask[i]))

    if isinstance(dataset, torch.Tensor):
        add(dataset)
    else:
        for item in dataset:
            if len(samples) >= num_samples:
                break
            if isinstance(item, dict):
                add(item["input_ids"], item.get("attention_mask"))
            elif isinstance(item, (list, tuple)):
                add(item[0], item[1] if len(item) > 1 else None)
            else:
                add(item)
    samples = samples[:num_samples]
    if not samples:
        raise ValueError("oneshot needs calibration samples")
    batches, i = [], 0
    while i < len(samples):
        L = samples[i][0].shape[-1]
        per = max(1, batch_tokens // max(1, L))
        j = i
        while j < len(samples) and j - i < per and samples[j][0].shape[-1] == L:
            j += 1
        ids = torch.stack([s[0] for s in samples[i:j]]).to(device, non_blocking=True)
        masks = [s[1] for s in samples[i:j]]
        batch = {"input_ids": ids}
        if any(m is not None for m in masks):
            batch["attention_mask"] = torch.stack(
                [m if m is not None else torch.ones_like(s[0]) for m, s in zip(masks, samples[i:j])]).to(device)
        batches.append(batch)
        i = j
    return batches


# ------------------------------------------------------------------ layers
def sequential_layers(model: torch.nn.Module, targets=None) -> list[torch.nn.Module]:
    """The decoder layers, in order: modules whose class is named in
    ``targets`` or, by default, in the model's ``_no_split_modules`` (the
    reference's ``infer_sequential_targets``)."""
    names = targets or getattr(model, "_no_split_modules", None) or []
    names = [names] if isinstance(names, str) else list(names)
    layers = [m for m in model.modules() if type(m).__name__ in names]
    if not layers:
        raise ValueError(f"no sequential target layers ({names}) found in {type(model).__name__}")
    return layers


class _Stop(Exception):
    pass


@torch.no_grad()
def _capture_layer_inputs(model, first_layer, batches) -> list[tuple[torch.Tensor, dict]]:
    """Run the model up to the first decoder layer for every batch and keep
    that layer's inputs (hidden states and keyword arguments)."""
    got = []

    def pre(mod, args, kwargs):
        got.append((args[0], dict(kwargs), args[1:]))
        raise _Stop

    h = first_layer.register_forward_pre_hook(pre, with_kwargs=True)
    try:
        for b in batches:
            try:
                model(**b, use_cache=False)
            except _Stop:
                pass
    finally:
        h.remove()
    return got


def _layer_out(out):
    return out[0] if isinstance(out, (tuple, list)) else out


# ------------------------------------------------------------------ modules
def _init_modules(found: dict) -> None:
    """Attach the compressed-tensors quantization parameters and scheme to
    every module (``initialize_module_for_quantization``), with fake-quant
    in the forward disabled while calibrating (``DisableQuantization``)."""
    from compressed_tensors.quantization import initialize_module_for_quantization
    from compressed_tensors.quantization.lifecycle.helpers import disable_quantization

    for _, (mod, sch) in found.items():
        initialize_module_for_quantization(mod, sch, force_zero_point=False)
        disable_quantization(mod)


def _finish_modules(found: dict) -> None:
    from compressed_tensors.quantization import QuantizationStatus
    from compressed_tensors.quantization.lifecycle.helpers import enable_quantization

    for _, (mod, _) in found.items():
        mod.quantization_status = QuantizationStatus.FROZEN
        enable_quantization(mod)


def _set_params(mod: torch.nn.Module, q: dict) -> None:
    """``update_offload_parameter(module, attr, val)`` for every result the
    module has a parameter for (compressed-tensors creates them at
    initialization: no zero point for symmetric schemes), plus ``weight_g_idx``
    / ``weight_global_scale``, registered when missing."""
    for k, v in q.items():
        p = getattr(mod, k, None)
        if isinstance(p, torch.nn.Parameter):
            if p.shape == v.shape:
                p.data.copy_(v.to(p.dtype))
            else:
                p.data = v.to(p.dtype)
        elif k in ("weight_g_idx", "weight_global_scale"):
            mod.register_parameter(k, torch.nn.Parameter(v, requires_grad=False))


def _rtn(found: dict) -> None:
    """Round-to-nearest weight qparams for every module (GPU observers)."""
    for name, (mod, sch) in found.items():
        qa = sch.weights
        mn, mx = ops.observe_minmax(mod.weight, qa)
        gs = None
        if getattr(qa.strategy, "value", qa.strategy) == "tensor_group":
            gs = ops.fused_global_scale(gptq._fused_weights(mod))
        scale, zp = ops.calculate_qparams(mn, mx, qa, gs)
        q = {"weight_scale": scale.to(mod.weight.dtype) if scale.dtype != torch.float32 or gs is None else scale,
             "weight_zero_point": zp}
        if gs is not None:
            q["weight_global_scale"] = gs
        _set_params(mod, q)


def _rtn_dist(found: dict, rank: int, ws: int) -> None:
    """Round-to-nearest qparams under DDP
    (``QuantizationModifier.on_sequential_epoch_end`` and
    ``_broadcast_qparam_onloads``, S/modifiers/quantization/quantization/base.py:85-137):
    modules are split across ranks by weight size (greedy bin packing), each
    rank observes its own, and every module's qparams are broadcast from its
    owner.  Every rank issues the same broadcasts in the same order."""
    import torch.distributed as dist

    from .distributed import greedy_owners

    owners = greedy_owners({n: float(m.weight.numel()) for n, (m, _) in found.items()}, ws)
    _rtn({n: v for n, v in found.items() if owners[n] == rank})
    works = []
    for n in sorted(found):
        mod = found[n][0]
        for attr in ("weight_scale", "weight_zero_point", "weight_global_scale"):
            t = getattr(mod, attr, None)
            if isinstance(t, torch.Tensor):
                works.append(dist.broadcast(t.data, src=owners[n], async_op=True))
    for w in works:
        w.wait()


# ------------------------------------------------------------------ GPTQ per layer
class _LayerCalibration:
    """Forward pre-hooks on one layer's quantized modules: modules that read
    the same tensor in a forward pass share one Hessian (``BatchedHessian``).

    The calibration pass only needs the modules' inputs; its layer output is
    discarded (the propagation pass recomputes it with the quantized
    weights).  So after the first batch, which runs whole and fixes the order
    in which the modules are called, the pass stops at the input of the last
    module called (for a Llama layer: before the down projection's GEMM)."""

    def __init__(self, modules: dict[str, torch.nn.Module], layer: torch.nn.Module | None = None,
                 all_experts: bool = False):
        self.modules = modules  # name -> module
        self.group_of: dict[str, int] = {}
        self.groups: list[list[str]] = []
        self.hess: list = []
        self.order: list[str] = []
        self._seen: dict[int, tuple] = {}
        self._handles = []
        self._sinks: list[moe.LinearExperts] = []
        self._first = True
        sunk: set[str] = set()
        if layer is not None and all_experts:
            name_of = {id(m): n for n, m in modules.items()}
            for le in layer.modules():
                if not isinstance(le, moe.LinearExperts):
                    continue
                names = [name_of.get(id(lin)) for ex in le for lin in (ex.gate_proj, ex.up_proj, ex.down_proj)]
                if all(names) and le.stacked_ready():
                    self._add_sink(le, names)
                    sunk.update(names)
        for name, mod in modules.items():
            if name not in sunk:
                self._handles.append(mod.register_forward_pre_hook(self._hook(name)))

    def _add_sink(self, le: "moe.LinearExperts", names: list[str]) -> None:
        """Experts in stacked all-expert form: every expert's gate/up share
        one Hessian of the block input; the experts' down inputs arrive
        concatenated and one grouped launch accumulates all their Hessians."""
        E = le.num_experts
        ex0 = le[0]
        inter, hidden = ex0.gate_proj.out_features, ex0.gate_proj.in_features
        dev = ex0.gate_proj.weight.device
        gu = [names[3 * e + k] for e in range(E) for k in (0, 1)]
        g_gu = len(self.groups)
        self.groups.append(gu)
        self.hess.append(gptq.BatchedHessian(hidden, dev))
        for n in gu:
            self.group_of[n] = g_gu
        down = _GroupedHessian(E, inter, dev)
        for e in range(E):
            n = names[3 * e + 2]
            self.group_of[n] = len(self.groups)
            self.groups.append([n])
            self.hess.append(down.view(e))
        key = f"experts@{id(le)}"

        def sink(mod, x, act):
            self.hess[g_gu].add(x)
            down.add(act)
            if self._first:
                self.order.append(key)
            elif self.order[-1] == key:
                raise _Stop

        le.calib_sink = sink
        self._sinks.append(le)

    def _hook(self, name):
        def hook(mod, args):
            x = args[0]
            if self._first:
                # the first batch decides the groups; the inputs are held until
                # it ends, so no id is reused by another tensor meanwhile
                g = self._seen.get(id(x), (None,))[0]
                if g is None:
                    g = len(self.groups)
                    self._seen[id(x)] = (g, x)
                    self.groups.append([])
                    self.hess.append(gptq.BatchedHessian(x.shape[-1], x.device))
                    self.hess[g].add(x)
                self.groups[g].append(name)
                self.group_of[name] = g
                self.order.append(name)
                return None
            g = self.group_of[name]
            if self.groups[g][0] == name:
                self.hess[g].add(x)
            if name == self.order[-1]:
                raise _Stop
            return None
        return hook

    def run(self, layer, h, rest, kw) -> None:
        """One calibration batch through the layer."""
        try:
            layer(h, *rest, **kw)
        except _Stop:
            pass
        self._first = False
        self._seen.clear()

    def remove(self):
        for h in self._handles:
            h.remove()
        self._handles = []
        for le in self._sinks:
            le.calib_sink = None
        self._sinks = []


class _GroupedHessian:
    """Block-diagonal Hessians of E experts' down projections, H (E*d, d),
    from their concatenated inputs (tokens, E*d): one grouped launch per
    batch.  ``view(e)`` is expert e's Hessian with ``BatchedHessian``'s
    interface (``finalize``, ``samples``, ``d``, ``H``)."""

    def __init__(self, E: int, d: int, device):
        self.E, self.d = int(E), int(d)
        self.H = torch.zeros(self.E * self.d, self.d, dtype=gptq.GPTQ_PRECISION, device=device)
        self.samples = 0

    def add(self, inp: torch.Tensor) -> None:
        self.samples += inp.shape[0] if inp.ndim > 2 else 1
        gptq.hessian_update_(self.H, inp.reshape(-1, self.E * self.d), 2.0, groups=self.E)

    def view(self, e: int) -> "_GroupView":
        return _GroupView(self, e)


class _GroupView:
    def __init__(self, parent: _GroupedHessian, e: int):
        self.parent, self.d = parent, parent.d
        self.H = parent.H[e * parent.d:(e + 1) * parent.d]
        self._buf = None

    @property
    def samples(self) -> int:
        return self.parent.samples

    def finalize(self) -> tuple[torch.Tensor, torch.Tensor]:
        return self.H, torch.full((), float(self.parent.samples), dtype=torch.float32, device=self.H.device)


def _solve_layer(cal: _LayerCalibration, found: dict, modifier: GPTQModifier, stats: OneshotStats,
                 defer: set | None = None) -> list:
    """Factor each group's Hessian once and quantize its modules; groups run
    concurrently on side streams (largest Hessian first), the caller's stream
    waits for all of them -- except the groups whose modules are all in
    ``defer``: their completion events are returned instead."""
    from .pipeline import _side_streams

    dev = next(iter(cal.modules.values())).weight.device
    main = torch.cuda.current_stream(dev)
    jobs, singles = _expert_batches(cal, found)
    order = sorted(singles, key=lambda g: -cal.hess[g].d)
    streams = _side_streams(dev, max(1, min(MAX_SIDE_STREAMS, len(order) + len(jobs))))
    done, deferred = [], []
    results = []
    for j, (gs, names, mods, qa) in enumerate(jobs):
        # experts' down projections: one batched solve over their Hessians
        st = streams[j % len(streams)]
        st.wait_stream(main)
        with torch.cuda.stream(st):
            Hp, n = cal.hess[gs[0]].parent.H, cal.hess[gs[0]].finalize()[1]
            Hp.record_stream(st)
            Hb = Hp / n  # the reference's hessian / num_samples, per expert (as the single-group path divides)
            status, res = gptq.quantize_batched(mods, qa, Hb, modifier.block_size, modifier.dampening_frac)
            for e, (nm, mod, (loss, q)) in enumerate(zip(names, mods, res)):
                _set_params(mod, q)
                results.append((nm, loss, gptq.BatchStatus(status, e)))
            ev = torch.cuda.Event()
            ev.record(st)
            done.append(ev)
        for g in gs:
            cal.hess[g] = None
    for i, g in enumerate(order, start=len(jobs)):
        st = streams[i % len(streams)]
        st.wait_stream(main)
        with torch.cuda.stream(st):
            bh = cal.hess[g]
            H, n = bh.finalize()
            for t in (bh.H, bh._buf):  # allocated on the caller's stream, read on this one
                if t is not None:
                    t.record_stream(st)
            H = H / n  # the reference's hessian / num_samples (S/modifiers/gptq/base.py:594)
            names = cal.groups[g]
            mods = [cal.modules[nm] for nm in names]
            qas = [found[nm][1].weights for nm in names]
            hinv, res = gptq.quantize_modules_shared(mods, qas, H, modifier.block_size, modifier.dampening_frac)
            for nm, mod, (loss, q) in zip(names, mods, res):
                _set_params(mod, q)
                results.append((nm, loss, hinv))
            ev = torch.cuda.Event()
            ev.record(st)
            (deferred if defer and set(names) <= defer else done).append(ev)
        cal.hess[g] = None  # release the Hessian buffers with the stream's work
    for ev in done:
        main.wait_event(ev)
    for nm, loss, hinv in results:
        stats.losses[nm] = (loss, hinv)
    return deferred


MAX_SIDE_STREAMS = 8  # concurrent solve streams (an MoE layer has one Hessian group per expert)
DEFER_BYTES = 8 << 30  # down-projection inputs held while the down projection's solve finishes


def _expert_batches(cal: _LayerCalibration, found: dict):
    """Split the layer's Hessian groups into batched solves (the groups of
    one grouped expert Hessian whose modules ``gptq.batchable`` takes: one
    module per expert, one shape and scheme) and the rest.  Returns
    ([(groups, names, modules, quant_args)], [other groups])."""
    by_parent: dict[int, list[int]] = {}
    singles = []
    for g in range(len(cal.groups)):
        h = cal.hess[g]
        if isinstance(h, _GroupView) and len(cal.groups[g]) == 1:
            by_parent.setdefault(id(h.parent), []).append(g)
        else:
            singles.append(g)
    jobs = []
    for gs in by_parent.values():
        names = [cal.groups[g][0] for g in gs]
        mods = [cal.modules[n] for n in names]
        qas = [found[n][1].weights for n in names]
        orders = [gptq.resolve_actorder(getattr(qa, "actorder", None)) for qa in qas]
        if len(gs) == cal.hess[gs[0]].parent.E and gptq.batchable(mods, qas, orders):
            jobs.append((gs, names, mods, qas[0]))
        else:
            singles.extend(gs)
    return jobs, singles


def _check_losses(stats: OneshotStats) -> None:
    """One host sync at the end: losses to floats, RTN-fallback warnings,
    kernel timeouts."""
    warned = set()
    for nm, v in list(stats.losses.items()):
        if isinstance(v, tuple):
            loss, hinv = v
            if id(hinv) not in warned:
                warned.add(id(hinv))
                if not hinv.ok():
                    gptq._warn_fallback()
            stats.losses[nm] = float(loss.item())


# ------------------------------------------------------------------ multi-GPU solve
def _solve_layer_dist(cal: _LayerCalibration, found: dict, modifier: GPTQModifier, stats: OneshotStats,
                      rank: int, ws: int, defer: set | None = None) -> list:
    """The multi-rank form of ``_solve_layer`` (the reference's
    ``compress_modules`` under DDP, S/modifiers/gptq/base.py:291-321,603-645,
    restructured): every shared Hessian is summed onto an owner rank chosen by
    solve cost, the owner factors it and broadcasts the upper factor (each
    rank forms its transpose locally), every rank quantizes an equal slice of
    the group's (stacked) rows, and the quantized rows are all-gathered so
    that every rank holds the whole quantized layer for the propagation pass.

    Groups go smallest Hessian first, each on its own stream: the owners'
    factorisations run concurrently, and the collectives are issued group by
    group (broadcast, then the row gathers) so that the small groups' row
    solves and gathers proceed while the largest factorisation is still
    running.  Every rank issues the same collectives in the same order."""
    import torch.distributed as dist

    from .distributed import greedy_owners, solve_cost
    from .pipeline import _side_streams

    dev = next(iter(cal.modules.values())).weight.device
    main = torch.cuda.current_stream(dev)
    jobs, singles = _expert_batches(cal, found)
    for job in jobs:  # experts first: owned by ranks, solved in batches
        _solve_experts_dist(cal, job, modifier, stats, rank, ws, dev)
    # the remaining groups, renumbered
    cal.groups = [cal.groups[g] for g in sorted(singles)]
    cal.hess = [cal.hess[g] for g in sorted(singles)]
    ng = len(cal.groups)
    if ng == 0:
        return []
    # pinned staging: a pageable host-to-device copy would wait for the stream
    counts = torch.tensor([float(cal.hess[g].samples) for g in range(ng)], dtype=torch.float64).pin_memory()
    counts = counts.to(dev, non_blocking=True)
    Hs = [cal.hess[g].finalize()[0] for g in range(ng)]
    dist.all_reduce(counts)
    keys = [f"g{g}" for g in range(ng)]
    rows_total = {f"g{g}": sum(cal.modules[n].weight.shape[0] for n in cal.groups[g]) for g in range(ng)}
    owners = greedy_owners({k: solve_cost(Hs[g].shape[0], rows_total[k]) for g, k in enumerate(keys)}, ws)
    order = sorted(range(ng), key=lambda g: (Hs[g].shape[0], g))  # smallest Hessian first
    nst = max(1, min(MAX_SIDE_STREAMS, ng))
    streams = _side_streams(dev, nst)
    red = {g: dist.reduce(Hs[g], dst=owners[keys[g]], async_op=True) for g in order}
    invs = {}
    done, deferred = [], []
    for i, g in enumerate(order):
        st = streams[(ng - 1 - i) % nst]  # the largest Hessian (the critical path) gets the high-priority stream
        st.wait_stream(main)
        names = cal.groups[g]
        qa0 = found[names[0]][1].weights
        act = gptq.resolve_actorder(getattr(qa0, "actorder", None))
        d = Hs[g].shape[0]
        with torch.cuda.stream(st):
            red[g].wait()
            if owners[keys[g]] == rank:
                inv = gptq.inverse_hessian(Hs[g] / counts[g].float(), modifier.dampening_frac, act)
            else:
                inv = gptq.InverseHessian(torch.empty(d, d, dtype=torch.float32, device=dev),
                                          torch.empty(d, dtype=torch.uint8, device=dev),
                                          torch.empty(1, dtype=torch.int32, device=dev), None,
                                          torch.empty(d, dtype=torch.int32, device=dev) if act else None)
            ts = (inv.hinv, inv.dead, inv.status) + ((inv.perm,) if inv.perm is not None else ())
            for w in [dist.broadcast(t, src=owners[keys[g]], async_op=True) for t in ts]:
                w.wait()
            if inv.hinv_t is None:
                inv.hinv_t = inv.hinv.t().contiguous()
            invs[g] = inv
            _solve_group_rows(cal, g, found, modifier, stats, inv, rank, ws, dev)
            ev = torch.cuda.Event()
            ev.record(st)
            (deferred if defer and set(names) <= defer else done).append(ev)
        cal.hess[g] = None
    for ev in done:
        main.wait_event(ev)
    return deferred


def _solve_experts_dist(cal, job, modifier, stats, rank: int, ws: int, dev) -> None:
    """One batched expert solve across ranks (experts assigned to ranks, as
    the reference assigns modules to owners): the experts' Hessians are
    summed and scattered by owner in one reduce-scatter, every rank solves
    its own experts in one batched call, and the quantized weights, qparams,
    losses and statuses are all-gathered so that every rank holds the whole
    quantized layer."""
    import torch.distributed as dist

    from .distributed import row_range

    gs, names, mods, qa = job
    E = len(gs)
    parent = cal.hess[gs[0]].parent
    d = parent.d
    rows = mods[0].weight.shape[0]
    per = -(-E // ws)  # experts per rank, the last ranks padded
    cnt = torch.full((1,), float(parent.samples), dtype=torch.float32, device=dev)
    dist.all_reduce(cnt)
    Hfull = parent.H if per * ws == E else torch.cat(
        [parent.H, torch.zeros((per * ws - E) * d, d, dtype=parent.H.dtype, device=dev)])
    Hmine = torch.empty(per * d, d, dtype=parent.H.dtype, device=dev)
    dist.reduce_scatter_tensor(Hmine, Hfull)
    for g in gs:
        cal.hess[g] = None
    del Hfull
    e0, e1 = row_range(E, rank, ws)  # rank r owns experts [r*per, min(E, (r+1)*per))
    k = e1 - e0
    # qparams dtypes and per-row shape, the same on every rank (a rank may own no expert)
    from . import ops

    mn1, mx1 = ops.observe_minmax(mods[0].weight.detach()[:1], qa)
    s1, z1 = ops.calculate_qparams(mn1, mx1, qa)
    parts = [torch.zeros((per, rows, d), dtype=torch.bfloat16, device=dev),
             torch.zeros((per * rows,) + tuple(s1.shape[1:]), dtype=s1.dtype, device=dev),
             torch.zeros((per * rows,) + tuple(z1.shape[1:]), dtype=z1.dtype, device=dev),
             torch.zeros((per,), dtype=torch.float32, device=dev),
             torch.zeros((per,), dtype=torch.int32, device=dev)]
    if k > 0:
        Hb = (Hmine[: k * d] / cnt).contiguous()
        for dst, src in zip(parts, gptq.solve_batched(mods[e0:e1], qa, Hb, modifier.block_size,
                                                      modifier.dampening_frac)):
            dst[: src.shape[0]] = src
    del Hmine
    gathered = []
    for t in parts:
        full = torch.empty((t.shape[0] * ws,) + tuple(t.shape[1:]), dtype=t.dtype, device=dev)
        dist.all_gather_into_tensor(full, t)
        gathered.append(full)
    out_all, scale_all, zp_all, loss_all, status_all = gathered
    # rank r's experts sit at [r*per, r*per + its count): back to expert order
    idx = torch.cat([torch.arange(r * per, r * per + (row_range(E, r, ws)[1] - row_range(E, r, ws)[0]),
                                  device=dev) for r in range(ws)])
    ridx = (idx[:, None] * rows + torch.arange(rows, device=dev)[None, :]).reshape(-1)
    res = gptq.batched_param_dicts(mods, qa, out_all[idx], scale_all[ridx], zp_all[ridx], loss_all[idx])
    status_e = status_all[idx]
    for e, (nm, mod, (loss, q)) in enumerate(zip(names, mods, res)):
        _set_params(mod, q)
        stats.losses[nm] = (loss, gptq.BatchStatus(status_e, e))


def _solve_group_rows(cal, g, found, modifier, stats, inv, rank, ws, dev) -> None:
    """Quantize this rank's share of group ``g``'s rows against the shared
    factor and all-gather the quantized rows (on the current stream)."""
    names = cal.groups[g]
    mods = [cal.modules[nm] for nm in names]
    qas = [found[nm][1].weights for nm in names]
    orders = [gptq.resolve_actorder(getattr(qa, "actorder", None)) for qa in qas]
    if len(mods) > 1 and gptq._stackable(mods, qas, orders):
        # one row split over the stacked rows of the group's modules
        qp = [gptq.weight_qparams(m, qas[0]) for m in mods]
        w = torch.cat([m.weight.detach() for m in mods])
        scale = torch.cat([q[0] for q in qp])
        zp = torch.cat([q[1] for q in qp])
        wq_full, row_loss = _solve_rows_dist(w, qas[0], inv, scale, zp, None, None, orders[0], 1,
                                             modifier.block_size, rank, ws, dev)
        r0 = 0
        for nm, mod, (sc, z, _) in zip(names, mods, qp):
            r1 = r0 + mod.weight.shape[0]
            _set_params(mod, {"weight": wq_full[r0:r1], "weight_scale": sc.to(mod.weight.dtype),
                              "weight_zero_point": z})
            stats.losses[nm] = (row_loss[r0:r1].sum().reshape(1), inv)
            r0 = r1
        return
    for nm, mod, qa, order in zip(names, mods, qas, orders):
        align = int(qa.block_structure[0]) if getattr(qa.strategy, "value", qa.strategy) == "block" else 1
        g_idx = None
        if order == "group":
            wp = gptq.permute_columns(mod.weight, inv.perm)
            scale, zp, gs = gptq.weight_qparams(mod, qa, weight=wp, stats_dtype=torch.float32)
            g_idx = torch.empty(mod.weight.shape[1], dtype=torch.int32, device=dev)
        else:
            scale, zp, gs = gptq.weight_qparams(mod, qa)
        wq_full, row_loss = _solve_rows_dist(mod.weight.detach(), qa, inv, scale, zp, gs, g_idx, order, align,
                                             modifier.block_size, rank, ws, dev)
        q = {"weight": wq_full, "weight_scale": scale.to(mod.weight.dtype), "weight_zero_point": zp}
        if gs is not None:
            q["weight_global_scale"] = gs.to(mod.weight.dtype)
        if g_idx is not None:
            q["weight_g_idx"] = g_idx
        _set_params(mod, q)
        stats.losses[nm] = (row_loss.sum().reshape(1), inv)


def _solve_rows_dist(w, qa, inv, scale, zp, gs, g_idx, order, align, blocksize, rank, ws, dev):
    """This rank's slice of the rows of ``w`` through the block loop, then
    every rank's rows and per-row losses all-gathered."""
    from .distributed import all_gather_rows, row_range

    rows = w.shape[0]
    r0, r1 = row_range(rows, rank, ws, align)

    def srow(t):
        return t if t is None or t.numel() <= 1 else t[r0 // align:(r1 + align - 1) // align]

    wq_full = torch.empty_like(w)
    row_loss_full = torch.empty(rows, dtype=torch.float32, device=dev)
    if r1 > r0:
        rl = torch.empty(r1 - r0, dtype=torch.float32, device=dev)
        wq, _ = gptq.quantize_with_inverse(w[r0:r1], qa, inv, srow(scale), srow(zp), blocksize, order, gs, g_idx,
                                           rl)
    else:
        wq = w[r0:r0]
        rl = torch.empty(0, dtype=torch.float32, device=dev)
    all_gather_rows(wq, wq_full, rows, align)
    all_gather_rows(rl, row_loss_full, rows, align)
    return wq_full, row_loss_full


# ------------------------------------------------------------------ entry point
class SequentialRunner:
    """The layer-by-layer GPTQ pipeline behind ``oneshot`` with its steps
    exposed: ``capture()`` runs the model up to the first layer for every
    calibration batch, ``run_layer(i)`` calibrates, quantizes and propagates
    decoder layer i, ``finish()`` reads the losses and errors back and marks
    the modules frozen.  ``bench.py`` times ``run_layer`` steps."""

    def __init__(self, model, modifiers, batches, device, sequential_targets=None, offload_layers=False,
                 moe_calibrate_all_experts: bool = True, fused_forward: bool = True,
                 moe_routed_propagation: bool = True):
        self.model = model
        self.fused = fused_forward
        # the propagation pass needs only the routed experts' outputs, which
        # all-expert mode computes too (and then discards for unrouted tokens)
        self.routed_propagation = moe_routed_propagation
        self.device = device
        self.offload = offload_layers
        self.all_experts = moe_calibrate_all_experts
        self.stats = OneshotStats()
        if moe.linearize_experts(model):
            # fused experts become per-expert Linear modules (the reference's
            # post-load linearize_moe) before the modules are matched
            from loguru import logger

            logger.info("MoE experts linearized into per-expert Linear modules for calibration")
        from .distributed import world

        self.rank, self.ws = world()
        found_all = {}
        for m in modifiers:
            for k, v in m.resolve(model).items():
                found_all.setdefault(k, (v[0], v[1], m))
        self.found = {k: (v[0], v[1]) for k, v in found_all.items()}
        self.gptq_found = {k: (v[0], v[1]) for k, v in found_all.items() if v[2].kind == "gptq"}
        self.rtn_found = {k: (v[0], v[1]) for k, v in found_all.items() if v[2].kind == "rtn"}
        gm = [m for m in modifiers if m.kind == "gptq"]
        self.modifier = gm[0] if gm else None
        _init_modules(self.found)
        self.layers = sequential_layers(model, sequential_targets) if self.gptq_found else []
        self.batches = batches
        self.cache = None
        self._host: dict[int, torch.Tensor] = {}
        self._name_of = {id(m): n for n, (m, _) in self.gptq_found.items()}

    def capture(self) -> None:
        self.cache = _capture_layer_inputs(self.model, self.layers[0], self.batches)
        self.stats.samples = sum(b["input_ids"].shape[0] for b in self.batches)
        self.stats.tokens = sum(b["input_ids"].numel() for b in self.batches)

    @torch.no_grad()
    def run_layer(self, li: int, phases: list | None = None, propagate: bool | None = None) -> None:
        """Calibrate, quantize and (unless it is the last layer) propagate
        layer ``li``.  ``phases``: if a list, CUDA events marking the ends of
        onload / calibration / solve / propagation / offload are appended."""
        def mark(name):
            if phases is not None:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                phases.append((name, e))

        layer = self.layers[li]
        will_propagate = propagate if propagate is not None else li + 1 < len(self.layers)
        pending: list = []
        mark("start")
        if self.offload:
            self._onload(layer)
        mark("onload")
        lm = {self._name_of[id(m)]: m for m in layer.modules() if id(m) in self._name_of}
        if lm:
            cal = _LayerCalibration(lm, layer, self.all_experts)
            with moe.calibrate_all_experts(self.all_experts), fused_layer_ops(layer, enabled=self.fused):
                for (h, kw, rest) in self.cache:
                    cal.run(layer, h, rest, kw)
            cal.remove()
            mark("calibrate")
            # the down projection's solve may finish behind the first batches'
            # propagation up to their down projections (deferred below)
            down = deferrable_down(layer) if self.fused and will_propagate else None
            defer = {self._name_of[id(down)]} if down is not None and id(down) in self._name_of else None
            if self.ws > 1:
                pending = _solve_layer_dist(cal, self.gptq_found, self.modifier, self.stats, self.rank, self.ws,
                                            defer)
            else:
                pending = _solve_layer(cal, self.gptq_found, self.modifier, self.stats, defer)
            mark("solve")
        mods = set(id(m) for m in layer.modules())
        rl = {n: v for n, v in self.rtn_found.items() if id(v[0]) in mods}
        if rl:
            _rtn(rl)
        main = torch.cuda.current_stream()
        if will_propagate:
            # propagate: the quantized layer's outputs are the next layer's inputs.
            # The reference keeps MoE layers in all-expert mode here too, whose
            # output keeps only the routed tokens' expert outputs: the routed
            # forward gives the same sum without the unrouted experts' work.
            all_ex = self.all_experts and not self.routed_propagation
            with moe.calibrate_all_experts(all_ex), fused_layer_ops(layer, enabled=self.fused):
                start = 0
                if pending:
                    # the first batches up to the down projection while its
                    # solve finishes, then their down projections
                    h0 = self.cache[0][0]
                    per = (h0.numel() // h0.shape[-1]) * down.in_features * h0.element_size()
                    start = min(len(self.cache), max(1, DEFER_BYTES // per))
                    store: list = []
                    with defer_down(store):
                        outs = [layer(h, *rest, **kw) for (h, kw, rest) in self.cache[:start]]
                    for ev in pending:
                        main.wait_event(ev)
                    it = iter(store)
                    for i, o in enumerate(outs):
                        _, kw, rest = self.cache[i]
                        self.cache[i] = (finish_deferred(next(it)) if o is None else _layer_out(o), kw, rest)
                    del store, outs
                for i in range(start, len(self.cache)):
                    h, kw, rest = self.cache[i]
                    self.cache[i] = (_layer_out(layer(h, *rest, **kw)), kw, rest)
        for ev in pending:
            main.wait_event(ev)
        moe.release_stacked()  # this layer's stacked expert weights, if any
        mark("propagate")
        if self.offload:
            self._offload(layer)
        mark("offload")

    def _onload(self, layer: torch.nn.Module) -> None:
        """Layer parameters to the device (from pinned host memory when the
        host copies are pinned: asynchronous on the current stream)."""
        for mod in layer.modules():
            for k, p in list(mod._parameters.items()):
                if p is not None and not p.is_cuda:
                    host = p.data
                    p.data = torch.empty_like(host, device=self.device)
                    p.data.copy_(host, non_blocking=host.is_pinned())
                    self._host[id(p)] = host
            for k, b in list(mod._buffers.items()):
                if b is not None and not b.is_cuda:
                    mod._buffers[k] = b.to(self.device)

    def _offload(self, layer: torch.nn.Module) -> None:
        """Layer parameters back to the host (into their pinned host copies
        when they have one, else new host tensors)."""
        for mod in layer.modules():
            for k, p in list(mod._parameters.items()):
                if p is None or not p.is_cuda:
                    continue
                host = self._host.pop(id(p), None)
                if host is not None and host.shape == p.shape and host.dtype == p.dtype:
                    host.copy_(p.data, non_blocking=host.is_pinned())
                    p.data = host
                else:
                    p.data = p.data.to("cpu")

    def finish(self) -> OneshotStats:
        in_layers = set(id(m) for l in self.layers for m in l.modules())
        rest = {n: v for n, v in self.gptq_found.items() if id(v[0]) not in in_layers}
        if rest:
            raise NotImplementedError(f"GPTQ targets outside the sequential layers: {sorted(rest)[:4]}")
        rtn_rest = {n: v for n, v in self.rtn_found.items() if id(v[0]) not in in_layers}
        if rtn_rest:
            for _, (mod, _) in rtn_rest.items():
                if not mod.weight.is_cuda:
                    mod.to(self.device)
            if self.ws > 1:
                _rtn_dist(rtn_rest, self.rank, self.ws)
            else:
                _rtn(rtn_rest)
        _check_losses(self.stats)
        _lib.check_device_errors(self.device, "oneshot")
        _finish_modules(self.found)
        self.cache = None
        return self.stats


def oneshot(
    model: torch.nn.Module,
    dataset=None,
    recipe=None,
    num_calibration_samples: int = 512,
    shuffle_calibration_samples: bool = True,
    pipeline: str | None = "sequential",
    sequential_targets=None,
    calibration_batch_tokens: int = 16384,
    device: torch.device | str | None = None,
    offload_layers: bool | None = None,
    moe_calibrate_all_experts: bool = True,
    fused_forward: bool = True,
    **kwargs,
) -> torch.nn.Module:
    """``oneshot`` (S/entrypoints/oneshot.py:285) for a ``GPTQModifier`` or
    ``QuantizationModifier`` recipe on a decoder model.

    ``dataset``: a DataLoader / iterable of ``{"input_ids", "attention_mask"}``
    samples or an (n, L) tensor of token ids; the first
    ``num_calibration_samples`` are used in order (a DataLoader's own order;
    shuffling is the DataLoader's business, as in the reference when one is
    passed).  Under ``torch.distributed`` every rank passes the same dataset
    and calibrates its own contiguous share of the samples, as the
    reference's DDP oneshot does with its per-rank data.  ``device``: the GPU
    to calibrate on (default: the model's, or the current CUDA device).  A
    model left on the CPU is moved there one layer at a time and each
    quantized layer is moved back (``offload_layers``, default: True when the
    model starts on the CPU).  Returns the model with quantized weights and
    compressed-tensors scales and zero points, ready for ``save_compressed``.
    Mixture-of-experts models have their fused experts split into per-expert
    Linear modules first; with ``moe_calibrate_all_experts`` (the default, as
    in the reference) every expert sees every token in the calibration pass.
    ``fused_forward``: run the decoder layers' elementwise ops (RMSNorm,
    rotary, SiLU * up, residual add) as fused kernels in the calibration and
    propagation passes (``layer_forward.fused_layer_ops``); False runs the HF
    forwards as they are.
    """
    mods = recipe if isinstance(recipe, (list, tuple)) else [recipe]
    mods = [m for m in mods if m is not None]
    if not mods:
        raise ValueError("oneshot needs a recipe (GPTQModifier or QuantizationModifier)")
    for m in mods:
        if not isinstance(m, _Modifier):
            raise NotImplementedError(f"recipe entry {type(m).__name__}: only GPTQModifier and "
                                      "QuantizationModifier run on this path")
    if pipeline not in (None, "sequential", "independent", "basic", "datafree"):
        raise ValueError(f"unknown pipeline {pipeline!r}")
    first_param = next(model.parameters())
    if device is None:
        device = first_param.device if first_param.is_cuda else torch.device("cuda", torch.cuda.current_device())
    device = torch.device(device)
    if offload_layers is None:
        offload_layers = not first_param.is_cuda
    t_all = time.perf_counter()
    needs_data = any(m.kind == "gptq" for m in mods)
    if not needs_data:
        # weight-only RTN: no calibration pass (the qparams do not depend on data)
        runner = SequentialRunner(model, mods, [], device)
        stats = runner.finish()  # every module is outside the (absent) GPTQ layers: round-to-nearest there
        stats.seconds["total"] = time.perf_counter() - t_all
        globals()["LAST_STATS"] = stats
        return model
    if dataset is None:
        raise ValueError("GPTQ needs calibration data (dataset)")
    from .distributed import row_range, world

    rank, ws = world()
    layers = sequential_layers(model, sequential_targets)
    if offload_layers:
        _to_device_except(model, {id(l) for l in layers}, device)
    else:
        model.to(device)
    batches_all = _calibration_batches(dataset, num_calibration_samples, calibration_batch_tokens, "cpu")
    if ws > 1:
        # contiguous share of the samples per rank
        samples = [(b["input_ids"][i], None if "attention_mask" not in b else b["attention_mask"][i])
                   for b in batches_all for i in range(b["input_ids"].shape[0])]
        s0, s1 = row_range(len(samples), rank, ws)
        mine = [{"input_ids": s[0]} if s[1] is None else {"input_ids": s[0], "attention_mask": s[1]}
                for s in samples[s0:s1]]
        batches = _calibration_batches(mine, len(mine), calibration_batch_tokens, device)
    else:
        batches = [{k: v.to(device) for k, v in b.items()} for b in batches_all]
    runner = SequentialRunner(model, mods, batches, device, sequential_targets, offload_layers,
                              moe_calibrate_all_experts, fused_forward)
    t0 = time.perf_counter()
    runner.capture()
    torch.cuda.synchronize(device)
    runner.stats.seconds["capture"] = time.perf_counter() - t0
    t0 = time.perf_counter()
    for li in range(len(runner.layers)):
        runner.run_layer(li)
    torch.cuda.synchronize(device)
    runner.stats.seconds["layers"] = time.perf_counter() - t0
    stats = runner.finish()
    if offload_layers:
        model.to("cpu")
    stats.seconds["total"] = time.perf_counter() - t_all
    globals()["LAST_STATS"] = stats
    return model


def _to_device_except(model: torch.nn.Module, skip_ids: set, device) -> None:
    """Move every parameter and buffer to ``device`` except those inside the
    modules in ``skip_ids`` (the decoder layers, moved one at a time)."""

    def visit(mod):
        if id(mod) in skip_ids:
            return
        for k, p in list(mod._parameters.items()):
            if p is not None and p.device != device:
                mod._parameters[k] = torch.nn.Parameter(p.data.to(device), requires_grad=p.requires_grad)
        for k, b in list(mod._buffers.items()):
            if b is not None and b.device != device:
                mod._buffers[k] = b.to(device)
        for c in mod.children():
            visit(c)

    visit(model)
