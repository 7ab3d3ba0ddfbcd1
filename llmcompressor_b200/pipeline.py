"""Layer-level GPTQ on the GPU: the per-decoder-layer work of the reference's
sequential pipeline (S/pipelines/sequential/pipeline.py:136-178) restricted
to the hot path -- Hessian accumulation from the hooks, the solve at
``sequential_epoch_end`` (S/modifiers/gptq/base.py:239-321) and the
compressed-tensors pack done at save time
(S/transformers/compression/compressed_tensors_utils.py:172-191).

Differences in structure (not in results) from the reference:

* one Hessian per distinct Linear input (q/k/v share ``attn_in``, gate/up
  share ``mlp_in``) instead of one per module, fed with batches of
  calibration tokens instead of one hook call per sample;
* one factorisation per Hessian, shared by the modules that read it;
* with several ranks: tokens are split across ranks, Hessians are reduced to
  an owner, the owner broadcasts the inverse factor, and every rank solves an
  equal slice of every module's rows (see ``distributed``).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import _lib, gptq, ops
from .distributed import (
    broadcast_inverse,
    gather_rows,
    greedy_owners,
    reduce_to_owners,
    row_range,
    solve_cost,
    world,
)


@dataclass(frozen=True)
class LinearSpec:
    name: str
    out_features: int
    in_features: int
    input_key: str


@dataclass
class LayerResult:
    """Compressed-tensors state of one module (``pack-quantized``)."""

    weight_packed: torch.Tensor
    weight_scale: torch.Tensor
    loss: torch.Tensor  # float32 device scalar (this rank's share of rows)
    rows: tuple[int, int]
    weight_shape: tuple[int, int] = field(default=(0, 0))


def llama_layer_specs(hidden: int, intermediate: int, heads: int, kv_heads: int, head_dim: int) -> list[LinearSpec]:
    """The seven Linear modules of a Llama decoder layer and the input each reads."""
    return [
        LinearSpec("self_attn.q_proj", heads * head_dim, hidden, "attn_in"),
        LinearSpec("self_attn.k_proj", kv_heads * head_dim, hidden, "attn_in"),
        LinearSpec("self_attn.v_proj", kv_heads * head_dim, hidden, "attn_in"),
        LinearSpec("self_attn.o_proj", hidden, heads * head_dim, "o_in"),
        LinearSpec("mlp.gate_proj", intermediate, hidden, "mlp_in"),
        LinearSpec("mlp.up_proj", intermediate, hidden, "mlp_in"),
        LinearSpec("mlp.down_proj", hidden, intermediate, "down_in"),
    ]


def input_dims(specs: list[LinearSpec]) -> dict[str, int]:
    dims: dict[str, int] = {}
    for s in specs:
        dims.setdefault(s.input_key, s.in_features)
    return dims


class LayerHessians:
    """Float32 Hessian buffers, one per distinct input, reused across layers."""

    def __init__(self, dims: dict[str, int], device: torch.device):
        self.dims = dict(dims)
        self.H = {k: torch.zeros(d, d, dtype=torch.float32, device=device) for k, d in dims.items()}

    def reset(self) -> None:
        for h in self.H.values():
            h.zero_()

    def accumulate(self, key: str, x2d: torch.Tensor, alpha: float) -> None:
        """H[key] += alpha * x^T x (tensor cores); alpha = 2 / num_samples
        gives the reference's averaged Hessian H / num_samples directly."""
        gptq.hessian_update_(self.H[key], x2d, alpha)


def _fold_timeouts(statuses: list[torch.Tensor], err: torch.Tensor) -> None:
    """Raise the device error word to ETIMEOUT if any factor's status says a
    solve kernel timed out (an ENOT_PD fallback is not an error); queued on
    the current stream, no host sync.  ``_lib.check_device_errors`` reads it."""
    if not statuses:
        return
    s = torch.cat([t.reshape(1) for t in statuses])
    hit = torch.where(s == _lib.ETIMEOUT, s, torch.zeros_like(s)).amax().reshape(1)
    torch.maximum(err, hit, out=err)


_STREAMS: dict[int, list[torch.cuda.Stream]] = {}


def _side_streams(dev: torch.device, n: int) -> list[torch.cuda.Stream]:
    """n side streams of this device; the first has the highest priority the
    device offers (the layer's critical path runs there)."""
    idx = dev.index if dev.index is not None else torch.cuda.current_device()
    pool = _STREAMS.setdefault(idx, [])
    if not pool:
        lo, hi = torch.cuda.Stream.priority_range() if hasattr(torch.cuda.Stream, "priority_range") else (0, -1)
        pool.append(torch.cuda.Stream(device=dev, priority=min(lo, hi)))
    while len(pool) < n:
        pool.append(torch.cuda.Stream(device=dev))
    return pool[:n]


def solve_layer(
    weights: dict[str, torch.Tensor],
    specs: list[LinearSpec],
    hessians: LayerHessians,
    quant_args,
    percdamp: float = 0.01,
    blocksize: int = 128,
    gather_to: int | None = 0,
    pack_events: list | None = None,
) -> dict[str, LayerResult]:
    """GPTQ-quantize and pack every module of one layer from its (averaged)
    Hessians.  On several ranks each rank returns its row slice; with
    ``gather_to`` set, that rank also receives the full packed tensors.

    The independent pieces run concurrently on side streams: the
    factorisations of the distinct Hessians, and each module's block loop as
    soon as its factor is ready.  The caller's stream waits for all of them
    before this function returns, so results are ordered on it as usual.

    Nothing here synchronises the host: a kernel timeout (Hessian
    accumulation or solve) is left in the device error word, which the
    caller reads once, when it syncs anyway, with
    ``_lib.check_device_errors``."""
    rank, ws = world()
    dims = hessians.dims
    # activation ordering WEIGHT / STATIC permutes each Hessian's columns;
    # GROUP would also regroup the packed codes (g_idx), which this layer
    # API does not write
    act = gptq.resolve_actorder(getattr(quant_args, "actorder", None))
    if act == "group":
        raise NotImplementedError("activation ordering GROUP in the layer solve; use gptq.quantize_weight")
    rows_of: dict[str, int] = {}
    for s in specs:
        rows_of[s.input_key] = rows_of.get(s.input_key, 0) + s.out_features
    owners = greedy_owners({k: solve_cost(d, rows_of[k]) for k, d in dims.items()}, ws)
    reduce_to_owners(hessians.H, owners)
    dev = next(iter(hessians.H.values())).device
    main = torch.cuda.current_stream(dev)
    streams = _side_streams(dev, max(len(dims), len(specs)))

    # factorisations, largest first, one side stream each
    order = sorted(dims, key=lambda k: (-dims[k], k))
    inv: dict[str, gptq.InverseHessian] = {}
    ready: dict[str, torch.cuda.Event] = {}
    for i, key in enumerate(order):
        d = dims[key]
        st = streams[i]
        st.wait_stream(main)
        with torch.cuda.stream(st):
            if owners[key] == rank:
                inv[key] = gptq.inverse_hessian(hessians.H[key], percdamp, act)
            else:
                inv[key] = gptq.InverseHessian(
                    torch.empty(d, d, dtype=torch.float32, device=dev),
                    torch.empty(d, dtype=torch.uint8, device=dev),
                    torch.empty(1, dtype=torch.int32, device=dev),
                    torch.empty(d, d, dtype=torch.float32, device=dev),
                    torch.empty(d, dtype=torch.int32, device=dev) if act else None,
                )
            ev = torch.cuda.Event()
            ev.record(st)
            ready[key] = ev
    if ws > 1:
        for ev in ready.values():
            main.wait_event(ev)
        broadcast_inverse({k: [v.hinv, v.dead, v.status, v.hinv_t] + ([v.perm] if act else [])
                           for k, v in inv.items()}, owners)
        bcast = torch.cuda.Event()
        bcast.record(main)
        ready = {k: bcast for k in ready}

    # block loops + int4 pack, one side stream per module; the modules that
    # read the largest Hessian follow its factorisation on the high-priority
    # stream (the layer's critical path), the others spread over the rest
    crit = order[0]
    others = streams[1:] or streams
    parts: dict[str, tuple] = {}
    done = []
    for j, s in enumerate(specs):
        st = streams[0] if s.input_key == crit else others[j % len(others)]
        st.wait_event(ready[s.input_key])
        r0, r1 = row_range(s.out_features, rank, ws)
        with torch.cuda.stream(st):
            if r1 > r0:
                wl = weights[s.name][r0:r1]
                mn, mx = ops.observe_minmax(wl, quant_args)
                scale, zp = ops.calculate_qparams(mn, mx, quant_args)
                wq, loss = gptq.quantize_with_inverse(wl, quant_args, inv[s.input_key], scale, zp, blocksize, act)
                if pack_events is not None:
                    e0 = torch.cuda.Event(enable_timing=True)
                    e0.record(st)
                packed = ops.quantize_pack(wq, quant_args, scale, None if quant_args.symmetric else zp,
                                           fmt=_lib.FMT_PACK_INT32)
                if pack_events is not None:
                    e1 = torch.cuda.Event(enable_timing=True)
                    e1.record(st)
                    pack_events.append((e0, e1, wq.numel()))
            else:
                pf = 32 // quant_args.num_bits
                packed = torch.empty(0, -(-s.in_features // pf), dtype=torch.int32, device=dev)
                scale = torch.empty(0, ops.stats_shape(1, s.in_features, quant_args)[-1], dtype=torch.bfloat16,
                                    device=dev)
                loss = torch.zeros(1, dtype=torch.float32, device=dev)
            ev = torch.cuda.Event()
            ev.record(st)
            done.append(ev)
        for t in (packed, scale, loss):
            t.record_stream(main)
        parts[s.name] = (packed, scale, loss, (r0, r1))
    for ev in done:
        main.wait_event(ev)
    for v in inv.values():
        for t in (v.hinv, v.dead, v.status, v.hinv_t, v.perm):
            if t is not None:
                t.record_stream(main)
    _fold_timeouts([v.status for v in inv.values()], _lib.error_word(dev))

    out: dict[str, LayerResult] = {}
    for s in specs:
        packed, scale, loss, rr = parts[s.name]
        if ws > 1 and gather_to is not None:
            fp = gather_rows(packed, s.out_features, dst=gather_to)
            fs = gather_rows(scale, s.out_features, dst=gather_to)
            if rank == gather_to:
                packed, scale = fp, fs
        out[s.name] = LayerResult(packed, scale, loss, rr, (s.out_features, s.in_features))
    return out
