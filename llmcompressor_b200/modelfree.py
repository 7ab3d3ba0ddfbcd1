"""Model-free PTQ of safetensors checkpoints on the GPU.

The per-shard driver of the reference's model-free entry point:
``process_file`` (S/entrypoints/model_free/process.py:74-125),
``process_file_microscale_scheme`` (:128-236, the NVFP4 fused-set global
scales) and ``split_fused_moe_experts`` (:239-299).  Each quantizable tensor
goes through one fused kernel (observe -> qparams -> quantize -> pack,
``ops.modelfree_quantize``); an NVFP4 fused set (q/k/v, gate/up, w1/w3,
wq_a/wkv_a_with_mqa) shares one global scale from one absmax over its
members (``ops.fused_global_scale``).

Host side: tensors are read on the CPU by ``safetensors``, staged through
pinned buffers and copied to the device on a copy stream while the previous
tensor is being quantized; results are copied back into pinned buffers and
written with ``save_file``.  Across several ranks, whole files are assigned
to ranks by size (no collective on the data path).
"""
from __future__ import annotations

import os
import re
from collections.abc import Iterable

import torch

from . import ops

# S/entrypoints/model_free/microscale.py:51-60: families of fused weights,
# each a regex whose group `k` is the key shared by the members of one set.
_FUSED_FAMILIES = [
    re.compile(r"^(?P<k>.*(?:attn|attention))\.(?:q_proj|k_proj|v_proj)\.weight$"),
    re.compile(r"^(?P<k>.*(?:attn|attention))\.(?:wq_a|wkv_a_with_mqa)\.weight$"),
    re.compile(r"^(?P<k>.*mlp)\.(?:gate_proj|up_proj)\.weight$"),
    re.compile(r"^(?P<k>.*)w[13]\.weight$"),
]


def is_microscale_scheme(scheme) -> bool:
    """S/entrypoints/model_free/microscale.py:63-65."""
    s = scheme.weights.strategy
    return getattr(s, "value", s) == "tensor_group"


def fused_groups(names: Iterable[str]) -> list[list[str]]:
    """Sets of tensor names that share an NVFP4 global scale (present members only)."""
    names = list(names)
    groups: dict[tuple[int, str], list[str]] = {}
    for n in names:
        for fi, rx in enumerate(_FUSED_FAMILIES):
            m = rx.match(n)
            if m:
                groups.setdefault((fi, m.group("k")), []).append(n)
                break
    return [sorted(v) for v in groups.values()]


def split_fused_moe_experts(tensors: dict[str, torch.Tensor]) -> dict[str, torch.Tensor]:
    """3-D fused expert tensors -> per-expert 2-D tensors
    (S/entrypoints/model_free/process.py:239-299): ``gate_up_proj`` (E, 2I, H) ->
    ``{e}.gate_proj`` / ``{e}.up_proj``; ``down_proj`` (E, H, I) -> ``{e}.down_proj``."""
    split = {"gate_up_proj": ("gate_proj", "up_proj"), "down_proj": ("down_proj",)}
    out: dict[str, torch.Tensor] = {}
    for name, t in tensors.items():
        keys = [k for k in split if k in name]
        if len(keys) >= 2:
            raise ValueError(f"Found multiple keys matching {name}: {keys}")
        if len(keys) == 1 and t.ndim == 3:
            parts = split[keys[0]]
            if t.shape[1] % len(parts):
                raise ValueError(f"{keys[0]} expects a second dimension divisible by {len(parts)} "
                                 f"but got shape: {tuple(t.shape)}")
            inter = t.shape[1] // len(parts)
            for e in range(t.shape[0]):
                for pn, piece in zip(parts, t[e].split(inter, dim=0)):
                    key = name.replace(keys[0], f"{e}.{pn}")
                    if not key.endswith(".weight"):
                        key = f"{key}.weight"
                    out[key] = piece
        else:
            out[name] = t
    return out


def quantizable(tensors: dict[str, torch.Tensor], ignore: Iterable[str], targets: Iterable[str]):
    """(module_name, tensor_name) pairs the reference quantizes
    (compressed_tensors ``match_quantizable_tensors``)."""
    from compressed_tensors.utils import match_quantizable_tensors

    return list(match_quantizable_tensors(tensors, list(ignore), list(targets or ())))


def process_tensors(tensors: dict[str, torch.Tensor], scheme, ignore: Iterable[str] = (),
                    device: str | torch.device = "cuda") -> dict[str, torch.Tensor]:
    """Quantize and compress every quantizable tensor of one shard; returns the
    shard's new contents on the CPU (untouched tensors pass through)."""
    dev = torch.device(device)
    tensors = split_fused_moe_experts(dict(tensors))
    todo = quantizable(tensors, ignore, scheme.targets)
    for _, name in todo:
        t = tensors[name]
        if t.ndim != 2:
            raise ValueError(f"Unable to quantize tensor `{name}`: expected 2D linear weight, "
                             f"but got shape {tuple(t.shape)}")
        try:
            ops.stats_shape(t.shape[0], t.shape[1], scheme.weights)
        except Exception as exc:  # noqa: BLE001 -- re-raised with the tensor name, as the reference does
            raise ValueError(f"Unable to quantize tensor `{name}`: {exc}") from exc
    args = scheme.weights
    copy = torch.cuda.Stream(dev)
    comp = torch.cuda.current_stream(dev)

    def stage(name: str) -> tuple[torch.Tensor, torch.cuda.Event]:
        src = tensors[name]
        if src.dtype != torch.bfloat16:
            raise NotImplementedError(f"weights of dtype {src.dtype}: the kernels take bf16 weights")
        host = src if src.is_pinned() or src.is_cuda else src.contiguous().pin_memory()
        with torch.cuda.stream(copy):
            d = host.to(dev, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(copy)
        d.record_stream(comp)
        return d, ev

    gscale: dict[str, torch.Tensor] = {}
    names = [n for _, n in todo]
    cached: dict[str, tuple[torch.Tensor, torch.cuda.Event]] = {}
    if is_microscale_scheme(scheme):
        # NVFP4: one global scale per fused set from all its members, so the
        # whole shard is staged first (S/entrypoints/model_free/process.py:204-223)
        cached = {n: stage(n) for n in names}
        for _, ev in cached.values():
            comp.wait_event(ev)
        members = set()
        for grp in fused_groups(names):
            gs = ops.fused_global_scale([cached[n][0] for n in grp])
            for n in grp:
                gscale[n] = gs
                members.add(n)
        for n in names:
            if n not in members:
                gscale[n] = ops.fused_global_scale([cached[n][0]])

    def get(i: int):
        return cached.pop(names[i]) if names[i] in cached else stage(names[i])

    out = dict(tensors)
    pending = None
    nxt = get(0) if names else None
    for i, (module_name, name) in enumerate(todo):
        d, ev = nxt
        nxt = get(i + 1) if i + 1 < len(names) else None  # the next copy overlaps this tensor's kernel
        comp.wait_event(ev)
        res = ops.modelfree_quantize(d, args, gscale.get(name))
        host = {}
        for k, v in res.items():
            if v.is_cuda:
                h = torch.empty(v.shape, dtype=v.dtype, pin_memory=True)
                h.copy_(v, non_blocking=True)
                host[k] = h
            else:
                host[k] = v
        del out[name]
        for k, v in host.items():
            out[f"{module_name}.{k}"] = v
        pending = torch.cuda.Event()
        pending.record(comp)
    if pending is not None:
        pending.synchronize()
    return out


def process_file(path: str | os.PathLike, save_path: str | os.PathLike, scheme, ignore: Iterable[str] = (),
                 device: str | torch.device = "cuda") -> tuple[int, dict[str, str]]:
    """One safetensors shard in, one out (S/entrypoints/model_free/process.py:74-125);
    returns (total bytes, weight map) as the reference does."""
    from safetensors.torch import load_file, save_file

    tensors = load_file(str(path), device="cpu")
    out = process_tensors(tensors, scheme, ignore, device)
    os.makedirs(os.path.dirname(os.path.abspath(save_path)) or ".", exist_ok=True)
    save_file({k: v.contiguous() for k, v in out.items()}, str(save_path))
    total = sum(t.nbytes for t in out.values())
    return total, {k: os.path.basename(str(save_path)) for k in out}


def assign_files(sizes: dict[str, int], world_size: int) -> dict[str, int]:
    """Files to ranks, largest first onto the least-loaded rank."""
    load = [0] * max(1, world_size)
    owner: dict[str, int] = {}
    for f in sorted(sizes, key=lambda k: (-sizes[k], k)):
        r = min(range(len(load)), key=lambda i: (load[i], i))
        owner[f] = r
        load[r] += sizes[f]
    return owner


def process_files(files: list[str], save_dir: str, scheme, ignore: Iterable[str] = (),
                  device: str | torch.device | None = None) -> dict[str, str]:
    """Process several shards; with torch.distributed initialised each rank
    handles the files assigned to it and returns its part of the weight map."""
    import torch.distributed as dist

    rank, ws = (dist.get_rank(), dist.get_world_size()) if dist.is_available() and dist.is_initialized() else (0, 1)
    owners = assign_files({f: os.path.getsize(f) for f in files}, ws)
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    weight_map: dict[str, str] = {}
    for f in files:
        if owners[f] != rank:
            continue
        _, wm = process_file(f, os.path.join(save_dir, os.path.basename(f)), scheme, ignore, device)
        weight_map.update(wm)
    return weight_map
