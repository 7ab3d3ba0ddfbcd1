"""Sharding of the GPTQ hot path across the GPUs of one node.

Reference behaviour (S/modifiers/gptq/base.py:291-321,603-645): every rank
accumulates Hessians over its slice of the calibration set, each Hessian is
``dist.reduce``d to an owner rank chosen by greedy bin packing, owners solve
their modules, and the fake-quantized bf16 weights are broadcast back.

Here the exchange is restructured around what GPTQ actually shares:

* Hessians: one per *distinct input* (q/k/v share one, gate/up share one),
  reduced to an owner (``reduce_to_owners``) -- the reference reduces one per
  module, duplicates included.
* The owner factors its Hessian once and broadcasts the inverse factor
  (``broadcast_inverse``); rows of a GPTQ weight are independent, so every
  rank then solves an equal slice of every module's rows (``row_range``),
  which balances the solve even when there are fewer distinct Hessians than
  ranks.
* Results travel as packed int4 codes + bf16 scales (0.52 B/weight instead
  of 2 B/weight) and are gathered to rank 0 for the compressed-tensors write
  (``gather_rows``).

Collectives are plain ``torch.distributed`` calls (NCCL on GPUs, gloo in the
CPU tests); every rank issues the same collectives in the same order.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def world() -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def greedy_owners(costs: dict[str, float], world_size: int) -> dict[str, int]:
    """Greedy bin packing by cost, largest first (the reference's
    ``greedy_bin_packing`` applied to solve cost instead of Hessian width).
    Ties break by name so every rank computes the same assignment."""
    load = [0.0] * world_size
    owners: dict[str, int] = {}
    for name in sorted(costs, key=lambda n: (-costs[n], n)):
        r = min(range(world_size), key=lambda i: (load[i], i))
        owners[name] = r
        load[r] += costs[name]
    return owners


def solve_cost(d: int, rows_total: int) -> float:
    """Relative GPTQ cost of one distinct Hessian: factorisation (~2/3 d^3)
    plus the rows' block loop and trailing update (~rows * d^2)."""
    return (2.0 / 3.0) * d**3 + rows_total * d**2


def row_range(rows: int, rank: int, world_size: int, align: int = 1) -> tuple[int, int]:
    """Contiguous slice of ``rows`` for ``rank`` (aligned to ``align`` rows)."""
    units = -(-rows // align)
    per = -(-units // world_size)
    r0 = min(rows, rank * per * align)
    r1 = min(rows, (rank + 1) * per * align)
    return r0, r1


@dataclass
class ShardPlan:
    owners: dict[str, int]
    rank: int
    world_size: int


def reduce_to_owners(hessians: dict[str, torch.Tensor], owners: dict[str, int]) -> None:
    """Sum each Hessian onto its owner rank (in place on the owner)."""
    _, ws = world()
    if ws == 1:
        return
    works = [dist.reduce(hessians[n], dst=owners[n], op=dist.ReduceOp.SUM, async_op=True) for n in sorted(hessians)]
    for w in works:
        w.wait()


def broadcast_inverse(tensors: dict[str, list[torch.Tensor]], owners: dict[str, int]) -> None:
    """Broadcast each owner's inverse factor (and companions) to every rank."""
    _, ws = world()
    if ws == 1:
        return
    works = []
    for n in sorted(tensors):
        for t in tensors[n]:
            works.append(dist.broadcast(t, src=owners[n], async_op=True))
    for w in works:
        w.wait()


def gather_rows(local: torch.Tensor, rows: int, dst: int = 0) -> torch.Tensor | None:
    """Gather row slices (``row_range`` layout) of a (rows, ...) tensor to ``dst``.
    Returns the assembled tensor on ``dst``, None elsewhere."""
    rank, ws = world()
    if ws == 1:
        return local
    per = -(-rows // ws)
    pad = torch.zeros((per,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    bufs = [torch.empty_like(pad) for _ in range(ws)] if rank == dst else None
    dist.gather(pad, bufs, dst=dst)
    if rank != dst:
        return None
    return torch.cat(bufs, dim=0)[:rows]


def all_gather_rows(local: torch.Tensor, out: torch.Tensor, rows: int, align: int = 1) -> torch.Tensor:
    """Every rank's ``row_range`` slice of a (rows, ...) tensor into ``out``
    on every rank (one padded ``all_gather_into_tensor``)."""
    _, ws = world()
    if ws == 1:
        out.copy_(local)
        return out
    units = -(-rows // align)
    per = -(-units // ws) * align
    pad = torch.zeros((per,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[: local.shape[0]] = local
    full = torch.empty((per * ws,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(full, pad)
    out.copy_(full[:rows])
    return out
