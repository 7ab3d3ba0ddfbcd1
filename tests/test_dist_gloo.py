"""Host-side logic of the multi-GPU sharding, on CPU ranks over gloo
(world_size 2): ownership assignment, row slicing, reduce-to-owner,
inverse broadcast, row gather, and a rank that fails between steps."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llmcompressor_b200 import distributed as D


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(rank, world, port, fn, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=20))
    try:
        q.put((rank, fn(rank, world)))
    except Exception as e:  # report to the parent instead of hanging
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


def spawn(fn, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_run, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, v = q.get(timeout=120)
        out[r] = v
    for p in procs:
        p.join(timeout=60)
    return out


def test_greedy_owners_deterministic_and_balanced():
    costs = {"attn_in": D.solve_cost(4096, 6144), "o_in": D.solve_cost(4096, 4096),
             "mlp_in": D.solve_cost(4096, 28672), "down_in": D.solve_cost(14336, 4096)}
    a = D.greedy_owners(costs, 2)
    assert a == D.greedy_owners(dict(reversed(list(costs.items()))), 2)
    assert set(a.values()) == {0, 1}
    assert D.greedy_owners(costs, 1) == {k: 0 for k in costs}


@pytest.mark.parametrize("rows,world", [(4096, 8), (1024, 3), (7, 4), (0, 2), (14336, 2)])
def test_row_range_partitions_rows(rows, world):
    seen = []
    for r in range(world):
        r0, r1 = D.row_range(rows, r, world)
        assert 0 <= r0 <= r1 <= rows
        seen.extend(range(r0, r1))
    assert seen == list(range(rows))


def _collectives(rank, world):
    owners = {"a": 0, "b": 1}
    H = {"a": torch.full((4, 4), float(rank + 1)), "b": torch.full((3, 3), float(10 * (rank + 1)))}
    D.reduce_to_owners(H, owners)
    red_a = H["a"][0, 0].item() if rank == 0 else None
    red_b = H["b"][0, 0].item() if rank == 1 else None
    inv = {"a": [torch.full((2,), float(rank))], "b": [torch.full((2,), float(rank + 5))]}
    D.broadcast_inverse(inv, owners)
    rows = 5
    r0, r1 = D.row_range(rows, rank, world)
    local = torch.arange(r0, r1, dtype=torch.int32).reshape(-1, 1).repeat(1, 3)
    full = D.gather_rows(local, rows, dst=0)
    return {"red_a": red_a, "red_b": red_b, "inv_a": inv["a"][0].tolist(), "inv_b": inv["b"][0].tolist(),
            "gathered": None if full is None else full[:, 0].tolist()}


def test_reduce_broadcast_gather_over_gloo():
    out = spawn(_collectives)
    assert out[0]["red_a"] == 3.0  # 1 + 2 on owner 0
    assert out[1]["red_b"] == 30.0  # 10 + 20 on owner 1
    for r in (0, 1):
        assert out[r]["inv_a"] == [0.0, 0.0]  # from owner 0
        assert out[r]["inv_b"] == [6.0, 6.0]  # from owner 1
    assert out[0]["gathered"] == [0, 1, 2, 3, 4]
    assert out[1]["gathered"] is None


def _rank_fails(rank, world):
    """Rank 1 leaves between steps; rank 0's next collective ends with an
    error after the process-group timeout instead of hanging."""
    if rank == 1:
        raise RuntimeError("rank 1 stopped between steps")
    t = torch.ones(3)
    dist.all_reduce(t)
    return "no error"


def test_failed_rank_surfaces_as_error_not_hang():
    out = spawn(_rank_fails)
    assert "stopped between steps" in out[1]
    assert out[0] != "no error"


def _observer_sync(rank, world):
    """sync_activation_stats of the static observer (S/observers/base.py:146-165):
    MIN / MAX reductions of the rank-local statistics; the memoryless observer
    has nothing to sync."""
    from compressed_tensors.quantization import QuantizationArgs

    from llmcompressor_b200 import act_observers as ao

    args = QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="group", group_size=16, dynamic=False)
    obs = ao.StaticMinMaxObserver("input", args)
    obs.min_vals = torch.tensor([-1.0 - rank, -2.0 + rank, -0.5], dtype=torch.bfloat16)
    obs.max_vals = torch.tensor([1.0 + rank, 2.0 - rank, 0.25 * (rank + 1)], dtype=torch.bfloat16)
    for w in obs.sync_activation_stats():
        w.wait()
    mem = ao.MemorylessMinMaxObserver("input", args)
    mem.min_vals = torch.zeros(3, dtype=torch.bfloat16)
    mem.max_vals = torch.zeros(3, dtype=torch.bfloat16)
    assert mem.sync_activation_stats() == []
    return obs.min_vals.float().tolist(), obs.max_vals.float().tolist()


def test_activation_observer_stats_sync_over_ranks():
    got = spawn(_observer_sync)
    for r in range(2):
        mn, mx = got[r]
        assert mn == [-2.0, -2.0, -0.5], got
        assert mx == [2.0, 2.0, 0.5], got
