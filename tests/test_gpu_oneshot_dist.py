"""``oneshot`` GPTQ W4A16 on two GPUs (NCCL, one process per GPU) on the
2-layer Llama (config C1): every rank calibrates half of the samples,
Hessians are summed onto their owners, the owners broadcast the factors,
rows are split and the quantized rows all-gathered.  Checks: both ranks end
with identical weights; against the reference's own oneshot run
(``tests/golden/oneshot_c1.npz``), layer 0's q/k/v codes are >= 99% identical
and the quantized model's final hidden-state error is within 5% of the
reference's.  Round-to-nearest (``QuantizationModifier``) under DDP splits
the modules across the ranks and broadcasts their qparams: both ranks must
hold exactly the single-GPU qparams.  The 2-layer Qwen3-MoE (all-expert
calibration, experts' down projections owned by ranks and solved in
batches): both ranks end with identical weights and the final hidden-state
error within 5% of the reference's.  Needs two GPUs; skipped otherwise."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

QKV = ("model.layers.0.self_attn.q_proj", "model.layers.0.self_attn.k_proj", "model.layers.0.self_attn.v_proj")


def _port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from llmcompressor_b200 import oneshot as O
        from llmcompressor_b200 import synthetic

        model = synthetic.random_llama("c1").to(dev)
        ids = synthetic.calibration_tokens("c1")
        O.oneshot(model, ids, recipe=O.GPTQModifier(targets="Linear", scheme="W4A16", ignore=["lm_head"],
                                                     actorder=None), num_calibration_samples=len(ids))
        torch.cuda.synchronize()
        sums = torch.stack([m.weight.detach().double().sum() for n, m in sorted(model.named_modules())
                            if hasattr(m, "weight_scale")])
        lo, hi = sums.clone(), sums.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        out = {"same": bool(torch.equal(lo, hi))}
        if rank == 0:
            fp = synthetic.random_llama("c1").to(dev)
            with torch.no_grad():
                hq = model.model(ids[:4].to(dev)).last_hidden_state.float()
                hf = fp.model(ids[:4].to(dev)).last_hidden_state.float()
            out["hidden_rel_err"] = (torch.linalg.norm((hq - hf).reshape(4, -1), dim=1)
                                     / torch.linalg.norm(hf.reshape(4, -1), dim=1)).cpu().numpy()
            for n in QKV:
                m = model.get_submodule(n)
                s = m.weight_scale.detach()[:128].float().repeat_interleave(128, dim=1)
                out[n] = torch.round(m.weight.detach()[:128].float() / s).clamp(-8, 7).cpu().numpy().astype(np.int32)
        q.put((rank, "ok", out))
    except Exception as e:  # report, then leave between steps
        q.put((rank, f"error: {type(e).__name__}: {e}", None))
    finally:
        dist.destroy_process_group()


def _rtn_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from llmcompressor_b200 import oneshot as O
        from llmcompressor_b200 import synthetic

        model = synthetic.random_llama("c1").to(dev)
        O.oneshot(model, recipe=O.QuantizationModifier(targets="Linear", scheme="W4A16_ASYM", ignore=["lm_head"]))
        torch.cuda.synchronize()
        out = {n: (m.weight_scale.detach().cpu(), m.weight_zero_point.detach().cpu())
               for n, m in model.named_modules() if hasattr(m, "weight_scale")}
        q.put((rank, "ok", out))
    except Exception as e:
        q.put((rank, f"error: {type(e).__name__}: {e}", None))
    finally:
        dist.destroy_process_group()


def _moe_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        from llmcompressor_b200 import moe
        from llmcompressor_b200 import oneshot as O
        from llmcompressor_b200 import synthetic

        model = synthetic.random_qwen3_moe("c3tiny")
        moe.linearize_experts(model)
        model = model.to(dev)
        ids = synthetic.calibration_tokens("c3tiny")
        before = moe.STACKED_CALLS
        O.oneshot(model, ids, recipe=O.GPTQModifier(targets="Linear", scheme="W4A16",
                                                     ignore=["lm_head", "re:.*mlp.gate$"], actorder=None),
                  num_calibration_samples=len(ids))
        torch.cuda.synchronize()
        sums = torch.stack([m.weight.detach().double().sum() for n, m in sorted(model.named_modules())
                            if hasattr(m, "weight_scale")])
        lo, hi = sums.clone(), sums.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        out = {"same": bool(torch.equal(lo, hi)), "stacked": moe.STACKED_CALLS - before}
        if rank == 0:
            fp = synthetic.random_qwen3_moe("c3tiny").to(dev)
            with torch.no_grad():
                hq = model.model(ids[:4].to(dev)).last_hidden_state.float()
                hf = fp.model(ids[:4].to(dev)).last_hidden_state.float()
            out["hidden_rel_err"] = (torch.linalg.norm((hq - hf).reshape(4, -1), dim=1)
                                     / torch.linalg.norm(hf.reshape(4, -1), dim=1)).cpu().numpy()
        q.put((rank, "ok", out))
    except Exception as e:
        q.put((rank, f"error: {type(e).__name__}: {e}", None))
    finally:
        dist.destroy_process_group()


def _spawn(target, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, status, out = q.get(timeout=600)
        got[r] = (status, out)
    for p in procs:
        p.join(timeout=120)
    return got


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_rtn_matches_one_gpu():
    from llmcompressor_b200 import oneshot as O
    from llmcompressor_b200 import synthetic

    got = _spawn(_rtn_worker)
    assert all(v[0] == "ok" for v in got.values()), {r: v[0] for r, v in got.items()}
    model = synthetic.random_llama("c1").cuda()
    O.oneshot(model, recipe=O.QuantizationModifier(targets="Linear", scheme="W4A16_ASYM", ignore=["lm_head"]))
    ref = {n: (m.weight_scale.detach().cpu(), m.weight_zero_point.detach().cpu())
           for n, m in model.named_modules() if hasattr(m, "weight_scale")}
    for r in (0, 1):
        out = got[r][1]
        assert set(out) == set(ref)
        for n in ref:
            assert torch.equal(out[n][0], ref[n][0]) and torch.equal(out[n][1], ref[n][1]), (r, n)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_oneshot_c1():
    from golden_io import load
    from test_gpu_oneshot import unpack_int4

    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, status, out = q.get(timeout=600)
        got[r] = (status, out)
    for p in procs:
        p.join(timeout=120)
    assert all(v[0] == "ok" for v in got.values()), {r: v[0] for r, v in got.items()}
    assert got[0][1]["same"] and got[1][1]["same"]
    ref = load("oneshot_c1")
    out = got[0][1]
    for n in QKV:
        theirs = unpack_int4(ref[f"{n}.weight_packed"], out[n].shape[1])
        agree = float(np.mean(out[n] == theirs))
        assert agree >= 0.99, (n, agree)
    theirs = ref["hidden_rel_err"]
    assert np.all(np.abs(out["hidden_rel_err"] - theirs) <= 0.05 * theirs), (out["hidden_rel_err"], theirs)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_oneshot_moe():
    from golden_io import load

    got = _spawn(_moe_worker)
    assert all(v[0] == "ok" for v in got.values()), {r: v[0] for r, v in got.items()}
    assert got[0][1]["same"] and got[1][1]["same"]
    assert got[0][1]["stacked"] > 0
    theirs = load("oneshot_c3tiny")["hidden_rel_err"]
    ours = got[0][1]["hidden_rel_err"]
    assert np.all(np.abs(ours - theirs) <= 0.05 * theirs), (ours, theirs)
