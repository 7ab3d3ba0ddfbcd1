#!/usr/bin/env python
"""Benchmark of oneshot GPTQ W4A16 g128 on a Llama-3-8B-shaped model.

Workload: 32 decoder layers (hidden 4096, intermediate 14336, 32 heads / 8 KV
heads, head_dim 128, vocab 128256), random bf16 weights ~N(0, 0.02) drawn on
the GPU, 512 calibration sequences x 2048 uniformly random tokens (seeded:
there are no checkpoints or datasets on the box).  The pipeline is
``llmcompressor_b200.oneshot``'s sequential runner, the code path
``oneshot(model, tokens, recipe=GPTQModifier(scheme="W4A16",
ignore=["lm_head"], actorder=None))`` executes.  One step = one decoder
layer: the calibration forward over all tokens with the Hessian hooks
(q/k/v, o, gate/up and down inputs), the GPTQ solve of the layer's seven
Linear weights, and the propagation forward through the quantized layer.

``value`` = oneshot wall seconds for the whole model = capture (embedding to
the first layer) + 32 x the mean timed layer step, device-resident model and
tokens, CUDA events between barriers, max over ranks.  ``e2e`` = the same
steps with every layer's weights copied in from pinned host memory before
it is processed and the quantized layer copied back after (the oneshot call
on a model that lives on the host).

``--impl reference`` times the CPU path on the host cores (a numpy
restatement of the reference's GPTQ arithmetic plus the model's torch
forward) on a bounded sample and extrapolates to the model.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "oneshot GPTQ W4A16 wall-s (Llama-3-8B shape); Hessian TFLOP/s; cast GB/s"
CFG = dict(layers=32, hidden=4096, intermediate=14336, heads=32, kv_heads=8, head_dim=128, samples=512, seq=2048)
CHUNK = 16384  # calibration tokens per forward batch and Hessian launch (8 sequences)


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16": d["bf16_tflops"], "bf16_sustained": d.get("bf16_tflops_sustained",
                                                                                          d["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16": 1590.0, "bf16_sustained": 1400.0, "source": "fallback"}


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, path: str):
        self.path = path
        self.proc = None

    def start(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self, gpu_index: int = 0) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.f.close()
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9 or not parts[0].isdigit() or int(parts[0]) != gpu_index:
                continue
            try:
                sm.append(float(parts[1]))
                mx = max(mx, float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- workload
def w4a16_args():
    from compressed_tensors.quantization import QuantizationArgs

    return QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128, actorder=None)


# DRAM bytes per k_hessian_pair launch measured by ncu (dram__bytes_read.sum +
# dram__bytes_write.sum) at the bench's batch size, and the algorithmic bytes
# (X once + the lower triangle of H read and written):
# profiles/k_hessian_pair__d4096_n16384.md, profiles/k_hessian_pair__d14336_n16384_traffic.md
HESSIAN_TRAFFIC = {4096: 267.5e6 + 39.8e6, 14336: 4865.2e6 + 805.8e6}


def hessian_algorithmic_bytes(d: int, tokens: int = CHUNK) -> float:
    return tokens * d * 2 + 2 * (d * (d + 1) // 2) * 4


def hessian_flops(dims, tokens):
    return sum(tokens * d * (d + 1) for d in dims.values())


# ----------------------------------------------------------------------------- our arm
def build_runner(args, rank, world, device, on_host: bool = False):
    """The C2 model, this rank's calibration tokens and the oneshot runner."""
    from llmcompressor_b200 import oneshot as O
    from llmcompressor_b200 import synthetic
    from llmcompressor_b200.distributed import row_range

    layers = args.layers or CFG["layers"]
    model = synthetic.random_llama("llama3_8b", device=device, init_device=device, num_hidden_layers=layers)
    ids = synthetic.calibration_tokens("llama3_8b", n=args.samples or CFG["samples"], seq_len=CFG["seq"])
    s0, s1 = row_range(ids.shape[0], rank, world)
    batches = O._calibration_batches(ids[s0:s1], s1 - s0, CHUNK, device)
    if on_host:
        # the layers live in pinned host memory; everything else stays on the device
        for layer in O.sequential_layers(model):
            for p in layer.parameters():
                p.data = p.data.cpu().pin_memory()
    mod = O.GPTQModifier(targets="Linear", scheme="W4A16", ignore=["lm_head"], actorder=None, block_size=128,
                         dampening_frac=0.01)
    runner = O.SequentialRunner(model, [mod], batches, device, offload_layers=on_host, fused_forward=args.fused)
    return model, runner


def _barrier(world):
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()


def _max_over_ranks(ms, world, device):
    t = torch.tensor([ms], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_ours(args, rank, world, device):
    from llmcompressor_b200 import _lib, gptq

    torch.cuda.set_device(device)
    pk = peaks()
    model, runner = build_runner(args, rank, world, device)
    L = len(runner.layers)
    _barrier(world)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record()
    runner.capture()
    c1.record()
    _barrier(world)
    capture_ms = _max_over_ranks(c0.elapsed_time(c1), world, device)
    # every step runs a layer with its propagation pass (layers 0 .. L-2, cycling)
    order = [i % max(1, L - 1) for i in range(args.warmup + args.steps)]
    for i in range(args.warmup):
        runner.run_layer(order[i], propagate=True)
    _barrier(world)
    clock_dir = tempfile.gettempdir()
    clocks = ClockSampler(os.path.join(clock_dir, f"clocks_rank{rank}.csv")) if rank == 0 else None
    if clocks:
        clocks.start()
    launches0 = _lib.kernel_launches()
    gptq.TIMING_EVENTS = []
    phases = []
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.warmup, args.warmup + args.steps):
        runner.run_layer(order[i], phases=phases, propagate=True)
    t1.record()
    _barrier(world)
    launches = _lib.kernel_launches() - launches0
    clk = clocks.stop(torch.cuda.current_device()) if clocks else None
    ms = _max_over_ranks(t0.elapsed_time(t1), world, device)
    hev = gptq.TIMING_EVENTS
    gptq.TIMING_EVENTS = None
    h_ms = sum(a.elapsed_time(b) for a, b, _ in hev)
    h_flops = sum(f for _, _, f in hev)
    # per-phase split of the timed steps (this rank)
    split = {}
    prev = None
    for name, ev in phases:
        if name != "start" and prev is not None:
            split[name] = split.get(name, 0.0) + prev.elapsed_time(ev)
        prev = ev
    split = {k: v / args.steps for k, v in split.items()}
    stats = runner.finish()
    casts = None
    mfree = None
    if rank == 0 and args.casts:
        from llmcompressor_b200 import oneshot as O

        lw = [{n: m.weight.data for n, m in l.named_modules() if isinstance(m, torch.nn.Linear)}
              for l in O.sequential_layers(model)[:4]]
        casts = measure_casts(lw)
    del model, runner
    torch.cuda.empty_cache()
    if rank == 0 and args.casts:
        mfree = modelfree_layers(device)
    out = {
        "ms": ms, "capture_ms": capture_ms, "layers": L, "launches": launches, "clocks": clk,
        "hessian_tflops": h_flops / (h_ms * 1e-3) / 1e12 if h_ms > 0 else None,
        "hessian_ms_per_step": h_ms / args.steps, "hessian_launches_per_step": len(hev) / args.steps,
        "hessian_flops_per_launch": h_flops / max(1, len(hev)),
        "phases_ms_per_step": split, "casts": casts, "modelfree": mfree, "peaks": pk,
        "loss_layers": len(stats.losses),
    }
    if args.e2e:
        out["e2e"] = run_e2e(args, rank, world, device)
    if args.c3:
        out["c3"] = run_c3(args, rank, world, device)
    return out


def run_e2e(args, rank, world, device):
    """The same steps with the layers in pinned host memory: each step copies
    the layer's weights in, runs it, and copies the quantized weights back;
    the step ends with the layer's summed GPTQ loss read on the host."""
    model, runner = build_runner(args, rank, world, device, on_host=True)
    L = len(runner.layers)
    layer_bytes = sum(p.numel() * p.element_size() for p in runner.layers[0].parameters())
    runner.capture()
    order = [i % max(1, L - 1) for i in range(args.warmup + args.steps)]

    def step(i):
        runner.run_layer(order[i], propagate=True)
        losses = [v[0] for k, v in runner.stats.losses.items() if isinstance(v, tuple)]
        return float(torch.stack([x.reshape(()) for x in losses[-7:]]).sum().item()) if losses else 0.0

    for i in range(args.warmup):
        step(i)
    _barrier(world)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.warmup, args.warmup + args.steps):
        step(i)
    t1.record()
    _barrier(world)
    ms = _max_over_ranks(t0.elapsed_time(t1), world, device)
    runner.finish()
    del model, runner
    torch.cuda.empty_cache()
    return {"ms": ms, "h2d_per_step": layer_bytes, "d2h_per_step": layer_bytes + 4 * 7, "layers": L}


C3 = dict(layers=48, samples=256, seq=2048)


def run_c3(args, rank, world, device):
    """Config C3: oneshot GPTQ W4A16 with all-expert calibration on the
    Qwen3-30B-A3B shape (128 experts top-8; every expert sees every token in
    the calibration pass), 256 x 2048 tokens.  The model is built with the
    layers the steps run (all 48 have the same shape); value = capture +
    48 x mean timed layer step."""
    from llmcompressor_b200 import _lib
    from llmcompressor_b200 import oneshot as O
    from llmcompressor_b200 import synthetic
    from llmcompressor_b200.distributed import row_range

    n_layers = min(C3["layers"], args.c3_warmup + args.c3_steps + 1)
    model = synthetic.random_qwen3_moe("qwen3_30b_a3b", device=device, init_device=device,
                                       num_hidden_layers=n_layers)
    ids = synthetic.calibration_tokens("qwen3_30b_a3b", n=C3["samples"], seq_len=C3["seq"])
    s0, s1 = row_range(ids.shape[0], rank, world)
    batches = O._calibration_batches(ids[s0:s1], s1 - s0, CHUNK, device)
    mod = O.GPTQModifier(targets="Linear", scheme="W4A16", ignore=["lm_head", "re:.*mlp.gate$"], actorder=None)
    runner = O.SequentialRunner(model, [mod], batches, device, fused_forward=args.fused)
    _barrier(world)
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c0.record()
    runner.capture()
    c1.record()
    for i in range(args.c3_warmup):
        runner.run_layer(i, propagate=True)
    _barrier(world)
    launches0 = _lib.kernel_launches()
    phases = []
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.c3_warmup, args.c3_warmup + args.c3_steps):
        runner.run_layer(i, phases=phases, propagate=True)
    t1.record()
    _barrier(world)
    ms = _max_over_ranks(t0.elapsed_time(t1), world, device)
    cap_ms = _max_over_ranks(c0.elapsed_time(c1), world, device)
    split, prev = {}, None
    for name, ev in phases:
        if name != "start" and prev is not None:
            split[name] = split.get(name, 0.0) + prev.elapsed_time(ev)
        prev = ev
    runner.finish()
    launches = _lib.kernel_launches() - launches0
    del model, runner
    torch.cuda.empty_cache()
    return {"value": (cap_ms + ms * C3["layers"] / args.c3_steps) * 1e-3, "unit": "s",
            "ms_per_step": ms / args.c3_steps, "steps": args.c3_steps, "warmup": args.c3_warmup,
            "phases_ms_per_step": {k: v / args.c3_steps for k, v in split.items()}, "gpu_launches": launches,
            "workload": "C3: oneshot GPTQ W4A16 g128, all-expert calibration, Qwen3-30B-A3B shape "
                        "(48 layers, 128 experts top-8), 256x2048 tokens; value = capture + 48 x mean layer step"}


CAST_SCHEMES = ("W4A16", "NVFP4A16", "MXFP4A16", "FP8_BLOCK", "FP8_DYNAMIC")


def measure_casts(layers, reps: int = 3) -> dict:
    """Model-free single-pass casts (observe + qparams + quantize + pack) over
    the Linear weights of a few layers (436 MB of bf16 per layer, so every
    launch streams from HBM), one format at a time, timed with CUDA events:
    one launch per tensor (``gbs``) and the batched launch over the same
    tensors (``batched_gbs``, as a shard is processed).  Bytes = bf16 weight
    read + codes and scales written."""
    from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme

    from llmcompressor_b200 import ops

    res = {}
    for name in CAST_SCHEMES:
        qa = preset_name_to_scheme(name, ["Linear"]).weights
        ws = [w for layer in layers for w in layer.values()]
        gss = [ops.fused_global_scale([w]) if name == "NVFP4A16" else None for w in ws]
        out_bytes = 0
        for w, gs in zip(ws, gss):
            o = ops.modelfree_quantize(w, qa, gs)
            out_bytes += sum(t.numel() * t.element_size() for k, t in o.items() if t.is_cuda and k != "weight_global_scale")
        in_bytes = sum(w.numel() * 2 for w in ws)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            for w, gs in zip(ws, gss):
                ops.modelfree_quantize(w, qa, gs)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        batch = ops.ModelfreeBatch(ws, qa, gss)
        batch.run()
        e0.record()
        for _ in range(reps):
            batch.run()
        e1.record()
        torch.cuda.synchronize()
        ms_b = e0.elapsed_time(e1) / reps
        res[name] = {"gbs": (in_bytes + out_bytes) / (ms * 1e-3) / 1e9, "ms": ms, "bytes": in_bytes + out_bytes,
                     "launches_per_pass": len(ws), "batched_gbs": (in_bytes + out_bytes) / (ms_b * 1e-3) / 1e9}
    return res


def modelfree_layers(device, reps: int = 10) -> dict:
    """Device-resident model-free passes at the C4 / C5 benchmark shapes, one
    layer (or expert sample) each, timed with CUDA events:

    * C4: one Llama-3-70B-shaped layer (q/k/v/o 8192-wide, gate/up/down 28672),
      ~N(0, 0.02) with 0.1% of values x50, NVFP4A16 with fused q/k/v and
      gate/up global scales: absmax pass + quantize/pack pass, 4.5625 B per
      weight (2 B absmax read + 2.5625 B quantize pass).
    * C5: DeepSeek-V3-shaped MoE expert matrices (32 experts x gate/up/down,
      7168 x 2048), rows 0.02 * Student-t(4), FP8_BLOCK (3.0001 B/weight) and
      MXFP4A16 (2.53125 B/weight), single pass, the expert set through the
      batched launch (48 tensors per launch)."""
    from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme

    from llmcompressor_b200 import ops

    g = torch.Generator(device=device).manual_seed(3)

    def normal_outliers(r, c):
        w = 0.02 * torch.randn(r, c, device=device, generator=g)
        m = torch.rand(r, c, device=device, generator=g) < 0.001
        return torch.where(m, w * 50, w).to(torch.bfloat16)

    def student_t(r, c):
        z = torch.randn(r, c, device=device, generator=g)
        chi = torch.distributions.Chi2(torch.tensor(4.0, device=device)).sample((r, 1))
        return (0.02 * z / torch.sqrt(chi / 4.0)).to(torch.bfloat16)

    out = {}
    h, inter = 8192, 28672
    c4 = {"q": normal_outliers(h, h), "k": normal_outliers(1024, h), "v": normal_outliers(1024, h),
          "o": normal_outliers(h, h), "gate": normal_outliers(inter, h), "up": normal_outliers(inter, h),
          "down": normal_outliers(h, inter)}
    nv = preset_name_to_scheme("NVFP4A16", ["Linear"]).weights
    sets = [["q", "k", "v"], ["o"], ["gate", "up"], ["down"]]

    def c4_pass():
        for st in sets:
            gs = ops.fused_global_scale([c4[n] for n in st])
            for n in st:
                ops.modelfree_quantize(c4[n], nv, gs)

    nweights = sum(w.numel() for w in c4.values())
    c4_pass()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        c4_pass()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    out["C4_llama70b_layer_NVFP4A16"] = {"weights": nweights, "ms": ms,
                                         "gbs": nweights * 4.5625 / (ms * 1e-3) / 1e9,
                                         "bytes_per_weight": 4.5625}
    del c4
    experts = [student_t(2048, 7168) for _ in range(64)] + [student_t(7168, 2048) for _ in range(32)]
    for name, bpw in (("FP8_BLOCK", 3.0001), ("MXFP4A16", 2.53125)):
        a = preset_name_to_scheme(name, ["Linear"]).weights
        batch = ops.ModelfreeBatch(experts, a)
        batch.run()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(reps):
            batch.run()  # the expert set in batched launches
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        n = sum(w.numel() for w in experts)
        out[f"C5_dsv3_32experts_{name}"] = {"weights": n, "ms": ms, "gbs": n * bpw / (ms * 1e-3) / 1e9,
                                            "bytes_per_weight": bpw}
    return out


# ----------------------------------------------------------------------------- CPU oracle arm
def cpu_sample(steps: int, warmup: int) -> dict:
    """Time the CPU oracle (numpy restatement of the reference's torch path)
    on bounded samples and extrapolate to the model with the reference's own
    work counts per layer: 7 Hessians (q/k/v/o/gate/up at d = 4096, down at
    14336; the reference keeps one per module) and 7 factorisations.
    Samples: Hessian of one 2048-token sequence at d = 4096 (every step) and
    d = 14336 (once); inverse factor at d = 4096 (once, d^3-scaled to 14336);
    block loop at 4096 columns on 64 and 512 rows (every step), fitted as
    a + b * rows and scaled to 14336 columns (a by c, b by c^2)."""
    from oracle import gptq as og
    from oracle.observers import QArgs

    cores = len(os.sched_getaffinity(0))
    rng = np.random.default_rng(0)
    qa = QArgs(4, "int", True, "group", 128)
    d1, d2 = CFG["hidden"], CFG["intermediate"]

    def t_hess(d):
        # H persists across the 512 calls of a layer: time a call on a
        # resident (already touched) H, as every call after the first is.
        x = rng.standard_normal((CFG["seq"], d), dtype=np.float32)
        H = np.full((d, d), 0.0, np.float32)
        og.accumulate_hessian(x[:64], H, 0)
        t = time.perf_counter()
        og.accumulate_hessian(x, H, 0)
        return time.perf_counter() - t

    def t_forward():
        # one 2048-token sequence through one decoder layer in bf16 on the host
        # cores (the reference's sequential pipeline runs every sample through
        # every layer twice: calibration and propagation)
        from transformers.models.llama.modeling_llama import LlamaDecoderLayer, LlamaRotaryEmbedding

        from llmcompressor_b200 import synthetic

        torch.set_num_threads(cores)
        cfg = synthetic.llama_config("llama3_8b")
        with torch.no_grad():
            layer = LlamaDecoderLayer(cfg, 0).to(torch.bfloat16)
            rot = LlamaRotaryEmbedding(cfg)
            xs = torch.randn(1, CFG["seq"], d1, dtype=torch.bfloat16)
            pos = torch.arange(CFG["seq"])[None]
            pe = rot(xs, pos)
            layer(xs, position_embeddings=pe, position_ids=pos)
            t = time.perf_counter()
            layer(xs, position_embeddings=pe, position_ids=pos)
            return time.perf_counter() - t

    t_fwd = t_forward()
    x = rng.standard_normal((4096, d1), dtype=np.float32)
    H = (x.T @ x) / 4096
    t = time.perf_counter()
    U, _ = og.hinv_upper(H, 0.01)
    t_inv = time.perf_counter() - t
    t_h14336 = t_hess(d2)
    w64 = (0.02 * rng.standard_normal((64, d1))).astype(np.float32)
    w512 = (0.02 * rng.standard_normal((512, d1))).astype(np.float32)
    h4096, a_fit, b_fit = [], [], []
    for i in range(warmup + steps):
        th = t_hess(d1)
        t = time.perf_counter()
        og.quantize_weight(w64, H, qa, hinv=U)
        t64 = time.perf_counter() - t
        t = time.perf_counter()
        og.quantize_weight(w512, H, qa, hinv=U)
        t512 = time.perf_counter() - t
        if i >= warmup:
            h4096.append(th)
            b = max((t512 - t64) / (512 - 64), 0.0)
            b_fit.append(b)
            a_fit.append(max(t64 - 64 * b, 0.0))
    th4096, a, b = statistics.median(h4096), statistics.median(a_fit), statistics.median(b_fit)
    s = CFG["samples"]
    rows4096 = [CFG["heads"] * CFG["head_dim"], CFG["kv_heads"] * CFG["head_dim"], CFG["kv_heads"] * CFG["head_dim"],
                CFG["hidden"], d2, d2]
    r = d2 / d1
    per_layer = (s * (6 * th4096 + t_h14336) + 6 * t_inv + t_inv * r**3
                 + sum(a + b * n for n in rows4096) + (a * r + b * r * r * d1)
                 + 2 * s * t_fwd)
    return {
        "value": per_layer * CFG["layers"],
        "unit": "s",
        "cores": cores,
        "kind": "port",
        "sample": (f"extrapolated to 32 layers x 7 modules from timings on {cores} host threads: two bf16 torch "
                   f"forward passes of every 2048-token sequence through a decoder layer (one timed); numpy-oracle "
                   f"Hessian of one 2048-token sequence at d=4096 (median of {steps}) and d=14336; inverse "
                   f"factor at d=4096 (x(14336/4096)^3 for 14336); block loop at 4096 columns on 64 and 512 rows "
                   f"(fit a + b*rows, scaled by c and c^2 to 14336 columns); reference work counts "
                   f"(7 Hessians, 7 factorisations per layer)"),
        "parts_s": {"forward_per_seq_layer": t_fwd, "hess4096_per_seq": th4096, "hess14336_per_seq": t_h14336,
                    "inv4096": t_inv,
                    "loop_a": a, "loop_b_per_row": b},
    }


def run_micro(args) -> None:
    """One kernel on a small case (profiling captures and per-kernel timing):
    hessian: H += alpha X^T X, X (tokens x d); gptq: factor + block loop of
    one (rows x d) weight; cast: model-free pass of --scheme over a (rows x d) weight;
    castbatch: --tensors such weights through the batched launch; hessianhook:
    --tokens in 2048-token calls through gptq.BatchedHessian; actobs: one
    activation-observer update (NVFP4 input statistics) over (tokens x d) bf16."""
    from llmcompressor_b200 import gptq, ops

    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(0)
    d, n, rows = args.d, args.tokens, args.rows
    qa = w4a16_args()
    if args.micro == "hessian":
        x = torch.randn(n, d, device=dev, generator=g).to(torch.bfloat16)
        H = torch.zeros(d, d, device=dev)
        fn = lambda: gptq.hessian_update_(H, x, 2.0 / n, fold_tokens=args.fold)  # noqa: E731
        work, unit = n * d * (d + 1) / 1e12, "TFLOP/s"
    elif args.micro in ("gptq", "hinv"):
        w = (0.02 * torch.randn(rows, d, device=dev, generator=g)).to(torch.bfloat16)
        x = torch.randn(4096, d, device=dev, generator=g).to(torch.bfloat16)
        H0 = torch.zeros(d, d, device=dev)
        gptq.hessian_update_(H0, x, 2.0 / 4096)
        mn, mx = ops.observe_minmax(w, qa)
        scale, zp = ops.calculate_qparams(mn, mx, qa)

        def fn():
            inv = gptq.inverse_hessian(H0.clone(), 0.01)
            if args.micro == "hinv":
                return inv
            return gptq.quantize_with_inverse(w, qa, inv, scale, zp)

        work, unit = None, "ms"
    elif args.micro == "hessianhook":
        # --tokens of calibration in calls of 2048 tokens (one sample each), as the
        # reference's forward hook delivers them, through gptq.BatchedHessian
        calls = max(1, n // 2048)
        xs = [torch.randn(1, 2048, d, device=dev, generator=g).to(torch.bfloat16) for _ in range(calls)]

        def fn():
            bh = gptq.BatchedHessian(d, dev)
            for x in xs:
                bh.add(x)
            return bh.finalize()

        work, unit = calls * 2048 * d * (d + 1) / 1e12, "TFLOP/s"
    elif args.micro == "actobs":
        from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme

        from llmcompressor_b200 import act_observers

        # NVFP4 input activations: per-16 statistics over all tokens, moving average
        aargs = preset_name_to_scheme("NVFP4", ["Linear"]).input_activations
        obs = act_observers.MinMaxObserver("input", aargs)
        x = torch.randn(n, d, device=dev, generator=g).to(torch.bfloat16)
        fn = lambda: obs(x)  # noqa: E731
        work, unit = x.numel() * 2 / 1e9, "GB/s"
    elif args.micro == "castbatch":
        from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme

        qa = preset_name_to_scheme(args.scheme, ["Linear"]).weights
        ws = [(0.02 * torch.randn(rows, d, device=dev, generator=g)).to(torch.bfloat16) for _ in range(args.tensors)]
        gss = [ops.fused_global_scale([w]) for w in ws] if args.scheme == "NVFP4A16" else None
        batch = ops.ModelfreeBatch(ws, qa, gss)
        outs = batch.run().results
        nbytes = sum(w.numel() * 2 for w in ws) + sum(t.numel() * t.element_size() for o in outs
                                                      for k, t in o.items() if t.is_cuda and k != "weight_global_scale")
        fn = batch.run
        work, unit = nbytes / 1e9, "GB/s"
    else:
        from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme

        qa = preset_name_to_scheme(args.scheme, ["Linear"]).weights
        w = (0.02 * torch.randn(rows, d, device=dev, generator=g)).to(torch.bfloat16)
        gs = ops.fused_global_scale([w]) if args.scheme == "NVFP4A16" else None
        o = ops.modelfree_quantize(w, qa, gs)
        nbytes = w.numel() * 2 + sum(t.numel() * t.element_size() for k, t in o.items()
                                     if t.is_cuda and k != "weight_global_scale")
        fn = lambda: ops.modelfree_quantize(w, qa, gs)  # noqa: E731
        work, unit = nbytes / 1e9, "GB/s"
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    rate = (work / (ms * 1e-3)) if work is not None else ms
    print(json.dumps({"micro": args.micro, "d": d, "tokens": n, "rows": rows, "ms_per_call": ms, unit: rate}),
          flush=True)


def _layer_hessian_dims():
    return [CFG["hidden"]] * 3 + [CFG["intermediate"]]


def traffic_per_launch() -> float | None:
    ds = _layer_hessian_dims()
    if any(HESSIAN_TRAFFIC[d] is None for d in ds):
        return None
    return sum(HESSIAN_TRAFFIC[d] for d in ds) / len(ds)


def algorithmic_per_launch() -> float:
    ds = _layer_hessian_dims()
    return sum(hessian_algorithmic_bytes(d) for d in ds) / len(ds)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--micro", choices=["hessian", "hessianhook", "gptq", "hinv", "cast", "castbatch", "actobs"], default=None,
                    help="time one kernel on a small case instead of the model benchmark")
    ap.add_argument("--d", type=int, default=4096)
    ap.add_argument("--fold", type=int, default=0, help="--micro hessian: tokens per tensor-core partial (0: default)")
    ap.add_argument("--tokens", type=int, default=16384)
    ap.add_argument("--rows", type=int, default=4096)
    ap.add_argument("--scheme", default="W4A16", choices=list(CAST_SCHEMES), help="format of --micro cast")
    ap.add_argument("--tensors", type=int, default=32, help="tensors of --micro castbatch")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--layers", type=int, default=0, help="decoder layers in the model (0: 32)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", dest="e2e", action="store_false")
    ap.add_argument("--no-c3", dest="c3", action="store_false", help="skip the MoE (Qwen3-30B-A3B shape) leg")
    ap.add_argument("--no-casts", dest="casts", action="store_false", help="skip the cast and model-free legs")
    ap.add_argument("--c3-steps", type=int, default=2)
    ap.add_argument("--c3-warmup", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", dest="cpu_baseline", action="store_false")
    ap.add_argument("--samples", type=int, default=0,
                    help="calibration samples of the C2 leg (0: 512); fewer only for profiling captures -- "
                         "a value with fewer samples is not the benchmark's")
    ap.add_argument("--eager-forward", dest="fused", action="store_false",
                    help="run the decoder layers' HF forwards as they are (no fused elementwise kernels)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.micro:
        run_micro(args)
        return

    if args.impl == "reference":
        if rank != 0:
            return
        ref_steps = max(1, min(args.steps, 8))
        cb = cpu_sample(ref_steps, min(args.warmup, 1))
        line = {
            "metric": METRIC, "value": cb["value"], "unit": "s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": cb["value"] * 1e3 / CFG["layers"], "higher_is_better": False,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "parts_s": cb["parts_s"],
            "config": {"workload": "C2: oneshot GPTQ W4A16 g128 (actorder off, damp 0.01), Llama-3-8B shape, "
                                   "512x2048 calibration tokens, sequential pipeline incl. decoder forward passes",
                       "parallelism": "host cores"},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return

    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"),
                                timeout=__import__("datetime").timedelta(seconds=600))
    device = torch.device(f"cuda:{local}")
    res = run_ours(args, rank, world, device)
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    pk = res["peaks"]
    L = res["layers"]
    model_s = (res["capture_ms"] + res["ms"] * L / args.steps) * 1e-3
    h_peak = pk["bf16_sustained"]
    line = {
        "metric": METRIC,
        "value": model_s,
        "unit": "s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": res["ms"] / args.steps,
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded random weights and uniform random token ids)",
        "config": {
            "workload": "C2: oneshot GPTQ W4A16 g128 (actorder off, damp 0.01), Llama-3-8B shape, "
                        f"{args.samples or CFG['samples']}x2048 calibration tokens, sequential pipeline incl. "
                        "decoder forward passes",
            "layers_in_model": L, "layers_timed": args.steps, "hidden": CFG["hidden"],
            "intermediate": CFG["intermediate"], "calibration_tokens": (args.samples or CFG["samples"]) * CFG["seq"],
            "forward_batch_tokens": CHUNK,
            "value_formula": "capture + layers x mean timed layer step",
            "capture_s": res["capture_ms"] * 1e-3,
            "phases_ms_per_step_rank0": res["phases_ms_per_step"],
            "l2": "inputs larger than L2 (every calibration batch is 134 MB of hidden states)",
            "parallelism": f"calibration samples dp{world} + GPTQ weight rows dp{world}",
        },
        "roofline": {
            "kernel": "k_hessian_pair",
            "bound": "tensor",
            "achieved": res["hessian_tflops"],
            "peak": h_peak,
            "unit": "TFLOP/s",
            "frac": res["hessian_tflops"] / h_peak if res["hessian_tflops"] else None,
            "peak_source": f"{pk['source']} bf16_tflops_sustained",
            "traffic": traffic_per_launch(),
            "traffic_algorithmic": algorithmic_per_launch(),
            "traffic_note": "ncu DRAM bytes per launch, mean over the step's launches (3 at d=4096, 1 at d=14336); "
                            "profiles/k_hessian_pair__*",
            "algorithmic": "N*d*(d+1) flop per launch (lower triangle incl. diagonal), N=16384 tokens; "
                           "achieved = these flops / CUDA-event time of the Hessian launches inside the timed steps",
            "launches_per_step": res["hessian_launches_per_step"],
            "ms_per_step": res["hessian_ms_per_step"],
        },
        "hessian_tflops": res["hessian_tflops"],
        "casts": ({k: {"gbs": v["gbs"], "frac": v["gbs"] / pk["hbm_gbs"], "batched_gbs": v["batched_gbs"],
                       "batched_frac": v["batched_gbs"] / pk["hbm_gbs"]} for k, v in res["casts"].items()}
                  if res["casts"] else None),
        "modelfree": ({k: {"gbs": v["gbs"], "frac": v["gbs"] / pk["hbm_gbs"], "ms": v["ms"], "weights": v["weights"]}
                       for k, v in res["modelfree"].items()} if res["modelfree"] else None),
        "gpu_launches": res["launches"],
        "clocks": res["clocks"],
    }
    if "e2e" in res:
        e = res["e2e"]
        line["e2e"] = {"value": (res["capture_ms"] + e["ms"] * L / args.steps) * 1e-3, "unit": "s",
                       "h2d_bytes_per_step": int(e["h2d_per_step"]), "d2h_bytes_per_step": int(e["d2h_per_step"]),
                       "note": "layer weights from pinned host memory in, quantized layer back out, loss read "
                               "on the host, every step"}
    if "c3" in res:
        line["c3"] = res["c3"]
    if args.cpu_baseline and world == 1:
        cb = cpu_sample(3, 1)
        line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
