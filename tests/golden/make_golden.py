"""Generate the golden fixtures in this directory from the reference itself.

Runs the reference llm-compressor (imported through ``ref_shim``) on CPU over
seeded synthetic inputs and stores inputs and outputs as ``.npz`` files:

* ``modelfree_<scheme>.npz`` -- the model-free per-tensor path
  (``S/entrypoints/model_free/lifecycle.py:38-60`` then
  ``CT/compressors/base.py:145`` ``compress_module``): bf16 weight in,
  compressed-tensors state dict out (packed codes, scales, global scale).
* ``observer_<case>.npz`` -- memoryless min-max statistics and
  ``calculate_qparams`` output (``S/observers/min_max.py:106-110``,
  ``S/observers/base.py:99-123``).
* ``mse_<case>.npz`` -- the ``memoryless_mse`` grid-search observer
  (``S/observers/mse.py``, ``S/observers/mse_quant.py``) and its qparams.
* ``repack_int4_int8.npz`` -- the checkpoint repacker's ``_pack_int4_to_int8``.
* ``actobs_<case>.npz`` -- the activation observers of static activation
  schemes (``S/observers/min_max.py:16-110``): statistics after each of four
  batches, then ``get_qparams``.
* ``hessian.npz`` -- ``accumulate_hessian`` over several calls
  (``S/modifiers/gptq/gptq_quantize.py:63-97``).
* ``gptq_<case>.npz`` -- ``quantize_weight``
  (``S/modifiers/gptq/gptq_quantize.py:100-296``) on a Hessian built from
  seeded activations.
* ``oneshot_c1.npz`` -- the reference's ``oneshot`` (sequential pipeline,
  ``GPTQModifier(scheme="W4A16", actorder=None, ignore=["lm_head"])``,
  ``S/entrypoints/oneshot.py:285``) on the 2-layer Llama of
  ``llmcompressor_b200.synthetic`` (hidden 1024, 32 x 512 calibration
  tokens), then ``compress_module`` of every quantized Linear: the first 128
  rows of each ``weight_packed`` / ``weight_scale`` (GPTQ rows are
  independent given the Hessian, so a row sample is a fair sample), the
  weight shapes, and the final hidden-state error of the quantized model.
* ``oneshot_c3tiny.npz`` -- the same for a 2-layer Qwen3-MoE at reduced width
  (``llmcompressor_b200.synthetic`` "c3tiny": 8 experts top-2) with the
  reference's all-expert calibration (``moe_calibrate_all_experts``, after its
  post-load ``linearize_moe``), the router ignored (``re:.*mlp.gate$``); all
  rows of every module.

bf16 tensors are stored as ``uint16`` bit patterns, fp8 as ``uint8``.
Only run where a reference checkout exists:
``LLMC_REFERENCE_SRC=<checkout>/src python tests/golden/make_golden.py``.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import ref_shim  # noqa: E402

ref_shim.install()

from compressed_tensors.compressors import compress_module  # noqa: E402
from compressed_tensors.quantization import (  # noqa: E402
    QuantizationArgs,
    QuantizationScheme,
    initialize_module_for_quantization,
)
from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme  # noqa: E402

from llmcompressor.modifiers.gptq.gptq_quantize import (  # noqa: E402
    accumulate_hessian,
    make_empty_hessian,
    quantize_weight,
)
from llmcompressor.modifiers.quantization.calibration import (  # noqa: E402
    apply_calibration_status,
    freeze_module_quantization,
    initialize_observer,
    observe,
    update_qparams,
)
from llmcompressor.observers import Observer  # noqa: E402
from llmcompressor.observers.helpers import fuse_weight_observers  # noqa: E402


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.uint16).numpy().astype(np.uint16)
    if t.dtype == torch.float8_e4m3fn:
        return t.view(torch.uint8).numpy()
    return t.numpy()


def make_weight(rows: int, cols: int, seed: int, kind: str = "normal") -> torch.Tensor:
    """Seeded bf16 weights with the value features the casts must handle."""
    g = torch.Generator().manual_seed(seed)
    if kind == "student_t":
        # Student-t(nu=4) rows scaled by 0.02: heavy tails
        z = torch.randn(rows, cols, generator=g)
        chi = torch.distributions.Chi2(torch.tensor(4.0)).sample((rows, 1))
        w = 0.02 * z / torch.sqrt(chi / 4.0)
    else:
        w = 0.02 * torch.randn(rows, cols, generator=g)
        mask = torch.rand(rows, cols, generator=g) < 0.001
        w = torch.where(mask, w * 50.0, w)
    # edge cases: an all-zero row, an all-positive row, a row of tiny values
    if rows >= 4:
        w[0, :] = 0.0
        w[1, :] = w[1, :].abs()
        w[2, :] = w[2, :] * 1e-6
        w[3, : cols // 2] = -w[3, : cols // 2].abs()
    return w.to(torch.bfloat16)


# --------------------------------------------------------------------------
# model-free path
# --------------------------------------------------------------------------


def modelfree_one(weight: torch.Tensor, scheme: QuantizationScheme) -> dict:
    """``initialize_quantized_linear`` + ``calibrate_weight`` + ``compress_module``.

    Version-skew notes for the installed compressed-tensors 0.15.0.1:

    * NVFP4: the scale is held in fp32 until ``compress_module``; the installed
      version rejects fp8/fp32 promotion in ``scale / global_scale``.  The fp32
      scale is already fp8-rounded by ``calculate_qparams``, so no value changes.
    * MXFP4: the scale is held in the weight dtype (compressed-tensors' own
      default scale dtype) until ``compress_module``, which encodes it as E8M0.
      Casting it to uint8 before calibration (``lifecycle.py:48-50``) would
      truncate the power-of-two scales through ``copy_``.
    """
    out_f, in_f = weight.shape
    module = torch.nn.Linear(in_f, out_f, bias=False, dtype=weight.dtype)
    module.weight.data.copy_(weight)
    initialize_module_for_quantization(module, scheme, force_zero_point=False)
    sd = scheme.weights.scale_dtype
    is_fp4 = scheme.weights.num_bits == 4 and scheme.weights.type == "float"
    if sd is not None and hasattr(module, "weight_scale") and not is_fp4:
        module.weight_scale.data = module.weight_scale.data.to(sd)
    if is_fp4 and scheme.weights.group_size == 16:
        module.weight_scale.data = module.weight_scale.data.to(torch.float32)
    initialize_observer(module, "weight")
    apply_calibration_status(module)
    observe(module, base_name="weight")
    update_qparams(module, base_name="weight")
    freeze_module_quantization(module)
    compress_module(module)
    return {k: v for k, v in module.state_dict().items()}


def gen_modelfree():
    cases = [
        ("W4A16", 64, 512, "normal"),
        ("W4A16_ASYM", 64, 512, "normal"),
        ("W8A16", 64, 256, "normal"),
        ("FP8_DYNAMIC", 64, 256, "student_t"),
        ("FP8", 64, 256, "normal"),
        ("FP8_BLOCK", 200, 300, "student_t"),
        ("MXFP4A16", 64, 256, "student_t"),
        ("NVFP4A16", 64, 256, "normal"),
    ]
    for i, (name, r, c, kind) in enumerate(cases):
        w = make_weight(r, c, seed=100 + i, kind=kind)
        scheme = preset_name_to_scheme(name, ["Linear"])
        sd = modelfree_one(w, scheme)
        arrays = {"weight": to_np(w)}
        for k, v in sd.items():
            arrays["out_" + k] = to_np(v)
        np.savez_compressed(os.path.join(HERE, f"modelfree_{name}.npz"), **arrays)
        print("modelfree", name, {k: (v.shape, v.dtype) for k, v in arrays.items()})


def gen_nvfp4_fused():
    """NVFP4 with q/k/v sharing one global scale (``S/observers/helpers.py:161-216``)."""

    class Attn(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = torch.nn.Linear(256, 128, bias=False, dtype=torch.bfloat16)
            self.k_proj = torch.nn.Linear(256, 64, bias=False, dtype=torch.bfloat16)
            self.v_proj = torch.nn.Linear(256, 64, bias=False, dtype=torch.bfloat16)

    m = Attn()
    ws = {}
    for j, n in enumerate(("q_proj", "k_proj", "v_proj")):
        w = make_weight(getattr(m, n).out_features, 256, seed=200 + j)
        if n == "k_proj":
            w[5, 7] = 3.0  # the fused absmax lives in k_proj
        getattr(m, n).weight.data.copy_(w)
        ws[n] = w
    scheme = preset_name_to_scheme("NVFP4A16", ["Linear"])
    for n in ("q_proj", "k_proj", "v_proj"):
        mod = getattr(m, n)
        initialize_module_for_quantization(mod, scheme, force_zero_point=False)
        mod.weight_scale.data = mod.weight_scale.data.to(torch.float32)
        initialize_observer(mod, "weight")
        apply_calibration_status(mod)
    fuse_weight_observers(m)
    arrays = {}
    for n in ("q_proj", "k_proj", "v_proj"):
        mod = getattr(m, n)
        observe(mod, base_name="weight")
        update_qparams(mod, base_name="weight")
    for n in ("q_proj", "k_proj", "v_proj"):
        mod = getattr(m, n)
        freeze_module_quantization(mod)
        compress_module(mod)
        arrays[f"{n}_weight"] = to_np(ws[n])
        for k, v in mod.state_dict().items():
            arrays[f"{n}_out_{k}"] = to_np(v)
    np.savez_compressed(os.path.join(HERE, "modelfree_NVFP4A16_fused_qkv.npz"), **arrays)
    print("nvfp4 fused", sorted(arrays))


# --------------------------------------------------------------------------
# observers
# --------------------------------------------------------------------------


def gen_observers():
    cases = {
        "int4_sym_group128": QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128),
        "int4_asym_group128": QuantizationArgs(num_bits=4, type="int", symmetric=False, strategy="group", group_size=128),
        "int8_sym_channel": QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="channel"),
        "int4_sym_tensor": QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="tensor"),
        "fp8_block_128": QuantizationArgs(num_bits=8, type="float", symmetric=True, strategy="block", block_structure=[128, 128]),
        "int8_asym_channel": QuantizationArgs(num_bits=8, type="int", symmetric=False, strategy="channel"),
    }
    for i, (name, args) in enumerate(cases.items()):
        r, c = (200, 300) if "block" in name else (96, 512)
        w = make_weight(r, c, seed=300 + i)
        obs = Observer.load_from_registry("memoryless_minmax", base_name="weight", args=args)
        obs(w)
        mn, mx = obs.min_vals.clone(), obs.max_vals.clone()
        qp = obs.get_qparams()
        np.savez_compressed(
            os.path.join(HERE, f"observer_{name}.npz"),
            weight=to_np(w),
            min_vals=to_np(mn),
            max_vals=to_np(mx),
            scale=to_np(qp["scale"]),
            zero_point=to_np(qp["zero_point"]),
        )
        print("observer", name, tuple(mn.shape), qp["scale"].dtype, qp["zero_point"].dtype)


MSE_CASES = {
    "int4_sym_group128": (QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128),
                          (96, 512)),
    "int4_asym_group128": (QuantizationArgs(num_bits=4, type="int", symmetric=False, strategy="group",
                                            group_size=128), (96, 512)),
    "int8_sym_channel": (QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="channel"), (96, 512)),
    "int8_asym_channel": (QuantizationArgs(num_bits=8, type="int", symmetric=False, strategy="channel"), (96, 512)),
    "int4_sym_tensor": (QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="tensor"), (64, 256)),
    "fp8_block_128": (QuantizationArgs(num_bits=8, type="float", symmetric=True, strategy="block",
                                       block_structure=[128, 128]), (200, 300)),
    "int4_sym_group32": (QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=32),
                         (64, 512)),
}


def gen_mse_observers():
    """``memoryless_mse`` (S/observers/mse.py:12-45 -> mse_quant.py:19-141, the
    eager grid search with the default maxshrink 0.2, grid 100, patience 5,
    norm 2.4) on bf16 weights, then ``get_qparams``."""
    for i, (name, (args, (r, c))) in enumerate(MSE_CASES.items()):
        w = make_weight(r, c, seed=500 + i, kind="student_t" if i % 2 else "normal")
        obs = Observer.load_from_registry("memoryless_mse", base_name="weight", args=args)
        obs(w)
        mn, mx = obs.min_vals.clone(), obs.max_vals.clone()
        qp = obs.get_qparams()
        np.savez_compressed(
            os.path.join(HERE, f"mse_{name}.npz"),
            weight=to_np(w),
            min_vals=to_np(mn),
            max_vals=to_np(mx),
            scale=to_np(qp["scale"]),
            zero_point=to_np(qp["zero_point"]),
        )
        print("mse", name, tuple(mn.shape), qp["scale"].dtype)


def gen_repack():
    """``_pack_int4_to_int8`` (S/utils/pack_int4_to_int8.py:13-28) on int4 codes
    and on arbitrary int8 values (the & 0x0F masking)."""
    from llmcompressor.utils.pack_int4_to_int8 import _pack_int4_to_int8

    g = torch.Generator().manual_seed(41)
    codes = torch.randint(-8, 8, (48, 96), generator=g, dtype=torch.int8)
    wild = torch.randint(-128, 128, (16, 64), generator=g, dtype=torch.int8)
    np.savez_compressed(os.path.join(HERE, "repack_int4_int8.npz"), codes=codes.numpy(),
                        codes_packed=_pack_int4_to_int8(codes).numpy(), wild=wild.numpy(),
                        wild_packed=_pack_int4_to_int8(wild).numpy())
    print("repack", tuple(codes.shape))


# --------------------------------------------------------------------------
# Hessian + GPTQ
# --------------------------------------------------------------------------


def gen_hessian():
    g = torch.Generator().manual_seed(7)
    d = 192
    lin = torch.nn.Linear(d, 64, bias=False, dtype=torch.bfloat16)
    H = make_empty_hessian(lin)
    n = torch.zeros(())
    xs = []
    for s in range(3):
        x = torch.randn(1, 80 + 16 * s, d, generator=g).to(torch.bfloat16)
        xs.append(to_np(x[0]))
        H, n = accumulate_hessian(x, lin, H, n)
    arrays = {f"x{i}": x for i, x in enumerate(xs)}
    arrays.update(H=to_np(H), num_samples=to_np(n))
    np.savez_compressed(os.path.join(HERE, "hessian.npz"), **arrays)
    print("hessian", H.shape, float(n))


def gptq_case(name, rows, cols, args, dead_cols=(), seed=11, tokens=512, blocksize=128, late_actorder=None):
    g = torch.Generator().manual_seed(seed)
    w = make_weight(rows, cols, seed=seed + 1)
    lin = torch.nn.Linear(cols, rows, bias=False, dtype=torch.bfloat16)
    lin.weight.data.copy_(w)
    # correlated activations: x = z @ M with a random mixing matrix
    mix = torch.randn(cols, cols, generator=g) / cols**0.5 + torch.eye(cols)
    H = make_empty_hessian(lin)
    n = torch.zeros(())
    xs = []
    for s in range(4):
        x = (torch.randn(tokens // 4, cols, generator=g) @ mix).to(torch.bfloat16)
        for dc in dead_cols:
            x[:, dc] = 0
        xs.append(to_np(x))
        H, n = accumulate_hessian(x.unsqueeze(0), lin, H, n)
    Hn = H / n
    scheme = QuantizationScheme(targets=["Linear"], weights=args)
    initialize_module_for_quantization(lin, scheme, force_zero_point=False)
    initialize_observer(lin, "weight")
    observe(lin, base_name="weight")
    if late_actorder is not None:
        # the installed compressed-tensors only accepts an ordering with group
        # strategies when args and schemes are validated, while quantize_weight
        # handles it for every strategy: set it on the args it reads
        args = args.model_copy()
        args.actorder = late_actorder
    loss, qd = quantize_weight(lin, args, Hn.clone(), blocksize=blocksize, percdamp=0.01)
    arrays = {
        "weight": to_np(w),
        "x": np.stack(xs),
        "hessian": to_np(Hn),
        "loss": np.array(loss, dtype=np.float64),
        "blocksize": np.array(blocksize),
        "out_weight": to_np(qd["weight"]),
        "out_scale": to_np(qd["weight_scale"]),
        "out_zero_point": to_np(qd["weight_zero_point"]),
    }
    if "weight_g_idx" in qd:
        arrays["out_g_idx"] = qd["weight_g_idx"].numpy().astype(np.int32)
    if "weight_global_scale" in qd:
        arrays["out_global_scale"] = to_np(qd["weight_global_scale"])
    np.savez_compressed(os.path.join(HERE, f"gptq_{name}.npz"), **arrays)
    print("gptq", name, loss)


def gen_gptq():
    gptq_case(
        "int4_group128",
        128,
        384,
        QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128, actorder=None),
    )
    gptq_case(
        "int4_channel_dead",
        96,
        256,
        QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="channel", actorder=None),
        dead_cols=(3, 100, 255),
        seed=21,
    )
    gptq_case(
        "int8_group64_asym",
        64,
        320,
        QuantizationArgs(num_bits=8, type="int", symmetric=False, strategy="group", group_size=64, actorder=None),
        seed=31,
    )


def gen_gptq_orderings():
    """Activation ordering, block strategy, float formats and a block size
    other than 128 (T/llmcompressor/modifiers/gptq/test_gptq_quantize.py
    covers the same options on toy shapes)."""
    from compressed_tensors.quantization import ActivationOrdering

    def nvfp4_args():
        return preset_name_to_scheme("NVFP4A16", ["Linear"]).weights

    def mxfp4_args():
        return preset_name_to_scheme("MXFP4A16", ["Linear"]).weights

    cases = [
        ("int4_group128_actweight", 128, 384,
         QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128,
                          actorder=ActivationOrdering.WEIGHT), {}),
        ("int4_group32_actgroup", 96, 256,
         QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=32,
                          actorder=ActivationOrdering.GROUP), {"seed": 41}),
        ("int4_channel_actstatic", 64, 256,
         QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="channel"),
         {"seed": 51, "dead_cols": (7, 200), "actorder": ActivationOrdering.STATIC}),
        ("int8_block32x64_bs64", 96, 320,
         QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="block", block_structure=[32, 64],
                          actorder=None), {"seed": 61, "blocksize": 64}),
        ("int8_block48x96_actweight", 100, 320,
         QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="block", block_structure=[48, 96]),
         {"seed": 71, "actorder": ActivationOrdering.WEIGHT}),
        ("fp8_channel", 64, 256,
         QuantizationArgs(num_bits=8, type="float", symmetric=True, strategy="channel", actorder=None),
         {"seed": 81}),
        ("nvfp4_actweight", 64, 256, None, {"seed": 91, "args_fn": nvfp4_args, "actorder": ActivationOrdering.WEIGHT}),
        ("mxfp4", 64, 256, None, {"seed": 101, "args_fn": mxfp4_args}),
    ]
    only = set(sys.argv[2:])
    for name, rows, cols, args, kw in cases:
        if only and name not in only:
            continue
        kw = dict(kw)
        fn = kw.pop("args_fn", None)
        order = kw.pop("actorder", None)
        if fn is not None:
            args = fn()
        gptq_case(name, rows, cols, args, late_actorder=order, **kw)


def gen_act_observers():
    """Activation observers of static activation schemes
    (S/observers/min_max.py:16-110) over several calibration batches: the
    statistics after every batch, then ``get_qparams``."""
    nvfp4_in = preset_name_to_scheme("NVFP4", ["Linear"]).input_activations
    cases = [
        ("minmax_int8_tensor", "minmax", "input", (2, 48, 256),
         QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="tensor", dynamic=False, observer="minmax")),
        ("static_int8_asym_tensor", "static_minmax", "input", (2, 48, 256),
         QuantizationArgs(num_bits=8, type="int", symmetric=False, strategy="tensor", dynamic=False,
                          observer="static_minmax")),
        ("minmax_nvfp4_tensor_group", "minmax", "input", (2, 48, 256), nvfp4_in),
        ("memoryless_int8_group128", "memoryless_minmax", "input", (3, 40, 512),
         QuantizationArgs(num_bits=8, type="int", symmetric=False, strategy="group", group_size=128, dynamic=False,
                          observer="memoryless_minmax")),
        ("static_fp8_kv_tensor", "static_minmax", "k", (2, 4, 24, 64),
         QuantizationArgs(num_bits=8, type="float", symmetric=True, strategy="tensor", dynamic=False,
                          observer="static_minmax")),
        ("minmax_c05_fp8_tensor", "minmax", "output", (2, 32, 256),
         QuantizationArgs(num_bits=8, type="float", symmetric=True, strategy="tensor", dynamic=False,
                          observer="minmax", observer_kwargs={"averaging_constant": 0.5})),
    ]
    for name, obs_name, base, shape, args in cases:
        g = torch.Generator().manual_seed(sum(map(ord, name)))
        obs = Observer.load_from_registry(obs_name, base_name=base, args=args)
        arrays = {}
        for b, mul in enumerate([1.0, 3.0, 0.5, 2.0]):
            feat = torch.exp(0.7 * torch.randn(shape[-1], generator=g))
            x = (mul * torch.randn(*shape, generator=g) * feat + 0.3 * mul).to(torch.bfloat16)
            obs(x)
            arrays[f"x{b}"] = to_np(x)
            arrays[f"min{b}"] = to_np(obs.min_vals.to(torch.bfloat16))
            arrays[f"max{b}"] = to_np(obs.max_vals.to(torch.bfloat16))
        q = obs.get_qparams()
        arrays["scale"] = to_np(q["scale"])
        arrays["zero_point"] = to_np(q["zero_point"])
        if q.get("global_scale") is not None:
            arrays["global_scale"] = to_np(q["global_scale"])
        np.savez_compressed(os.path.join(HERE, f"actobs_{name}.npz"), **arrays)
        print("actobs", name, arrays["min3"][:4], arrays["max3"][:4], arrays["scale"].reshape(-1)[:2])


# --------------------------------------------------------------------------
# oneshot GPTQ W4A16 end to end (config C1)
# --------------------------------------------------------------------------

ONESHOT_ROWS = 128


def gen_oneshot_c1():
    import time

    from torch.utils.data import DataLoader

    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from llmcompressor_b200 import synthetic

    from llmcompressor import oneshot
    from llmcompressor.modifiers.gptq import GPTQModifier

    model = synthetic.random_llama("c1")
    ids = synthetic.calibration_tokens("c1")
    data = [{"input_ids": ids[i:i + 1], "attention_mask": torch.ones_like(ids[i:i + 1])} for i in range(len(ids))]
    t0 = time.time()
    oneshot(model=model, dataset=DataLoader(data, batch_size=None, shuffle=False), processor=object(),
            recipe=GPTQModifier(targets="Linear", scheme="W4A16", ignore=["lm_head"], actorder=None,
                                block_size=128, dampening_frac=0.01),
            pipeline="sequential", num_calibration_samples=len(ids), shuffle_calibration_samples=False)
    secs = time.time() - t0
    arrays = {"oneshot_seconds": np.array(secs), "rows": np.array(ONESHOT_ROWS)}
    # end-to-end effect: final hidden states of the quantized model against the unquantized one
    fp = synthetic.random_llama("c1")
    with torch.no_grad():
        hq = model.model(ids[:4]).last_hidden_state.float()
        hf = fp.model(ids[:4]).last_hidden_state.float()
    arrays["hidden_rel_err"] = (torch.linalg.norm((hq - hf).reshape(4, -1), dim=1)
                                / torch.linalg.norm(hf.reshape(4, -1), dim=1)).numpy()
    names = []
    for name, mod in model.named_modules():
        if not isinstance(mod, torch.nn.Linear) or not hasattr(mod, "weight_scale"):
            continue
        compress_module(mod)
        sd = mod.state_dict()
        arrays[f"{name}.weight_packed"] = sd["weight_packed"][:ONESHOT_ROWS].numpy()
        arrays[f"{name}.weight_scale"] = to_np(sd["weight_scale"][:ONESHOT_ROWS])
        arrays[f"{name}.weight_shape"] = sd["weight_shape"].numpy()
        names.append(name)
    arrays["modules"] = np.array(names)
    np.savez_compressed(os.path.join(HERE, "oneshot_c1.npz"), **arrays)
    print("oneshot c1", f"{secs:.1f}s", names, arrays["hidden_rel_err"])


def gen_oneshot_c3tiny():
    import time

    from torch.utils.data import DataLoader

    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    from llmcompressor_b200 import synthetic

    from llmcompressor import oneshot
    from llmcompressor.modifiers.gptq import GPTQModifier

    model = synthetic.random_qwen3_moe("c3tiny")
    ids = synthetic.calibration_tokens("c3tiny")
    data = [{"input_ids": ids[i:i + 1], "attention_mask": torch.ones_like(ids[i:i + 1])} for i in range(len(ids))]
    t0 = time.time()
    oneshot(model=model, dataset=DataLoader(data, batch_size=None, shuffle=False), processor=object(),
            recipe=GPTQModifier(targets="Linear", scheme="W4A16", ignore=["lm_head", "re:.*mlp.gate$"],
                                actorder=None, block_size=128, dampening_frac=0.01),
            pipeline="sequential", num_calibration_samples=len(ids), shuffle_calibration_samples=False,
            moe_calibrate_all_experts=True)
    secs = time.time() - t0
    arrays = {"oneshot_seconds": np.array(secs)}
    fp = synthetic.random_qwen3_moe("c3tiny")
    with torch.no_grad():
        hq = model.model(ids[:4]).last_hidden_state.float()
        hf = fp.model(ids[:4]).last_hidden_state.float()
    arrays["hidden_rel_err"] = (torch.linalg.norm((hq - hf).reshape(4, -1), dim=1)
                                / torch.linalg.norm(hf.reshape(4, -1), dim=1)).numpy()
    names = []
    for name, mod in model.named_modules():
        if not isinstance(mod, torch.nn.Linear) or not hasattr(mod, "weight_scale"):
            continue
        compress_module(mod)
        sd = mod.state_dict()
        arrays[f"{name}.weight_packed"] = sd["weight_packed"].numpy()
        arrays[f"{name}.weight_scale"] = to_np(sd["weight_scale"])
        arrays[f"{name}.weight_shape"] = sd["weight_shape"].numpy()
        names.append(name)
    arrays["modules"] = np.array(names)
    np.savez_compressed(os.path.join(HERE, "oneshot_c3tiny.npz"), **arrays)
    print("oneshot c3tiny", f"{secs:.1f}s", len(names), arrays["hidden_rel_err"])


if __name__ == "__main__":
    torch.manual_seed(0)
    if sys.argv[1:2] == ["oneshot_c3tiny"]:
        gen_oneshot_c3tiny()
        sys.exit(0)
    if sys.argv[1:2] == ["oneshot_c1"]:
        gen_oneshot_c1()
        sys.exit(0)
    if sys.argv[1:2] == ["act_observers"]:
        gen_act_observers()
        sys.exit(0)
    if sys.argv[1:2] == ["gptq_orderings"]:
        gen_gptq_orderings()
        sys.exit(0)
    if sys.argv[1:] == ["mse"]:
        gen_mse_observers()
        sys.exit(0)
    if sys.argv[1:] == ["repack"]:
        gen_repack()
        sys.exit(0)
    gen_observers()
    gen_mse_observers()
    gen_repack()
    gen_modelfree()
    gen_nvfp4_fused()
    gen_hessian()
    gen_gptq()
    gen_gptq_orderings()
    gen_act_observers()
    gen_oneshot_c1()
    gen_oneshot_c3tiny()
