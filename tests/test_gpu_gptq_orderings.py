"""GPU parity of GPTQ with activation ordering (WEIGHT / STATIC / GROUP), the
BLOCK and TENSOR_GROUP strategies, FP8 / FP4 types and block sizes other than
128 (S/modifiers/gptq/gptq_quantize.py:100-310), through the C ABI.

Bar: scales (and g_idx, global scales) bit-exact; GPTQ codes >= 99%
identical to the reference's; loss and ||(W-Q)X||^2/||WX||^2 within 1%."""
import numpy as np
import pytest
import torch
from compressed_tensors.quantization import ActivationOrdering, QuantizationArgs
from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme

from golden_io import bf16, load
from gpu_util import np_f32, to_dev_bf16
from llmcompressor_b200 import gptq
from oracle import gptq as ogptq
from oracle import numerics
from oracle.observers import QArgs

pytestmark = pytest.mark.gpu
CODE_AGREE = 0.99
REL = 0.01


def _args(kind, **kw):
    if kind == "nvfp4":
        return preset_name_to_scheme("NVFP4A16", ["Linear"]).weights
    if kind == "mxfp4":
        return preset_name_to_scheme("MXFP4A16", ["Linear"]).weights
    return QuantizationArgs(**kw)


def _with_order(args, order):
    """The ordering set on the args quantize_weight reads (the installed
    compressed-tensors validates it only for group strategies at
    construction)."""
    if order is None:
        return args
    args = args.model_copy()
    args.actorder = order
    return args


# fixture -> (QuantizationArgs, oracle QArgs, ordering)
CASES = {
    "int4_group128_actweight": (_args(None, num_bits=4, type="int", symmetric=True, strategy="group", group_size=128),
                                QArgs(4, "int", True, "group", 128), ActivationOrdering.WEIGHT),
    "int4_group32_actgroup": (_args(None, num_bits=4, type="int", symmetric=True, strategy="group", group_size=32),
                              QArgs(4, "int", True, "group", 32), ActivationOrdering.GROUP),
    "int4_channel_actstatic": (_args(None, num_bits=4, type="int", symmetric=True, strategy="channel"),
                               QArgs(4, "int", True, "channel", None), ActivationOrdering.STATIC),
    "int8_block32x64_bs64": (_args(None, num_bits=8, type="int", symmetric=True, strategy="block",
                                   block_structure=[32, 64]), QArgs(8, "int", True, "block", None, (32, 64)), None),
    "int8_block48x96_actweight": (_args(None, num_bits=8, type="int", symmetric=True, strategy="block",
                                        block_structure=[48, 96]), QArgs(8, "int", True, "block", None, (48, 96)),
                                  ActivationOrdering.WEIGHT),
    "fp8_channel": (_args(None, num_bits=8, type="float", symmetric=True, strategy="channel"),
                    QArgs(8, "float", True, "channel", None, zp_dtype="fp8"), None),
    "nvfp4_actweight": (_args("nvfp4"), QArgs(4, "float", True, "tensor_group", 16, scale_dtype="fp8", zp_dtype="fp8"),
                        ActivationOrdering.WEIGHT),
    "mxfp4": (_args("mxfp4"), QArgs(4, "float", True, "group", 32, scale_dtype="uint8", zp_dtype="uint8"), None),
}


def _linear(w: torch.Tensor) -> torch.nn.Linear:
    lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=False, dtype=torch.bfloat16, device="cuda")
    lin.weight.data.copy_(w)
    return lin


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("case", sorted(CASES))
def test_orderings_golden_fixture(case):
    g = load(f"gptq_{case}")
    args, qa, order = CASES[case]
    args = _with_order(args, order)
    w = to_dev_bf16(g["weight"])
    H = torch.from_numpy(g["hessian"]).cuda()
    loss, qd = gptq.quantize_weight(_linear(w), args, H.clone(), blocksize=int(g["blocksize"]), percdamp=0.01)
    np.testing.assert_array_equal(_bits(qd["weight_scale"]), g["out_scale"].reshape(tuple(qd["weight_scale"].shape)))
    g_idx = None
    if "out_g_idx" in g:
        g_idx = qd["weight_g_idx"].cpu().numpy()
        np.testing.assert_array_equal(g_idx, g["out_g_idx"])
    else:
        assert "weight_g_idx" not in qd
    gs = None
    if "out_global_scale" in g:
        np.testing.assert_array_equal(_bits(qd["weight_global_scale"]).reshape(-1), g["out_global_scale"].reshape(-1))
        gs = np.float32(numerics.bf16_bits_to_f32(_bits(qd["weight_global_scale"])).reshape(-1)[0])
    scale = np_f32(qd["weight_scale"])
    zp = qd["weight_zero_point"].to(torch.float32).cpu().numpy()
    ours = ogptq.codes_from_weight(np_f32(qd["weight"]), scale, zp, qa, g_idx, gs)
    ref = ogptq.codes_from_weight(bf16(g["out_weight"]), scale, zp, qa, g_idx, gs)
    agree = float(np.mean(ours == ref))
    assert agree >= CODE_AGREE, agree
    assert abs(loss - float(g["loss"])) <= REL * abs(float(g["loss"])), (loss, float(g["loss"]))
    x = bf16(g["x"])
    wf = bf16(g["weight"])
    e_ref = ogptq.layer_output_error(wf, bf16(g["out_weight"]), x)
    e_new = ogptq.layer_output_error(wf, np_f32(qd["weight"]), x)
    assert abs(e_new - e_ref) <= REL * e_ref, (e_new, e_ref)


def _problem(rows, cols, seed):
    g = torch.Generator().manual_seed(seed)
    w = (0.02 * torch.randn(rows, cols, generator=g)).to(torch.bfloat16)
    mix = torch.randn(cols, cols, generator=g) / cols ** 0.5 + torch.eye(cols)
    x = (torch.randn(4 * cols, cols, generator=g) * torch.exp(torch.randn(cols, generator=g)) @ mix)
    x = x.to(torch.bfloat16).float()
    H = 2.0 * x.T @ x / x.shape[0]
    return w, H


@pytest.mark.parametrize("case", ["int4_g128_weight", "int4_g64_group", "int8_block_weight", "nvfp4_weight",
                                  "fp8_channel_bs32"])
def test_orderings_vs_oracle_random(case):
    """Shapes past one 128-column block and one 64-row CTA, against the oracle."""
    rows, cols = 192, 640
    bs = 128
    if case == "int4_g128_weight":
        args = _args(None, num_bits=4, type="int", symmetric=True, strategy="group", group_size=128)
        qa, order = QArgs(4, "int", True, "group", 128), ActivationOrdering.WEIGHT
    elif case == "int4_g64_group":
        args = _args(None, num_bits=4, type="int", symmetric=False, strategy="group", group_size=64)
        qa, order = QArgs(4, "int", False, "group", 64), ActivationOrdering.GROUP
    elif case == "int8_block_weight":
        args = _args(None, num_bits=8, type="int", symmetric=True, strategy="block", block_structure=[64, 128])
        qa, order = QArgs(8, "int", True, "block", None, (64, 128)), ActivationOrdering.WEIGHT
    elif case == "nvfp4_weight":
        args = _args("nvfp4")
        qa, order = QArgs(4, "float", True, "tensor_group", 16, scale_dtype="fp8", zp_dtype="fp8"), \
            ActivationOrdering.WEIGHT
    else:
        args = _args(None, num_bits=8, type="float", symmetric=True, strategy="channel")
        qa, order, bs = QArgs(8, "float", True, "channel", None, zp_dtype="fp8"), None, 32
    args = _with_order(args, order)
    w, H = _problem(rows, cols, seed=sum(map(ord, case)))
    loss, qd = gptq.quantize_weight(_linear(w.cuda()), args, H.cuda(), blocksize=bs)
    res = ogptq.quantize_weight(np_f32(w), H.numpy(), qa, blocksize=bs, actorder=order)
    oloss, owq, oscale, ozp, ok = res[:5]
    extra = res[5] if len(res) > 5 else {}
    assert ok
    np.testing.assert_array_equal(_bits(qd["weight_scale"]), numerics.f32_to_bf16_bits(oscale).reshape(-1).reshape(
        tuple(qd["weight_scale"].shape)))
    g_idx = extra.get("g_idx")
    if g_idx is not None:
        np.testing.assert_array_equal(qd["weight_g_idx"].cpu().numpy(), g_idx)
    gs = extra.get("global_scale")
    zp = qd["weight_zero_point"].to(torch.float32).cpu().numpy()
    scale = np_f32(qd["weight_scale"])
    ours = ogptq.codes_from_weight(np_f32(qd["weight"]), scale, zp, qa, g_idx, gs)
    ref = ogptq.codes_from_weight(owq, scale, zp, qa, g_idx, gs)
    agree = float(np.mean(ours == ref))
    assert agree >= CODE_AGREE, agree
    assert abs(loss - oloss) <= REL * abs(oloss), (loss, oloss)


def test_actorder_perm_and_permutations():
    """argsort(diag(H), descending) with ties in index order; H[perm][:, perm]
    and w[:, perm] exact."""
    d = 1000
    g = torch.Generator().manual_seed(3)
    H = torch.randn(d, d, generator=g)
    diag = torch.randint(0, 50, (d,), generator=g).float()  # many ties
    diag[::97] = 0.0
    H[torch.arange(d), torch.arange(d)] = diag
    perm = gptq.actorder_perm(H.cuda()).cpu().numpy()
    np.testing.assert_array_equal(perm, np.argsort(-diag.numpy(), kind="stable"))
    Hp = gptq.permute_hessian(H.cuda(), torch.from_numpy(perm).cuda()).cpu().numpy()
    np.testing.assert_array_equal(Hp, H.numpy()[perm][:, perm])
    w = torch.randn(37, d, generator=g).to(torch.bfloat16)
    wp = gptq.permute_columns(w.cuda(), torch.from_numpy(perm).cuda()).cpu()
    assert torch.equal(wp, w[:, torch.from_numpy(perm).long()])


# --- T/llmcompressor/modifiers/gptq/test_gptq_quantize.py, on bf16 Linear weights ----
def _reference_style(module, args, hessian, **kw):
    return gptq.quantize_weight(module=module, quant_args=args, hessian=hessian, **kw)


@pytest.mark.parametrize("actorder", [None, ActivationOrdering.WEIGHT, ActivationOrdering.GROUP])
def test_quantize_weight_group_strategy_actorder(actorder):
    torch.manual_seed(0)
    module = torch.nn.Linear(8, 6, bias=False, dtype=torch.bfloat16, device="cuda")
    args = QuantizationArgs(num_bits=4, symmetric=True, strategy="group", group_size=2, actorder=actorder)
    hessian = gptq.make_empty_hessian(module)
    hessian += torch.diag(torch.arange(1, hessian.shape[0] + 1, dtype=hessian.dtype, device=hessian.device))
    loss, q = _reference_style(module, args, hessian)
    assert loss >= 0
    assert q["weight"].shape == module.weight.shape
    assert q["weight_scale"].shape == (6, 4)
    assert q["weight_zero_point"].shape == (6, 4)
    if actorder == ActivationOrdering.GROUP:
        assert q["weight_g_idx"].shape == (8,)
        # descending diag -> reversed columns -> groups of the reversed order
        np.testing.assert_array_equal(q["weight_g_idx"].cpu().numpy(), (7 - np.arange(8)) // 2)


@pytest.mark.parametrize("actorder", [None, ActivationOrdering.WEIGHT])
def test_quantize_weight_supports_block_strategy(actorder):
    torch.manual_seed(0)
    module = torch.nn.Linear(7, 5, bias=False, dtype=torch.bfloat16, device="cuda")
    args = _with_order(QuantizationArgs(num_bits=8, symmetric=True, strategy="block", block_structure=[2, 4]),
                       actorder)
    hessian = gptq.make_empty_hessian(module)
    hessian += torch.eye(hessian.shape[0], dtype=hessian.dtype, device=hessian.device)
    loss, q = _reference_style(module, args, hessian, blocksize=3)
    assert loss >= 0
    assert q["weight"].shape == module.weight.shape
    assert q["weight_scale"].shape == (3, 2)
    assert q["weight_zero_point"].shape == (3, 2)
    assert "weight_g_idx" not in q
    # against the oracle on the same inputs
    qa = QArgs(8, "int", True, "block", None, (2, 4))
    res = ogptq.quantize_weight(np_f32(module.weight), hessian.cpu().numpy(), qa, blocksize=3,
                                actorder=actorder)
    np.testing.assert_array_equal(_bits(q["weight_scale"]), numerics.f32_to_bf16_bits(res[2]))
    assert abs(loss - res[0]) <= REL * max(abs(res[0]), 1e-6)


def test_quantize_weight_channel_actorder_weight():
    torch.manual_seed(0)
    module = torch.nn.Linear(8, 4, bias=False, dtype=torch.bfloat16, device="cuda")
    args = _with_order(QuantizationArgs(num_bits=4, symmetric=True, strategy="channel"), ActivationOrdering.WEIGHT)
    hessian = gptq.make_empty_hessian(module)
    hessian += torch.diag(torch.arange(1, hessian.shape[0] + 1, dtype=hessian.dtype, device=hessian.device))
    loss, q = _reference_style(module, args, hessian, blocksize=4)
    assert loss >= 0
    assert q["weight"].shape == module.weight.shape
    assert q["weight_scale"].shape[0] == module.weight.shape[0]
    assert q["weight_zero_point"].shape[0] == module.weight.shape[0]
    assert "weight_g_idx" not in q


def test_group_ordering_on_channel_falls_back():
    """GROUP ordering with a non-group strategy warns and runs without ordering (:126-134)."""
    module = torch.nn.Linear(64, 32, bias=False, dtype=torch.bfloat16, device="cuda")
    args = _with_order(QuantizationArgs(num_bits=4, symmetric=True, strategy="channel"), ActivationOrdering.GROUP)
    args_none = QuantizationArgs(num_bits=4, symmetric=True, strategy="channel")
    H = torch.eye(64, device="cuda") * torch.arange(1, 65, device="cuda")
    l1, q1 = gptq.quantize_weight(module, args, H.clone())
    l2, q2 = gptq.quantize_weight(module, args_none, H.clone())
    assert torch.equal(q1["weight"], q2["weight"]) and l1 == l2
    assert "weight_g_idx" not in q1
