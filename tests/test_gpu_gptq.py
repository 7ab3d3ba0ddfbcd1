"""GPU parity of the GPTQ solve (damping, inverse factor, block loop) through the C ABI.

Bar: GPTQ integer codes >= 99% identical to the
reference's, loss and per-layer output error ||(W-Q)X||^2/||WX||^2 within 1%
relative of the reference's."""
import numpy as np
import pytest
import torch
from compressed_tensors.quantization import QuantizationArgs

from golden_io import bf16, load
from gpu_util import np_f32, to_dev_bf16
from llmcompressor_b200 import gptq, ops
from oracle import gptq as ogptq
from oracle.observers import QArgs

pytestmark = pytest.mark.gpu
CODE_AGREE = 0.99
REL = 0.01

CASES = {
    "int4_group128": (QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128,
                                       actorder=None), QArgs(4, "int", True, "group", 128)),
    "int4_channel_dead": (QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="channel", actorder=None),
                          QArgs(4, "int", True, "channel", None)),
    "int8_group64_asym": (QuantizationArgs(num_bits=8, type="int", symmetric=False, strategy="group", group_size=64,
                                           actorder=None), QArgs(8, "int", False, "group", 64)),
}


def _linear(w: torch.Tensor) -> torch.nn.Linear:
    lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=False, dtype=torch.bfloat16, device="cuda")
    lin.weight.data.copy_(w)
    return lin


def _codes(wq: np.ndarray, scale: np.ndarray, zp, qa: QArgs) -> np.ndarray:
    return ogptq.codes_from_weight(wq, scale, zp, qa)


@pytest.mark.parametrize("case", sorted(CASES))
def test_gptq_golden_fixture(case):
    g = load(f"gptq_{case}")
    args, qa = CASES[case]
    w = to_dev_bf16(g["weight"])
    H = torch.from_numpy(g["hessian"]).cuda()
    loss, qd = gptq.quantize_weight(_linear(w), args, H.clone(), blocksize=128, percdamp=0.01)
    scale = np_f32(qd["weight_scale"])
    np.testing.assert_array_equal(qd["weight_scale"].view(torch.int16).cpu().numpy().view(np.uint16),
                                  g["out_scale"].reshape(tuple(qd["weight_scale"].shape)))
    zp = qd["weight_zero_point"].cpu().numpy()
    ours = _codes(np_f32(qd["weight"]), scale, zp, qa)
    ref = _codes(bf16(g["out_weight"]), scale, zp, qa)
    agree = float(np.mean(ours == ref))
    assert agree >= CODE_AGREE, agree
    assert abs(loss - float(g["loss"])) <= REL * abs(float(g["loss"])), (loss, float(g["loss"]))
    x = bf16(g["x"])
    wf = bf16(g["weight"])
    e_ref = ogptq.layer_output_error(wf, bf16(g["out_weight"]), x)
    e_new = ogptq.layer_output_error(wf, np_f32(qd["weight"]), x)
    assert abs(e_new - e_ref) <= REL * e_ref, (e_new, e_ref)


def _random_problem(rows, cols, tokens, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (0.02 * torch.randn(rows, cols, device="cuda", generator=g)).to(torch.bfloat16)
    mix = torch.randn(cols, cols, device="cuda", generator=g) / cols**0.5 + torch.eye(cols, device="cuda")
    x = (torch.randn(tokens, cols, device="cuda", generator=g) @ mix).to(torch.bfloat16)
    H = torch.zeros(cols, cols, device="cuda")
    gptq.hessian_update_(H, x, 2.0)
    H /= 1.0
    return w, x, H


def test_gptq_vs_oracle_random():
    args, qa = CASES["int4_group128"]
    w, x, H = _random_problem(256, 1024, 2048, seed=3)
    loss, qd = gptq.quantize_weight(_linear(w), args, H.clone())
    oloss, owq, oscale, ozp, ok = ogptq.quantize_weight(np_f32(w), H.cpu().numpy(), qa)
    assert ok
    ours = _codes(np_f32(qd["weight"]), oscale, ozp, qa)
    ref = _codes(owq, oscale, ozp, qa)
    assert float(np.mean(ours == ref)) >= CODE_AGREE
    assert abs(loss - oloss) <= REL * oloss
    xn = np_f32(x)
    e_ref = ogptq.layer_output_error(np_f32(w), owq, xn)
    e_new = ogptq.layer_output_error(np_f32(w), np_f32(qd["weight"]), xn)
    assert abs(e_new - e_ref) <= REL * e_ref


@pytest.mark.parametrize("d", [256, 1000, 4096])
def test_inverse_factor_vs_fp64(d):
    _, _, H = _random_problem(8, d, 4 * d, seed=d)
    A = H.double().clone()
    damp = 0.01 * torch.mean(torch.diag(A))
    A += damp * torch.eye(d, device="cuda", dtype=torch.float64)
    inv = gptq.inverse_hessian(H.clone(), 0.01)
    assert inv.ok()
    U = inv.hinv.double()
    ref = torch.linalg.cholesky(torch.cholesky_inverse(torch.linalg.cholesky(A)), upper=True)
    rel = float(torch.linalg.norm(U - ref) / torch.linalg.norm(ref))
    assert rel < 2e-3, rel
    assert torch.all(torch.tril(inv.hinv, -1) == 0)


def test_not_positive_definite_falls_back_to_rtn():
    args, qa = CASES["int4_channel_dead"]
    g = torch.Generator().manual_seed(9)
    w = (0.02 * torch.randn(64, 256, generator=g)).to(torch.bfloat16)
    H = -torch.eye(256)
    loss, qd = gptq.quantize_weight(_linear(w.cuda()), args, H.cuda())
    oloss, owq, _, _, ok = ogptq.quantize_weight(np_f32(w), H.numpy(), qa)
    assert not ok
    np.testing.assert_array_equal(np_f32(qd["weight"]), owq)
    assert abs(loss - oloss) <= 1e-5 * abs(oloss)


def test_shared_inverse_matches_separate_calls():
    """q/k/v share one Hessian: one factorisation, three block loops."""
    args, _ = CASES["int4_group128"]
    g = torch.Generator(device="cuda").manual_seed(4)
    cols = 512
    ws = [(0.02 * torch.randn(r, cols, device="cuda", generator=g)).to(torch.bfloat16) for r in (512, 128, 128)]
    _, _, H = _random_problem(8, cols, 1024, seed=5)
    inv = gptq.inverse_hessian(H.clone(), 0.01)
    for w in ws:
        mn, mx = ops.observe_minmax(w, args)
        scale, zp = ops.calculate_qparams(mn, mx, args)
        wq_shared, loss_shared = gptq.quantize_with_inverse(w, args, inv, scale, zp)
        loss_sep, qd = gptq.quantize_weight(_linear(w), args, H.clone())
        assert torch.equal(wq_shared, qd["weight"])
        assert float(loss_shared) == loss_sep


def test_gptq_beats_rtn_on_output_error_at_scale():
    """Size-independent property at a full Llama-3-8B shape (4096 x 4096):
    GPTQ's layer output error is below round-to-nearest's."""
    args, qa = CASES["int4_group128"]
    w, x, H = _random_problem(4096, 4096, 8192, seed=11)
    loss, qd = gptq.quantize_weight(_linear(w), args, H.clone())
    rtn = ops.quantize_pack(w, args, *ops.calculate_qparams(*ops.observe_minmax(w, args), args))
    assert loss > 0 and np.isfinite(loss)
    mn, mx = ops.observe_minmax(w, args)
    scale, _ = ops.calculate_qparams(mn, mx, args)
    # dequantize the RTN codes on the host
    packed = rtn.cpu().numpy().view(np.uint32)
    codes = np.stack([(packed >> (4 * j)) & 0xF for j in range(8)], axis=-1).reshape(4096, 4096).astype(np.int32) - 8
    s = np.repeat(np_f32(scale), 128, axis=1)
    w_rtn = (codes * s).astype(np.float32)
    xs = x[:2048].float()
    wf = w.float()
    e_gptq = float(torch.sum(((wf - qd["weight"].float()) @ xs.T) ** 2) / torch.sum((wf @ xs.T) ** 2))
    e_rtn = float(torch.sum(((wf - torch.from_numpy(w_rtn).cuda()) @ xs.T) ** 2) / torch.sum((wf @ xs.T) ** 2))
    assert e_gptq < e_rtn, (e_gptq, e_rtn)
