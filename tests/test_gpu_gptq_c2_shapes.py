"""GPTQ at the Llama-3-8B module shapes against the CPU oracle (the numpy
restatement of the reference's ``quantize_weight``, pinned to the
reference's fixtures in test_oracle_golden.py).

q_proj 4096 x 4096, k_proj 1024 x 4096 and gate_proj 14336 x 4096 read a
4096-wide Hessian; down_proj 4096 x 14336 reads a 14336-wide one -- the
factorisation and the 14336-column block loop on the critical path of every
layer.  Our solve runs on the whole weight; the oracle solves a sample of
rows at full width (GPTQ rows are independent given the Hessian, so a row
sample is a fair sample).  Bar: codes >= 99% identical, loss and
||(W - Q) X||^2 / ||W X||^2 within 1% relative, on the sampled rows.  The
Hessians come from 8192 tokens with per-feature log-normal scales, built by
the tensor-core kernel (within 1e-5 of the exact sum)."""
import numpy as np
import pytest
import torch
from compressed_tensors.quantization import QuantizationArgs

from gpu_util import np_f32
from llmcompressor_b200 import gptq
from oracle import gptq as ogptq
from oracle.observers import QArgs

pytestmark = pytest.mark.gpu
ARGS = QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128, actorder=None)
QA = QArgs(4, "int", True, "group", 128)
ROWS = 256
TOKENS = 8192
SHAPES = [("q_proj", 4096, 4096), ("k_proj", 1024, 4096), ("gate_proj", 14336, 4096), ("down_proj", 4096, 14336)]


@pytest.fixture(scope="module")
def problems():
    out = {}
    for d in (4096, 14336):
        g = torch.Generator(device="cuda").manual_seed(d)
        x = (torch.randn(TOKENS, d, device="cuda", generator=g)
             * torch.exp(0.5 * torch.randn(d, device="cuda", generator=g))).to(torch.bfloat16)
        H = torch.zeros(d, d, device="cuda")
        gptq.hessian_update_(H, x, 2.0 / TOKENS)
        Hn = H.cpu().numpy()
        U, ok = ogptq.hinv_upper(Hn, 0.01)  # the oracle's factor, once per Hessian
        assert ok
        out[d] = (H, Hn, U, x[:2048].float())
    return out


@pytest.mark.parametrize("name,rows,cols", SHAPES)
def test_c2_shape_against_oracle(problems, name, rows, cols):
    H, Hn, U, xs = problems[cols]
    g = torch.Generator(device="cuda").manual_seed(rows * 7 + cols)
    w = (0.02 * torch.randn(rows, cols, device="cuda", generator=g)).to(torch.bfloat16)
    lin = torch.nn.Linear(cols, rows, bias=False, dtype=torch.bfloat16, device="cuda")
    lin.weight.data.copy_(w)
    inv = gptq.inverse_hessian(H.clone(), 0.01)
    scale, zp, _ = gptq.weight_qparams(lin, ARGS)
    row_loss = torch.empty(rows, dtype=torch.float32, device="cuda")
    wq, _ = gptq.quantize_with_inverse(w, ARGS, inv, scale, zp, row_loss_out=row_loss)
    assert inv.ok()
    ours_loss = float(row_loss[:ROWS].double().sum())
    oloss, owq, oscale, ozp, ok = ogptq.quantize_weight(np_f32(w[:ROWS]), Hn, QA, hinv=U)
    assert ok
    mine = ogptq.codes_from_weight(np_f32(wq[:ROWS]), oscale, ozp, QA)
    theirs = ogptq.codes_from_weight(owq, oscale, ozp, QA)
    agree = float(np.mean(mine == theirs))
    assert agree >= 0.99, (name, agree)
    assert abs(ours_loss - oloss) <= 0.01 * abs(oloss), (name, ours_loss, oloss)
    wf = w[:ROWS].float()
    den = float(torch.sum((wf @ xs.T) ** 2))
    e_ours = float(torch.sum(((wf - wq[:ROWS].float()) @ xs.T) ** 2)) / den
    e_ref = float(torch.sum(((wf - torch.from_numpy(owq).cuda()) @ xs.T) ** 2)) / den
    assert abs(e_ours - e_ref) <= 0.01 * e_ref, (name, e_ours, e_ref)
