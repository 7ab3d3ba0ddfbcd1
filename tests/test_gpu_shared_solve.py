"""Modules that share a Hessian (q/k/v, gate/up) solved together
(``gptq.quantize_modules_shared``: one factorisation, one block-loop call
over their stacked rows) against ``quantize_weight`` per module: GPTQ rows
are independent given the factor, so the weights must be bit-identical and
the per-module losses equal up to float32 summation order."""
import pytest
import torch
from compressed_tensors.quantization import QuantizationArgs

from llmcompressor_b200 import gptq

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("strategy,group,sym", [("group", 128, True), ("channel", None, True), ("group", 64, False)])
def test_stacked_rows_match_per_module(strategy, group, sym):
    g = torch.Generator(device="cuda").manual_seed(3)
    cols = 1024
    qa = QuantizationArgs(num_bits=4, type="int", symmetric=sym, strategy=strategy, group_size=group, actorder=None)
    mods = []
    for rows in (256, 128, 96):
        lin = torch.nn.Linear(cols, rows, bias=False, dtype=torch.bfloat16, device="cuda")
        lin.weight.data.copy_((0.02 * torch.randn(rows, cols, device="cuda", generator=g)).to(torch.bfloat16))
        mods.append(lin)
    x = (torch.randn(4096, cols, device="cuda", generator=g)
         * torch.exp(0.5 * torch.randn(cols, device="cuda", generator=g))).to(torch.bfloat16)
    H = torch.zeros(cols, cols, device="cuda")
    gptq.hessian_update_(H, x, 2.0 / 4096)
    hinv, res = gptq.quantize_modules_shared(mods, qa, H.clone())
    assert hinv.ok()
    for m, (loss, q) in zip(mods, res):
        ref_loss, ref = gptq.quantize_weight(m, qa, H.clone())
        assert torch.equal(q["weight"], ref["weight"])
        assert torch.equal(q["weight_scale"], ref["weight_scale"])
        assert torch.equal(q["weight_zero_point"], ref["weight_zero_point"])
        assert abs(float(loss) - ref_loss) <= 1e-5 * abs(ref_loss), (float(loss), ref_loss)
