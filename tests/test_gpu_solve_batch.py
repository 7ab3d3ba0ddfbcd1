"""The batched GPTQ solve (``llmc_gptq_solve_batch``: many Hessians of one
size, one weight each -- the experts' down projections of an MoE layer)
against the one-module path on the same inputs: the same kernels in the same
order per expert, so the quantized weights, scales and losses are
bit-identical; a non-positive-definite expert falls back alone."""
import pytest
import torch
from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme

from llmcompressor_b200 import gptq

pytestmark = pytest.mark.gpu


def _lin(w):
    m = torch.nn.Linear(w.shape[1], w.shape[0], bias=False, device="cuda", dtype=torch.bfloat16)
    m.weight.data.copy_(w)
    return m


def _hessian(d, n, g):
    x = torch.randn(n, d, device="cuda", generator=g)
    return (2.0 / n) * (x.T @ x)


@pytest.mark.parametrize("scheme,rows,d,E", [("W4A16", 96, 256, 5), ("W4A16_ASYM", 64, 384, 3),
                                             ("W8A16", 128, 256, 4)])
def test_batched_equals_per_module(scheme, rows, d, E):
    qa = preset_name_to_scheme(scheme, ["Linear"]).weights
    g = torch.Generator(device="cuda").manual_seed(rows + d + E)
    mods = [_lin((0.02 * torch.randn(rows, d, device="cuda", generator=g)).to(torch.bfloat16)) for _ in range(E)]
    Hs = [_hessian(d, 512, g) for _ in range(E)]
    assert gptq.batchable(mods, [qa] * E, [None] * E)
    status, res = gptq.quantize_batched(mods, qa, torch.cat(Hs).contiguous(), 128, 0.01)
    for e in range(E):
        hinv, [(loss, q)] = gptq.quantize_modules_shared([mods[e]], qa, Hs[e].clone(), 128, 0.01)
        assert gptq.BatchStatus(status, e).ok() and hinv.ok()
        b_loss, bq = res[e]
        assert torch.equal(bq["weight"], q["weight"]), e
        assert torch.equal(bq["weight_scale"], q["weight_scale"]), e
        assert torch.equal(bq["weight_zero_point"], q["weight_zero_point"]), e
        assert torch.equal(b_loss, loss), e


def test_one_expert_not_positive_definite():
    qa = preset_name_to_scheme("W4A16", ["Linear"]).weights
    g = torch.Generator(device="cuda").manual_seed(7)
    E, rows, d = 3, 64, 256
    mods = [_lin((0.02 * torch.randn(rows, d, device="cuda", generator=g)).to(torch.bfloat16)) for _ in range(E)]
    Hs = [_hessian(d, 512, g) for _ in range(E)]
    Hs[1] = -torch.eye(d, device="cuda")  # negative definite, no dead columns: the factorisation fails
    status, res = gptq.quantize_batched(mods, qa, torch.cat(Hs).contiguous(), 128, 0.01)
    assert [gptq.BatchStatus(status, e).ok() for e in range(E)] == [True, False, True]
    hinv, [(_, q)] = gptq.quantize_modules_shared([mods[1]], qa, Hs[1].clone(), 128, 0.01)
    assert not hinv.ok()
    assert torch.equal(res[1][1]["weight"], q["weight"])  # the same round-to-nearest fallback
