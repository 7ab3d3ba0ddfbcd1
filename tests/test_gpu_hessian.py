"""GPU parity of the tensor-core Hessian accumulation (through the C ABI).

Bar: relative Frobenius error <= 1e-5 against the
reference's float32 accumulation; bf16 x bf16 products are exact in float32,
so only summation order differs."""
import numpy as np
import pytest
import torch

from golden_io import load
from gpu_util import to_dev_bf16
from llmcompressor_b200 import gptq

pytestmark = pytest.mark.gpu
TOL = 1e-5


def rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.double(), b.double()
    return float(torch.linalg.norm(a - b) / torch.linalg.norm(b))


def test_hessian_golden_fixture():
    g = load("hessian")
    d = g["H"].shape[0]
    lin = torch.nn.Linear(d, 64, bias=False, dtype=torch.bfloat16, device="cuda")
    H = gptq.make_empty_hessian(lin)
    n = torch.zeros((), device="cuda")
    for i in range(3):
        x = to_dev_bf16(g[f"x{i}"]).unsqueeze(0)
        H, n = gptq.accumulate_hessian(x, lin, H, n)
    ref = torch.from_numpy(g["H"]).cuda()
    assert float(n) == float(g["num_samples"])
    assert rel(H, ref) <= TOL
    assert torch.equal(H, H.T)


@pytest.mark.parametrize(
    "d,tokens",
    [(4096, 2048), (1024, 777), (2816, 512), (1000, 300), (336, 64), (4100, 257), (14336, 2048), (8, 5)],
)
def test_hessian_vs_fp64(d, tokens):
    g = torch.Generator(device="cuda").manual_seed(d + tokens)
    x = torch.randn(tokens, d, device="cuda", generator=g).to(torch.bfloat16)
    H = torch.zeros(d, d, device="cuda")
    gptq.hessian_update_(H, x, 2.0)
    xd = x.double()
    ref = 2.0 * xd.T @ xd
    torch.cuda.synchronize()
    assert rel(H, ref) <= TOL, (d, tokens)
    assert torch.equal(H, H.T)


def test_hessian_accumulates_over_calls():
    d = 2048
    g = torch.Generator(device="cuda").manual_seed(1)
    xs = [torch.randn(512, d, device="cuda", generator=g).to(torch.bfloat16) for _ in range(4)]
    H1 = torch.zeros(d, d, device="cuda")
    for x in xs:
        gptq.hessian_update_(H1, x)
    H2 = torch.zeros(d, d, device="cuda")
    gptq.hessian_update_(H2, torch.cat(xs))
    assert rel(H1, H2) <= TOL  # float32 accumulation order differs between 4 calls and 1
    assert rel(H1, 2 * torch.cat(xs).double().T @ torch.cat(xs).double()) <= TOL


def test_hessian_batch_counting_and_dead_columns():
    """num_samples counts the batch dim (2-D input counts one); zero input
    features give exactly zero rows/columns (the dead-column case)."""
    d = 512
    lin = torch.nn.Linear(d, 8, bias=False, dtype=torch.bfloat16, device="cuda")
    H = gptq.make_empty_hessian(lin)
    n = torch.zeros((), device="cuda")
    x = torch.randn(3, 100, d, device="cuda").to(torch.bfloat16)
    x[..., 17] = 0
    H, n = gptq.accumulate_hessian(x, lin, H, n)
    H, n = gptq.accumulate_hessian(x[0], lin, H, n)
    assert float(n) == 4.0
    assert torch.all(H[17] == 0) and torch.all(H[:, 17] == 0)


def test_hessian_empty_input():
    d = 256
    H = torch.zeros(d, d, device="cuda")
    n = torch.zeros((), device="cuda")
    gptq.hessian_update_(H, torch.empty(0, d, dtype=torch.bfloat16, device="cuda"), 2.0, n, 1.0)
    assert torch.count_nonzero(H) == 0 and float(n) == 1.0


def test_accumulate_hessian_long_input_stays_within_bar():
    """A 40000-token input through the drop-in: folded in 2048-token launches,
    H stays within 1e-5 of the exact sum (one 40000-token launch would be
    off by about 1.8e-4: the tensor-core accumulation's bias)."""
    d = 1024
    g = torch.Generator(device="cuda").manual_seed(40)
    x = (torch.randn(1, 40000, d, device="cuda", generator=g) * 0.5).to(torch.bfloat16)
    lin = torch.nn.Linear(d, 8, bias=False, dtype=torch.bfloat16, device="cuda")
    H = gptq.make_empty_hessian(lin)
    n = torch.zeros((), device="cuda")
    H, n = gptq.accumulate_hessian(x, lin, H, n)
    xd = x[0].double()
    assert rel(H, 2.0 * xd.T @ xd) <= TOL
    assert float(n) == 1.0
