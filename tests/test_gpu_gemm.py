"""GPU parity of the float32-accurate tensor-core GEMM (3xTF32), C = A * B^T,
against a float64 product.  Bar: relative error <= 1e-5 (measured ~1e-6)."""
import pytest
import torch

from llmcompressor_b200 import _lib, gptq  # noqa: F401  (gptq registers the signature)

pytestmark = pytest.mark.gpu


def _run(m, n, k, mode, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    A = torch.randn(m, k, device="cuda", generator=g)
    Bt = torch.randn(n, k, device="cuda", generator=g)
    C0 = torch.randn(m, n, device="cuda", generator=g)
    C = C0.clone()
    st = _lib.lib().llmc_gemm_f32_nt(m, n, k, A.data_ptr(), A.stride(0), Bt.data_ptr(), Bt.stride(0), C.data_ptr(),
                                     C.stride(0), mode, torch.cuda.current_stream().cuda_stream)
    assert st == 0, _lib.lib().llmc_status_string(st)
    prod = A.double() @ Bt.double().T
    ref = {0: prod, 1: C0.double() - prod, 2: -prod}[mode]
    torch.cuda.synchronize()
    return float(torch.linalg.norm(C.double() - ref) / torch.linalg.norm(ref))


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("m,n,k", [(256, 384, 128), (300, 200, 96), (1000, 516, 128), (4096, 4096, 128)])
def test_gemm_nt(m, n, k, mode):
    assert _run(m, n, k, mode, seed=m + n + k) <= 1e-5
