"""gptq.BatchedHessian and the per-call drop-in ``accumulate_hessian``
(S/modifiers/gptq/gptq_quantize.py:63-97) on the same calls: both within the
Hessian bar of the exact sum (relative Frobenius error <= 1e-5) and the same
sample count, for call sizes below, across and above the buffer."""
import pytest
import torch

from llmcompressor_b200 import gptq

pytestmark = pytest.mark.gpu
REL = 1e-5


def _calls(d, gen):
    shapes = [(1, 2048, d), (1, 2048, d), (1000, d), (2, 1500, d), (1, 2048, d), (1, 40000, d), (3, 700, d),
              (2048, d)]
    return [(torch.randn(*s, device="cuda", generator=gen) * 0.5).to(torch.bfloat16) for s in shapes]


@pytest.mark.parametrize("d,chunk", [(1024, 2048), (512, 1024), (2048, 2000)])
def test_batched_hessian_matches_per_call(d, chunk):
    gen = torch.Generator(device="cuda").manual_seed(d)
    calls = _calls(d, gen)
    lin = torch.nn.Linear(d, 16, bias=False, dtype=torch.bfloat16, device="cuda")
    H = gptq.make_empty_hessian(lin)
    n = torch.zeros((), device="cuda")
    bh = gptq.BatchedHessian(d, "cuda", chunk_tokens=chunk)
    for x in calls:
        H, n = gptq.accumulate_hessian(x, lin, H, n)
        bh.add(x)
    Hb, nb = bh.finalize()
    torch.cuda.synchronize()
    assert float(nb) == float(n)
    # both are float32 sums in different orders: each is held to the bar
    # against the exact (float64) sum
    exact = torch.zeros(d, d, dtype=torch.float64, device="cuda")
    for x in calls:
        xd = x.reshape(-1, d).double()
        exact += 2.0 * xd.T @ xd
    rel_b = float(torch.linalg.norm(Hb.double() - exact) / torch.linalg.norm(exact))
    rel_p = float(torch.linalg.norm(H.double() - exact) / torch.linalg.norm(exact))
    assert rel_b <= REL, (rel_b, rel_p)
    assert rel_p <= REL, (rel_b, rel_p)
    # finalize leaves nothing pending; a second one changes nothing
    H2, _ = bh.finalize()
    assert torch.equal(H2, Hb)


def test_batched_hessian_into_caller_h():
    d = 768
    gen = torch.Generator(device="cuda").manual_seed(1)
    H = torch.zeros(d, d, device="cuda")
    x = (torch.randn(1, 5000, d, device="cuda", generator=gen)).to(torch.bfloat16)
    bh = gptq.BatchedHessian(d, "cuda", chunk_tokens=2048, H=H)
    bh.add(x)
    bh.flush()
    ref = (2.0 * x[0].double().T @ x[0].double()).float()
    assert bh.H is H
    rel = float(torch.linalg.norm(H - ref) / torch.linalg.norm(ref))
    assert rel <= REL, rel
    with pytest.raises(ValueError):
        bh.add(torch.zeros(1, 10, d + 8, device="cuda", dtype=torch.bfloat16))


@pytest.mark.parametrize("d,chunk", [(4096, 16384), (4096, 65536), (14336, 16384), (14336, 65536)])
def test_batched_hessian_long_chunks_within_bar(d, chunk):
    """The layer pipeline's launch sizes (16384-token default chunk, and
    65536): within 1e-5 of the exact sum."""
    gen = torch.Generator(device="cuda").manual_seed(d + chunk)
    scale = torch.exp(0.5 * torch.randn(d, device="cuda", generator=gen))
    xs = [(torch.randn(1, n, d, device="cuda", generator=gen) * scale).to(torch.bfloat16)
          for n in (chunk - 1000, 2048, 1000 + chunk // 2)]
    bh = gptq.BatchedHessian(d, "cuda", chunk_tokens=chunk)
    for x in xs:
        bh.add(x)
    Hb, nb = bh.finalize()
    exact = torch.zeros(d, d, dtype=torch.float64, device="cuda")
    for x in xs:
        xd = x.reshape(-1, d).double()
        exact += 2.0 * xd.T @ xd
        del xd
    r = float(torch.linalg.norm(Hb.double() - exact) / torch.linalg.norm(exact))
    assert r <= REL, r
    assert float(nb) == len(xs)


def test_gptq_from_16384_token_launches_meets_gptq_bar():
    """The layer API's launch size at a realistic token count: GPTQ from H
    accumulated in 16384-token launches against GPTQ from the exact sum
    (float64, rounded to float32) -- codes >= 99% identical, loss within 1%."""
    from compressed_tensors.quantization import QuantizationArgs

    from llmcompressor_b200 import ops

    d, rows, tokens = 2048, 512, 65536
    gen = torch.Generator(device="cuda").manual_seed(7)
    x = (torch.randn(tokens, d, device="cuda", generator=gen)
         * torch.exp(0.5 * torch.randn(d, device="cuda", generator=gen))).to(torch.bfloat16)
    w = (0.02 * torch.randn(rows, d, device="cuda", generator=gen)).to(torch.bfloat16)
    bh = gptq.BatchedHessian(d, "cuda")
    bh.add(x.unsqueeze(0))
    Hb, _ = bh.finalize()
    xd = x.double()
    He = (2.0 * xd.T @ xd).float()
    qa = QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128, actorder=None)
    mn, mx = ops.observe_minmax(w, qa)
    scale, zp = ops.calculate_qparams(mn, mx, qa)
    out = {}
    for name, H in (("batched", Hb), ("exact", He)):
        inv = gptq.inverse_hessian(H.clone() / tokens, 0.01)
        wq, loss = gptq.quantize_with_inverse(w, qa, inv, scale, zp)
        codes = torch.round(wq.float() / scale.float().repeat_interleave(128, dim=1))
        out[name] = (codes, float(loss))
    agree = float((out["batched"][0] == out["exact"][0]).float().mean())
    assert agree >= 0.99, agree
    lb, le = out["batched"][1], out["exact"][1]
    assert abs(lb - le) <= 0.01 * abs(le), (lb, le)
