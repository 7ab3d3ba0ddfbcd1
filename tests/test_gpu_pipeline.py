"""GPU parity of the layer-level pipeline (one decoder layer of the reference's
sequential GPTQ pipeline: Hessians from the hooks, solve, int4 pack).

``solve_layer`` runs the factorisations and block loops of a layer
concurrently on side streams; its packed tensors and scales must be
bit-identical to the same modules solved one at a time through the module
API, and its codes must agree with the CPU oracle at the GPTQ bar."""
import numpy as np
import pytest
import torch
from compressed_tensors.quantization import QuantizationArgs

from gpu_util import bits, np_f32
from llmcompressor_b200 import _lib, gptq, ops
from llmcompressor_b200.pipeline import LayerHessians, input_dims, llama_layer_specs, solve_layer
from oracle import casts as ocasts
from oracle import gptq as ogptq
from oracle.observers import QArgs

pytestmark = pytest.mark.gpu
CODE_AGREE = 0.99
REL = 0.01

QA = QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128, actorder=None)
OQA = QArgs(4, "int", True, "group", 128)


def _layer(seed, hidden=512, intermediate=1024, heads=8, kv_heads=2, head_dim=64, tokens=2048, samples=16):
    specs = llama_layer_specs(hidden, intermediate, heads, kv_heads, head_dim)
    dims = input_dims(specs)
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = {s.name: (0.02 * torch.randn(s.out_features, s.in_features, device="cuda", generator=g)).to(torch.bfloat16)
         for s in specs}
    x = {k: (torch.randn(tokens, d, device="cuda", generator=g)
             * torch.exp(0.5 * torch.randn(d, device="cuda", generator=g))).to(torch.bfloat16)
         for k, d in dims.items()}
    hess = LayerHessians(dims, torch.device("cuda"))
    alpha = 2.0 / samples
    for k in dims:
        for c in range(0, tokens, 512):
            hess.accumulate(k, x[k][c:c + 512], alpha)
    return specs, dims, w, x, hess, alpha


def _sequential(specs, w, H):
    out = {}
    inv = {k: gptq.inverse_hessian(h.clone(), 0.01) for k, h in H.items()}
    for s in specs:
        mn, mx = ops.observe_minmax(w[s.name], QA)
        scale, zp = ops.calculate_qparams(mn, mx, QA)
        wq, loss = gptq.quantize_with_inverse(w[s.name], QA, inv[s.input_key], scale, zp)
        out[s.name] = (ops.quantize_pack(wq, QA, scale, None, fmt=_lib.FMT_PACK_INT32), scale, loss)
    return out


@pytest.mark.parametrize("seed", [0, 1])
def test_solve_layer_matches_module_api(seed):
    specs, dims, w, x, hess, _ = _layer(seed)
    H = {k: h.clone() for k, h in hess.H.items()}
    ref = _sequential(specs, w, H)
    res = solve_layer(w, specs, hess, QA)
    torch.cuda.synchronize()
    assert set(res) == {s.name for s in specs}
    for s in specs:
        r = res[s.name]
        p, sc, loss = ref[s.name]
        assert r.rows == (0, s.out_features)
        np.testing.assert_array_equal(bits(r.weight_packed), bits(p), err_msg=s.name)
        np.testing.assert_array_equal(bits(r.weight_scale), bits(sc), err_msg=s.name)
        assert float(r.loss.reshape(())) == float(loss.reshape(())), s.name


def test_solve_layer_on_side_stream_caller():
    """Results are ordered on the caller's stream, whatever stream that is."""
    specs, dims, w, x, hess, _ = _layer(3, hidden=256, intermediate=512, heads=4, kv_heads=2, head_dim=64)
    H = {k: h.clone() for k, h in hess.H.items()}
    torch.cuda.synchronize()
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        res = solve_layer(w, specs, hess, QA)
        packed = {k: r.weight_packed.clone() for k, r in res.items()}
    st.synchronize()
    ref = _sequential(specs, w, H)
    torch.cuda.synchronize()
    for s in specs:
        np.testing.assert_array_equal(bits(packed[s.name]), bits(ref[s.name][0]), err_msg=s.name)


def test_solve_layer_vs_oracle():
    specs, dims, w, x, hess, alpha = _layer(5, hidden=256, intermediate=512, heads=4, kv_heads=2, head_dim=64,
                                            tokens=1024)
    res = solve_layer(w, specs, hess, QA)
    torch.cuda.synchronize()
    for s in specs:
        xs = np_f32(x[s.input_key])
        Ho = np.zeros((s.in_features, s.in_features), np.float32)
        Ho += (alpha * (xs.T.astype(np.float64) @ xs)).astype(np.float32)
        wo = np_f32(w[s.name])
        loss_o, wq_o, scale_o, zp_o, ok = ogptq.quantize_weight(wo, Ho, OQA)
        assert ok
        codes_o = ogptq.codes_from_weight(wq_o, scale_o, zp_o, OQA)
        packed_o = ocasts.pack_to_int32(codes_o, 4)
        got = bits(res[s.name].weight_packed)
        assert got.shape == packed_o.shape
        # unpack both to codes and compare element-wise
        sh = np.arange(8, dtype=np.uint32) * 4
        c_got = ((got.view(np.uint32)[..., None] >> sh) & 0xF).reshape(got.shape[0], -1)
        c_ref = ((packed_o.view(np.uint32)[..., None] >> sh) & 0xF).reshape(got.shape[0], -1)
        agree = float(np.mean(c_got == c_ref))
        assert agree >= CODE_AGREE, (s.name, agree)
        lg, lo = float(res[s.name].loss.reshape(())), float(loss_o)
        assert abs(lg - lo) <= REL * abs(lo), (s.name, lg, lo)


def test_solve_layer_weight_ordering_matches_module_api():
    """Activation ordering WEIGHT (the reference's default STATIC) through the
    layer solve: bit-identical to the drop-in quantize_weight per module,
    whose parity with the reference is pinned by its own fixtures."""
    from compressed_tensors.quantization import ActivationOrdering

    qa = QA.model_copy()
    qa.actorder = ActivationOrdering.WEIGHT
    specs, dims, w, x, hess, _ = _layer(7, hidden=256, intermediate=512, heads=4, kv_heads=2, head_dim=64)
    H = {k: h.clone() for k, h in hess.H.items()}
    res = solve_layer(w, specs, hess, qa)
    torch.cuda.synchronize()
    for s in specs:
        lin = torch.nn.Linear(s.in_features, s.out_features, bias=False, dtype=torch.bfloat16, device="cuda")
        lin.weight.data.copy_(w[s.name])
        loss, qd = gptq.quantize_weight(lin, qa, H[s.input_key].clone())
        packed = ops.quantize_pack(qd["weight"], qa, qd["weight_scale"], None, fmt=_lib.FMT_PACK_INT32)
        np.testing.assert_array_equal(bits(res[s.name].weight_packed), bits(packed), err_msg=s.name)
        np.testing.assert_array_equal(bits(res[s.name].weight_scale), bits(qd["weight_scale"]), err_msg=s.name)
        assert float(res[s.name].loss.reshape(())) == loss, s.name
