"""The compressed-tensors save path with the cast kernels plugged in
(``compressors.register_with_compressed_tensors``): the reference's
``compress_module`` / ``ModelCompressor.compress_model``
(S/transformers/compression/compressed_tensors_utils.py:172-191) must write
the same bytes as compressed-tensors' own torch compressors.

* The reference's own C1 oneshot output (``tests/golden/oneshot_c1.npz``):
  its fake-quantized weights and scales, compressed here, give its
  ``weight_packed`` byte for byte.
* MX scales: ``MXFP4PackedCompressor`` scale encoding equals
  ``compress_mx_scale`` on every input (powers of two or not, subnormal,
  zero).
* Activation-ordered groups (``weight_g_idx``) and a whole model through
  ``ModelCompressor`` equal compressed-tensors' torch path."""
import numpy as np
import pytest
import torch
from compressed_tensors.quantization import QuantizationArgs, QuantizationScheme, initialize_module_for_quantization
from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme

from golden_io import load
from llmcompressor_b200 import compressors, ops
from test_gpu_oneshot import bf16_of, unpack_int4

pytestmark = pytest.mark.gpu


@pytest.fixture
def plugged():
    compressors.register_with_compressed_tensors()
    yield
    compressors.unregister_from_compressed_tensors()


def _module(w: torch.Tensor, scheme) -> torch.nn.Linear:
    lin = torch.nn.Linear(w.shape[1], w.shape[0], bias=False, dtype=w.dtype, device=w.device)
    lin.weight.data.copy_(w)
    initialize_module_for_quantization(lin, scheme, force_zero_point=False)
    return lin


def _ct_compress(module) -> dict:
    from compressed_tensors.compressors import compress_module

    compress_module(module)
    return {k: v.detach() for k, v in module.state_dict().items()}


def test_c1_reference_outputs_compress_byte_exact(plugged):
    ref = load("oneshot_c1")
    scheme = preset_name_to_scheme("W4A16", ["Linear"])
    for n in [str(x) for x in ref["modules"]]:
        packed = ref[f"{n}.weight_packed"]
        cols = int(ref[f"{n}.weight_shape"][1])
        codes = torch.from_numpy(unpack_int4(packed, cols)).float()
        scale = bf16_of(ref[f"{n}.weight_scale"])
        q = (codes * scale.float().repeat_interleave(128, dim=1)).to(torch.bfloat16).cuda()
        mod = _module(q, scheme)
        mod.weight_scale.data.copy_(scale.cuda())
        out = _ct_compress(mod)
        np.testing.assert_array_equal(out["weight_packed"].cpu().numpy(), packed, err_msg=n)
        assert torch.equal(out["weight_scale"].cpu(), scale)
        assert "weight_zero_point" not in out  # symmetric: removed


def test_mx_scale_encoding_matches_compress_mx_scale():
    from compressed_tensors.compressors.mx_utils import compress_mx_scale

    g = torch.Generator(device="cuda").manual_seed(0)
    vals = torch.cat([
        torch.exp2(torch.randint(-140, 120, (256,), device="cuda", generator=g).float()),  # powers of two, subnormals
        torch.rand(256, device="cuda", generator=g) * 10,                                     # arbitrary
        torch.tensor([0.0, 1e-40, 3.0e38, 1.9961], device="cuda"),
    ])
    args = preset_name_to_scheme("MXFP4A16", ["Linear"]).weights
    for dt in (torch.bfloat16, torch.float32):
        s = vals.to(dt)
        ours = compressors.MXFP4PackedCompressor._compress_scale(s, args)
        theirs = compress_mx_scale(s, args.scale_dtype or torch.uint8)
        assert torch.equal(ours, theirs), dt


def test_activation_ordered_groups_match_compressed_tensors():
    args = QuantizationArgs(num_bits=4, type="int", symmetric=False, strategy="group", group_size=128,
                            actorder="group")
    scheme = QuantizationScheme(targets=["Linear"], weights=args)
    g = torch.Generator(device="cuda").manual_seed(1)
    rows, cols = 96, 512
    w = (0.02 * torch.randn(rows, cols, device="cuda", generator=g)).to(torch.bfloat16)
    mn, mx = ops.observe_minmax(w, args)
    scale, zp = ops.calculate_qparams(mn, mx, args)
    perm = torch.randperm(cols, device="cuda", generator=g)
    g_idx = (torch.argsort(perm) // 128).to(torch.int32)  # column -> its group in the permuted order
    outs = []
    for use_kernels in (False, True):
        if use_kernels:
            compressors.register_with_compressed_tensors()
        try:
            mod = _module(w, scheme)
            mod.weight_scale.data.copy_(scale)
            mod.weight_zero_point.data.copy_(zp.to(mod.weight_zero_point.dtype))
            mod.weight_g_idx.data.copy_(g_idx)
            outs.append(_ct_compress(mod))
        finally:
            compressors.unregister_from_compressed_tensors()
    theirs, ours = outs
    assert set(ours) == set(theirs)
    for k in theirs:
        assert torch.equal(ours[k].cpu(), theirs[k].cpu()), k


@pytest.mark.parametrize("scheme_name", ["W4A16", "W8A16", "FP8_DYNAMIC", "NVFP4A16", "W4A16_ASYM"])
def test_model_compressor_matches_compressed_tensors(scheme_name):
    """A small model quantized round-to-nearest by the GPU QuantizationModifier,
    then compressed by ModelCompressor.compress_model with and without the
    kernels plugged in: identical state dicts."""
    from compressed_tensors.compressors import ModelCompressor

    from llmcompressor_b200 import oneshot as O

    def build():
        torch.manual_seed(0)
        m = torch.nn.Sequential(torch.nn.Linear(512, 256, bias=False), torch.nn.Linear(256, 384, bias=False))
        m = m.to(torch.bfloat16).cuda()
        return O.oneshot(m, recipe=O.QuantizationModifier(targets="Linear", scheme=scheme_name))

    outs = []
    for use_kernels in (False, True):
        if use_kernels:
            compressors.register_with_compressed_tensors()
        try:
            m = build()
            mc = ModelCompressor.from_pretrained_model(m)
            mc.compress_model(m)
            outs.append({k: v.detach().cpu() for k, v in m.state_dict().items()})
        finally:
            compressors.unregister_from_compressed_tensors()
    theirs, ours = outs
    assert set(ours) == set(theirs), (sorted(ours), sorted(theirs))
    for k in theirs:
        a, b = ours[k], theirs[k]
        if a.dtype in (torch.float8_e4m3fn,):
            a, b = a.view(torch.uint8), b.view(torch.uint8)
        assert torch.equal(a, b), k
