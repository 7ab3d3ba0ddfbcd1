"""The no-allocation GPTQ entry point, called through the C ABI.

``llmc_gptq_quantize_noalloc`` serves callers that cannot allocate device
memory -- code recorded under CUDA stream capture, hosts that keep all device
memory to themselves, bare FFI bindings -- by taking its scratch from a fixed
32 MiB array inside the library instead of a caller workspace.  It runs the
same kernels in the same order as the workspace entry point
``llmc_gptq_quantize``, so its output weight and loss must be bit-identical
to that entry point's, on two calls in a row (the second sees the first
call's leftovers in the shared array); weights too large for the array must
be rejected without launching anything.

This file is collected last so that a run stopping at its first failure has
already run every other test.
"""
import ctypes

import pytest
import torch
from compressed_tensors.quantization import QuantizationArgs

from llmcompressor_b200 import _lib, gptq, ops

pytestmark = pytest.mark.gpu

ARGS = QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128, actorder=None)


def _problem(rows, cols, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    w = (0.02 * torch.randn(rows, cols, device="cuda", generator=g)).to(torch.bfloat16)
    x = torch.randn(2048, cols, device="cuda", generator=g).to(torch.bfloat16)
    H = torch.zeros(cols, cols, device="cuda")
    gptq.hessian_update_(H, x, 2.0 / 2048)
    return w, H


def _call_noalloc(w, inv, scale, out, loss):
    qa = _lib.qargs_struct(ARGS)
    rows, cols = w.shape
    return _lib.lib().llmc_gptq_quantize_noalloc(
        w.data_ptr(), rows, cols, inv.hinv.data_ptr(), inv.hinv_t.data_ptr(), inv.dead.data_ptr(), ctypes.byref(qa),
        scale.data_ptr(),
        None, 128, out.data_ptr(), loss.data_ptr(), inv.status.data_ptr(), torch.cuda.current_stream().cuda_stream)


def test_noalloc_matches_workspace_entry_point_on_two_calls():
    import llmcompressor_b200.noalloc  # noqa: F401  (registers the signature)

    for seed, (rows, cols) in [(1, (512, 1024)), (2, (1024, 4096))]:
        w, H = _problem(rows, cols, seed)
        inv = gptq.inverse_hessian(H, 0.01)
        mn, mx = ops.observe_minmax(w, ARGS)
        scale, zp = ops.calculate_qparams(mn, mx, ARGS)
        ref_wq, ref_loss = gptq.quantize_with_inverse(w, ARGS, inv, scale, zp)  # workspace entry point
        out = torch.empty_like(w)
        loss = torch.empty(1, dtype=torch.float32, device="cuda")
        st = _call_noalloc(w, inv, scale, out, loss)
        assert st == _lib.OK, _lib.lib().llmc_status_string(st)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_wq)
        assert torch.equal(loss, ref_loss)


def test_noalloc_python_wrapper_asymmetric_matches_workspace_entry_point():
    from llmcompressor_b200.noalloc import quantize_with_inverse_noalloc

    args = QuantizationArgs(num_bits=4, type="int", symmetric=False, strategy="group", group_size=128,
                            actorder=None)
    for seed in (3, 4):
        w, H = _problem(256, 1024, seed)
        inv = gptq.inverse_hessian(H, 0.01)
        mn, mx = ops.observe_minmax(w, args)
        scale, zp = ops.calculate_qparams(mn, mx, args)
        zp8 = zp.to(torch.int8).contiguous()
        ref_wq, ref_loss = gptq.quantize_with_inverse(w, args, inv, scale, zp)
        out = torch.empty_like(w)
        loss = torch.empty(1, dtype=torch.float32, device="cuda")
        quantize_with_inverse_noalloc(w, args, inv, scale.to(torch.bfloat16).contiguous(), zp8, out, loss)
        torch.cuda.synchronize()
        assert torch.equal(out, ref_wq)
        assert torch.equal(loss, ref_loss)
    # inputs the kernels would misread are refused, not converted
    with pytest.raises(ValueError):
        quantize_with_inverse_noalloc(w, args, inv, scale.float(), zp8, out, loss)
    with pytest.raises(ValueError):
        quantize_with_inverse_noalloc(w, args, inv, scale.to(torch.bfloat16), zp8.to(torch.int32), out, loss)


def test_noalloc_rejects_weights_beyond_the_fixed_scratch():
    qa = _lib.qargs_struct(ARGS)
    st = _lib.lib().llmc_gptq_quantize_noalloc(None, 4096, 4096, None, None, None, ctypes.byref(qa), None, None, 128,
                                               None, None, None, torch.cuda.current_stream().cuda_stream)
    assert st == _lib.EINVAL_SHAPE
