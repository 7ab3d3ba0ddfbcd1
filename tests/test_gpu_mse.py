"""GPU parity of the MSE grid-search weight observer (``memoryless_mse``,
S/observers/mse.py:12-45 -> S/observers/mse_quant.py:19-141) through the C ABI.

Bar: the chosen (min, max) and the resulting qparams bit-exact against the
fixtures made by the reference itself and against the CPU oracle on larger
seeded weights."""
import numpy as np
import pytest
import torch
from compressed_tensors.quantization import QuantizationArgs

from golden_io import load
from gpu_util import bits, np_f32, rand_bf16, to_dev_bf16
from llmcompressor_b200 import ops
from oracle import numerics as onum
from oracle import observers as oobs

pytestmark = pytest.mark.gpu

CASES = {
    "int4_sym_group128": (QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128),
                          oobs.QArgs(4, "int", True, "group", 128)),
    "int4_asym_group128": (QuantizationArgs(num_bits=4, type="int", symmetric=False, strategy="group",
                                            group_size=128), oobs.QArgs(4, "int", False, "group", 128)),
    "int8_sym_channel": (QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="channel"),
                         oobs.QArgs(8, "int", True, "channel", None)),
    "int8_asym_channel": (QuantizationArgs(num_bits=8, type="int", symmetric=False, strategy="channel"),
                          oobs.QArgs(8, "int", False, "channel", None)),
    "int4_sym_tensor": (QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="tensor"),
                        oobs.QArgs(4, "int", True, "tensor", None)),
    "fp8_block_128": (QuantizationArgs(num_bits=8, type="float", symmetric=True, strategy="block",
                                       block_structure=[128, 128]),
                      oobs.QArgs(8, "float", True, "block", None, (128, 128), zp_dtype="fp8")),
    "int4_sym_group32": (QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=32),
                         oobs.QArgs(4, "int", True, "group", 32)),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_mse_golden_bit_exact(case):
    g = load(f"mse_{case}")
    args, _ = CASES[case]
    w = to_dev_bf16(g["weight"])
    mn, mx = ops.observe_mse(w, args)
    np.testing.assert_array_equal(bits(mn).reshape(g["min_vals"].shape), g["min_vals"])
    np.testing.assert_array_equal(bits(mx).reshape(g["max_vals"].shape), g["max_vals"])
    scale, zp = ops.calculate_qparams(mn, mx, args)
    np.testing.assert_array_equal(bits(scale).reshape(g["scale"].shape), g["scale"])


@pytest.mark.parametrize("case,rows,cols", [("int4_sym_group128", 512, 4096), ("int4_asym_group128", 256, 2048),
                                            ("int8_sym_channel", 64, 14336), ("fp8_block_128", 300, 1000),
                                            ("int4_sym_group32", 128, 1024)])
def test_mse_vs_oracle(case, rows, cols):
    args, qa = CASES[case]
    wt = rand_bf16(rows, cols, seed=rows + cols, kind="student_t")
    mn, mx = ops.observe_mse(wt.cuda(), args)
    omn, omx = oobs.mse_minmax(np_f32(wt), qa)
    np.testing.assert_array_equal(bits(mn).reshape(omn.shape), onum.f32_to_bf16_bits(omn))
    np.testing.assert_array_equal(bits(mx).reshape(omx.shape), onum.f32_to_bf16_bits(omx))


def test_mse_observer_object_and_knobs():
    """The observer mirror reads observer_kwargs; get_qparams drops the statistics."""
    args = QuantizationArgs(num_bits=4, type="int", symmetric=True, strategy="group", group_size=128,
                            observer="memoryless_mse", observer_kwargs={"maxshrink": 0.5, "patience": 3,
                                                                        "grid": 50.0, "norm": 2.0})
    w = rand_bf16(64, 1024, seed=2, kind="student_t")
    obs = ops.MemorylessMSEObserver(args)
    qp = obs(w.cuda()).get_qparams()
    assert obs.min_vals is None
    qa = oobs.QArgs(4, "int", True, "group", 128)
    omn, omx = oobs.mse_minmax(np_f32(w), qa, maxshrink=0.5, patience=3, grid=50.0, norm=2.0)
    osc, _ = oobs.calculate_qparams(omn, omx, qa)
    np.testing.assert_array_equal(bits(qp["scale"]).reshape(osc.shape), onum.f32_to_bf16_bits(osc))
    with pytest.raises(AssertionError):
        obs.get_qparams()


@pytest.mark.parametrize("case", ["int4_sym_group128", "int8_sym_channel", "int4_sym_tensor", "fp8_block_128"])
def test_grid_search_view_dropin(case):
    """The drop-in for _grid_search_mse takes the reference's flattened weight views."""
    g = load(f"mse_{case}")
    args, qa = CASES[case]
    w = to_dev_bf16(g["weight"])
    r, c = w.shape
    s = getattr(args.strategy, "value", args.strategy)
    if s == "group":
        view = w.reshape(1, r, c // args.group_size, args.group_size)
    elif s == "channel":
        view = w.reshape(1, r, 1, c)
    elif s == "tensor":
        view = w.reshape(1, 1, r * c)
    else:
        bh, bw = args.block_structure
        pr, pc = -(-r // bh) * bh, -(-c // bw) * bw
        p = torch.zeros(pr, pc, dtype=w.dtype, device=w.device)
        p[:r, :c] = w
        view = p.reshape(pr // bh, bh, pc // bw, bw).transpose(1, 2).reshape(1, pr // bh, pc // bw, bh * bw)
    mn, mx = ops.grid_search_mse(view, args)
    np.testing.assert_array_equal(bits(mn).reshape(g["min_vals"].shape), g["min_vals"])
    np.testing.assert_array_equal(bits(mx).reshape(g["max_vals"].shape), g["max_vals"])
