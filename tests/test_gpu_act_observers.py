"""GPU parity of the activation observers of static activation schemes
(S/observers/min_max.py:16-110) through ``llmc_observe_activation``:
statistics after every batch and the final qparams bit-exact against the
reference's fixtures and the oracle."""
import numpy as np
import pytest
import torch
from compressed_tensors.quantization import QuantizationArgs
from compressed_tensors.quantization.quant_scheme import preset_name_to_scheme

from golden_io import load
from gpu_util import to_dev_bf16
from llmcompressor_b200 import act_observers as ao
from oracle import numerics
from oracle.observers import QArgs, activation_minmax, update_activation_minmax

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16)


CASES = {
    "minmax_int8_tensor": ("minmax", "input", lambda: QuantizationArgs(
        num_bits=8, type="int", symmetric=True, strategy="tensor", dynamic=False, observer="minmax")),
    "static_int8_asym_tensor": ("static_minmax", "input", lambda: QuantizationArgs(
        num_bits=8, type="int", symmetric=False, strategy="tensor", dynamic=False, observer="static_minmax")),
    "minmax_nvfp4_tensor_group": ("minmax", "input",
                                  lambda: preset_name_to_scheme("NVFP4", ["Linear"]).input_activations),
    "memoryless_int8_group128": ("memoryless_minmax", "input", lambda: QuantizationArgs(
        num_bits=8, type="int", symmetric=False, strategy="group", group_size=128, dynamic=False,
        observer="memoryless_minmax")),
    "static_fp8_kv_tensor": ("static_minmax", "k", lambda: QuantizationArgs(
        num_bits=8, type="float", symmetric=True, strategy="tensor", dynamic=False, observer="static_minmax")),
    "minmax_c05_fp8_tensor": ("minmax", "output", lambda: QuantizationArgs(
        num_bits=8, type="float", symmetric=True, strategy="tensor", dynamic=False, observer="minmax",
        observer_kwargs={"averaging_constant": 0.5})),
}


@pytest.mark.parametrize("case", sorted(CASES))
def test_activation_observer_golden(case):
    g = load(f"actobs_{case}")
    name, base, make_args = CASES[case]
    obs = ao.OBSERVERS[name](base, make_args())
    for b in range(4):
        x = to_dev_bf16(g[f"x{b}"])
        assert obs(x) is obs
        np.testing.assert_array_equal(_bits(obs.min_vals), g[f"min{b}"], err_msg=f"min after batch {b}")
        np.testing.assert_array_equal(_bits(obs.max_vals), g[f"max{b}"], err_msg=f"max after batch {b}")
    q = obs.get_qparams()
    assert not obs.has_statistics
    if "global_scale" in g:
        np.testing.assert_array_equal(q["global_scale"].cpu().numpy().reshape(-1), g["global_scale"].reshape(-1))
        np.testing.assert_array_equal(q["scale"].float().cpu().numpy().reshape(-1), g["scale"].reshape(-1))
    else:
        np.testing.assert_array_equal(_bits(q["scale"]).reshape(-1), g["scale"].reshape(-1))
    zp = q["zero_point"]
    if zp.dtype == torch.float8_e4m3fn:
        assert not torch.any(zp.float() != 0)
    else:
        np.testing.assert_array_equal(zp.cpu().numpy().astype(np.int64).reshape(-1),
                                      g["zero_point"].astype(np.int64).reshape(-1))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("kind", ["tensor", "group16", "group256"])
@pytest.mark.parametrize("obs_name", ["minmax", "static_minmax"])
def test_activation_observer_vs_oracle_large(dtype, kind, obs_name):
    """Batches of 4096 x 4096 (every slab and column block of the reduction),
    several observations, both activation dtypes."""
    gen = torch.Generator(device="cuda").manual_seed(5)
    if kind == "tensor":
        args = QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="tensor", dynamic=False)
        qa = QArgs(8, "int", True, "tensor", None)
    else:
        gs = int(kind[5:])
        args = QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="group", group_size=gs,
                                dynamic=False)
        qa = QArgs(8, "int", True, "group", gs)
    obs = ao.OBSERVERS[obs_name]("input", args)
    mn = mx = None
    for b in range(3):
        x = (torch.randn(2, 2048, 4096, device="cuda", generator=gen) * (b + 1)
             * torch.exp(torch.randn(4096, device="cuda", generator=gen))).to(dtype)
        obs(x)
        nmn, nmx = activation_minmax(x.float().cpu().numpy(), qa)
        mn, mx = update_activation_minmax(mn, mx, nmn, nmx, obs_name, 0.01,
                                          dtype="bf16" if dtype == torch.bfloat16 else "f32")
        np.testing.assert_array_equal(obs.min_vals.float().cpu().numpy(), mn)
        np.testing.assert_array_equal(obs.max_vals.float().cpu().numpy(), mx)


def test_minmax_observer_value_update_known_answers():
    """T/llmcompressor/observers/test_min_max.py:48-86 on the GPU (float32
    input of 8 features: the kernel reads whole 8-feature vectors)."""
    args = QuantizationArgs(num_bits=8, strategy="tensor", symmetric=True, observer="minmax")
    obs = ao.MinMaxObserver("input", args)
    base = [1.0] * 8
    seq = [base, base, [127.0] + [1.0] * 7, base, [-128.0] + [1.0] * 7]
    cur_max, cur_min = 1.0, 1.0
    for i, row in enumerate(seq):
        obs(torch.tensor([row], device="cuda"))
        cur_max = max(float(obs.max_vals[0]), cur_max)
        cur_min = min(float(obs.min_vals[0]), cur_min)
        if i < 2:
            assert cur_max == 1 and cur_min == 1
        elif i < 4:
            assert abs(cur_max - 2.26) < 1e-6 and cur_min == 1
        else:
            assert abs(cur_max - 2.26) < 1e-6 and abs(cur_min - (-0.29)) < 1e-6


def test_activation_observer_edges():
    args = QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="tensor", dynamic=False)
    obs = ao.StaticMinMaxObserver("input", args)
    obs(torch.empty(0, 64, device="cuda", dtype=torch.bfloat16))  # an empty batch changes nothing
    assert not obs.has_statistics
    x = torch.randn(3, 64, device="cuda").to(torch.bfloat16)
    obs(x)
    before = (obs.min_vals.clone(), obs.max_vals.clone())
    obs(torch.empty(0, 64, device="cuda", dtype=torch.bfloat16))
    assert torch.equal(obs.min_vals, before[0]) and torch.equal(obs.max_vals, before[1])
    with pytest.raises(AssertionError):
        ao.StaticMinMaxObserver("input", args).get_qparams()
    with pytest.raises(ValueError):
        ao.StaticMinMaxObserver("input", QuantizationArgs(num_bits=8, strategy="channel"))(x)
    with pytest.raises(ValueError):
        ao.StaticMinMaxObserver("weight", args)(x)
    # a fresh observer on memoryless semantics keeps only the last batch
    m = ao.MemorylessMinMaxObserver("input", args)
    m(x * 4)
    m(x)
    assert torch.equal(m.max_vals, x.reshape(-1).max().reshape(1))
    assert torch.equal(m.min_vals, x.reshape(-1).min().reshape(1))
