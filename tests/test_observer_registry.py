"""The reference's observer registry routed to the GPU activation observers
(``act_observers.register_with_llmcompressor``): ``Observer.load_from_registry``
returns a subclass of the reference's own class (so ``initialize_observer``
attaches it unchanged), weight observations and CPU tensors keep the
reference's path, and unregistering restores the registry.  Runs where the
reference package can be imported (``LLMC_REFERENCE_SRC`` names its ``src``
directory, as for the fixture generator); skipped elsewhere."""
import os
import sys

import pytest
import torch

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def ref_observer():
    src = os.environ.get("LLMC_REFERENCE_SRC", "")
    if not src or not os.path.isdir(src):
        pytest.skip("reference package not available (set LLMC_REFERENCE_SRC)")
    sys.path.insert(0, HERE)
    import ref_shim

    ref_shim.install()
    from llmcompressor.observers.base import Observer

    return Observer


def test_registry_routes_activation_observers(ref_observer):
    from compressed_tensors.quantization import QuantizationArgs

    from llmcompressor_b200 import act_observers

    Observer = ref_observer
    args = QuantizationArgs(num_bits=8, type="int", symmetric=True, strategy="tensor", dynamic=False,
                            observer="static_minmax")
    before = type(Observer.load_from_registry("static_minmax", base_name="input", args=args))
    names = act_observers.register_with_llmcompressor()
    try:
        assert names == ["memoryless_minmax", "minmax", "static_minmax"]
        obs = Observer.load_from_registry("static_minmax", base_name="input", args=args)
        assert isinstance(obs, before) and type(obs) is not before
        assert isinstance(obs, torch.nn.Module)
        # CPU activations keep the reference's arithmetic
        x = torch.randn(2, 16, 64).to(torch.bfloat16)
        ref = before(base_name="input", args=args)
        obs(x)
        ref(x)
        assert torch.equal(obs.min_vals, ref.min_vals) and torch.equal(obs.max_vals, ref.max_vals)
        # registering twice is harmless
        assert act_observers.register_with_llmcompressor() == names
    finally:
        act_observers.unregister_from_llmcompressor()
    assert type(Observer.load_from_registry("static_minmax", base_name="input", args=args)) is before
