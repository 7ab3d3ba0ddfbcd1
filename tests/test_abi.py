"""CPU checks of the C-ABI boundary: the library loads and exports every
entry point include/llmc_b200.h declares.  No kernel is launched."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in sorted(os.listdir(os.path.join(ROOT, "include"))) if f.endswith(".h")]


def declared_symbols():
    names = set()
    for h in HEADERS:
        src = open(h).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(llmc_\w+)\s*\(", src, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "llmc_version" in syms and "llmc_modelfree_quantize" in syms
    assert len(syms) >= 9


def test_library_loads_and_exports_every_declared_symbol():
    from llmcompressor_b200 import _lib

    lib = _lib.lib()
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_every_declared_symbol_has_a_python_signature():
    from llmcompressor_b200 import _lib

    import llmcompressor_b200  # noqa: F401  (submodules register their signatures)

    _lib.lib()
    missing = [s for s in declared_symbols() if s not in _lib._SIGS]
    assert not missing, missing


def test_version_and_status_strings_without_gpu():
    from llmcompressor_b200 import _lib

    lib = _lib.lib()
    assert lib.llmc_version() >= 100
    assert lib.llmc_status_string(0) == b"ok"
    assert b"positive definite" in lib.llmc_status_string(3)


def test_status_mapping_to_reference_exceptions():
    from llmcompressor_b200 import _lib

    with pytest.raises(ValueError):
        _lib.check(_lib.EINVAL_SHAPE)
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.ENOSUPPORT)
    with pytest.raises(_lib.NotPositiveDefinite):
        _lib.check(_lib.ENOT_PD)


def test_product_path_refuses_cpu_tensors():
    import torch

    from llmcompressor_b200 import ops
    from compressed_tensors.quantization import QuantizationArgs

    w = torch.zeros(8, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.observe_minmax(w, QuantizationArgs(num_bits=4, type="int", strategy="group", group_size=128))
