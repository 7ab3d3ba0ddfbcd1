"""B200-native (sm_100a) kernels behind llm-compressor's PTQ hot-path API.

The host side mirrors the reference's Python interfaces (``accumulate_hessian``,
``quantize_weight``, the observer registry, the compressed-tensors compressors,
``model_free_ptq``); the arithmetic runs in ``libllmc_b200.so`` (C ABI in
``include/llmc_b200.h``).  There is no CPU fallback: without the library or a
CUDA device the entry points raise.
"""
from . import _lib, ops, gptq  # noqa: F401
from . import act_observers, layer_forward, noalloc  # noqa: F401  (each registers its entry points)

__version__ = "0.1.0"
