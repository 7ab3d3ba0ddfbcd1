"""Test-only import shim for the reference llm-compressor (CPU, this container only).

The reference package (``src/llmcompressor`` of the reference checkout) imports
seven names that the installed compressed-tensors 0.15.0.1 does not provide,
plus ``accelerate.accelerator``.  All of them are distributed/IO plumbing; none
is arithmetic.  This module injects small stand-ins into ``sys.modules`` so that
the reference's own numerics (observers, ``calculate_qparams``, fake-quant,
compressors, ``accumulate_hessian``, ``quantize_weight``) can be imported and
run to produce golden fixtures.

It is used only by ``make_golden.py`` in this directory, never by the product,
the GPU tests, ``smoke()`` or ``bench.py`` (the reference checkout does not
exist on the GPU box).
"""
from __future__ import annotations

import os
import sys
import types

# the reference checkout's `src` directory (the fixture generator's input)
REFERENCE_SRC = os.environ.get("LLMC_REFERENCE_SRC", "")


def _stub(name: str, **attrs):
    mod = types.ModuleType(name)
    for k, v in attrs.items():
        setattr(mod, k, v)
    sys.modules[name] = mod
    parent, _, child = name.rpartition(".")
    if parent and parent in sys.modules:
        setattr(sys.modules[parent], child, mod)
    return mod


def _greedy_bin_packing(items, num_bins, item_weight_fn=lambda x: 1):
    items.sort(key=item_weight_fn, reverse=True)
    bins = [[] for _ in range(num_bins)]
    totals = [0] * num_bins
    item_to_bin = {}
    for it in items:
        b = min(range(num_bins), key=lambda i: totals[i])
        bins[b].append(it)
        totals[b] += item_weight_fn(it)
        item_to_bin[it] = b
    return items, bins, item_to_bin


def _wait_for_comms(works):
    for w in works:
        w.wait()
    works.clear()


def install() -> None:
    """Install the stand-ins and put the reference source on ``sys.path``."""
    if "llmcompressor" in sys.modules:
        return
    os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
    import compressed_tensors  # noqa: F401
    import compressed_tensors.offload.dist_utils as du
    import compressed_tensors.utils.safetensors_load as sl
    import compressed_tensors.entrypoints.convert as conv

    _stub(
        "compressed_tensors.distributed",
        greedy_bin_packing=_greedy_bin_packing,
        wait_for_comms=_wait_for_comms,
        as_broadcastable=du.as_broadcastable,
        is_distributed=du.is_distributed,
        is_source_process=lambda: True,
    )
    if not hasattr(du, "is_source_process"):
        du.is_source_process = lambda: True
    for n in (
        "InverseWeightMap",
        "find_safetensors_index_file",
        "get_weight_map",
        "load_tensors_from_inverse_weight_map",
    ):
        if not hasattr(sl, n):
            setattr(sl, n, dict if n == "InverseWeightMap" else (lambda *a, **k: None))
    if not hasattr(conv, "build_inverse_weight_maps"):
        conv.build_inverse_weight_maps = lambda *a, **k: None
    if "accelerate" not in sys.modules:
        _stub("accelerate")
        _stub("accelerate.accelerator", get_state_dict_offloaded_model=lambda m: m.state_dict())
    if not REFERENCE_SRC or not os.path.isdir(REFERENCE_SRC):
        raise RuntimeError("set LLMC_REFERENCE_SRC to the `src` directory of a reference llm-compressor checkout")
    if REFERENCE_SRC not in sys.path:
        sys.path.insert(0, REFERENCE_SRC)
