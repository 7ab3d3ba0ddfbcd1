"""CPU oracle for the llm-compressor PTQ hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (scipy for the dense factorisations of the
GPTQ solve), the arithmetic of the reference's post-training-quantization hot
path: min-max observers, ``calculate_qparams``/``generate_gparam``, the
compressed-tensors casts and packers (int4/int8 into int32, FP8 E4M3 per
tensor/channel/128x128 block, NVFP4, MXFP4), GPTQ Hessian accumulation and the
GPTQ block solve.  Each function cites the reference file:line it follows.

It is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` may import it.  The product path
(``llmcompressor_b200``) never imports this package and fails loudly when its
CUDA library is missing.

Parity is pinned: ``tests/golden/make_golden.py`` runs the reference itself
(llm-compressor from its source checkout, compressed-tensors 0.15.0.1 as
installed) on seeded inputs, and ``tests/test_oracle_golden.py`` checks every
oracle function against those fixtures bit for bit (GPTQ: code agreement and
loss, the GPTQ acceptance criteria).

Citation prefixes: ``S/`` = ``src/llmcompressor/`` of the reference,
``CT/`` = the installed ``compressed_tensors`` package (third-party, 0.15.0.1).
"""

from . import numerics, observers, casts, gptq  # noqa: F401
