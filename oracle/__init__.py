"""CPU oracle for the quantized-matmul path (test infrastructure only).

This package is the checker, never the product: only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) may import it. The CUDA path in ``pico_kernels_b200``
never calls into it and fails loudly when its extension is missing.

Parity is pinned: ``tests/golden/make_golden.py`` ran the reference's own
functions (``quantize.quantize_col``, ``quantize.gptq_layer``,
``gemm_int4.quantize_int4``, ``gemm_int4.pack_int4_n``, ``gemm_fp8.quantize``)
on seeded inputs and committed their outputs; ``tests/test_oracle_golden.py``
checks this oracle against them bit for bit.
"""

from .quant_ref import *  # noqa: F401,F403
