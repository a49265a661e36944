"""B200 (sm_100a) quantized-matmul path: a drop-in for pico-kernels'
``gemm_int4``, ``gemm_fp8``, ``gemm_splitk``, ``gemm`` and ``quantize``
(round-to-nearest, and a GPTQ producer of packed int4 weights).

The kernels live in ``libpico_b200.so`` (hand-written CUDA, C ABI in
``include/pico_b200.h``); these modules are thin PyTorch-facing wrappers.
"""

from . import gemm, gemm_fp8, gemm_int4, gemm_splitk, gptq, linear, quantize  # noqa: F401
from ._lib import (DtypeError, KernelError, ShapeError, device_status, load,  # noqa: F401
                   reset_workspaces, set_wait_limit)
from .gemm_fp8 import fp8_gemm, fp8_gemm_precast  # noqa: F401
from .gemm_splitk import triton_gemm, triton_gemm_splitk  # noqa: F401
from .gemm_int4 import (int4_gemm, int4_gemm_host, pack_int4_n, quantize_int4,  # noqa: F401
                        quantize_int4_grouped, unpack_int4_n)
from .gptq import gptq_quantize_int4  # noqa: F401
from .linear import W4A16Linear, quantize_linear_layers  # noqa: F401

__version__ = "0.1.0"
