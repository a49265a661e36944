"""Dense fp16/bf16 GEMM with split-K -- drop-in for pico-kernels'
``gemm_splitk`` (gemm_splitk.py) and ``gemm`` (gemm.py) modules.

* ``triton_gemm_splitk(a, b, split_k=4, BLOCK_M, BLOCK_N, BLOCK_K) -> fp32``
  gemm_splitk.py:67-80. The reference adds fp32 partials with atomics into a
  zeroed C (order-dependent); here each K slice writes its partial tile and
  the last slice to finish sums them in slice order, so results are
  deterministic run to run.
* ``triton_gemm(a, b) -> fp32`` (gemm.py:103-128): the same kernel without a
  K split. Any M, N; K and N multiples of 8 (16-byte rows).

The names keep the reference's ``triton_`` prefix so callers drop in; the
kernels are hand-written sm_100a CUDA (tcgen05), not Triton.
"""

from __future__ import annotations

import torch

from . import _lib

__all__ = ["triton_gemm_splitk", "triton_gemm"]


def _gemm(a: torch.Tensor, b: torch.Tensor, split_k: int) -> torch.Tensor:
    _lib.require_cuda(a, b)
    if a.dtype != b.dtype or a.dtype not in (torch.float16, torch.bfloat16):
        raise _lib.DtypeError(f"a and b must both be fp16 or bf16 (got {a.dtype}, {b.dtype})")
    if a.dim() != 2 or b.dim() != 2:
        raise _lib.ShapeError("a and b must be 2-D")
    M, K = a.shape
    K2, N = b.shape
    if K != K2:
        raise _lib.ShapeError(f"inner dims must match ({K} vs {K2})")
    a = a.contiguous()
    b = b.contiguous()
    lib = _lib.load()
    c = torch.empty((M, N), dtype=torch.float32, device=a.device)
    ws_bytes = lib.pk_gemm_splitk_workspace_size(M, N, K, split_k)
    ws = _lib.workspace(a.device, ws_bytes, tag="dense_splitk")
    _lib.check(lib.pk_gemm_splitk(a.data_ptr(), b.data_ptr(), _lib.dtype_code(a.dtype), M, N, K,
                                  split_k, c.data_ptr(), _lib.ptr(ws), ws_bytes,
                                  _lib.stream_of(a)), "gemm")
    return c


def triton_gemm_splitk(a: torch.Tensor, b: torch.Tensor, split_k: int = 4,
                       BLOCK_M: int = 128, BLOCK_N: int = 128, BLOCK_K: int = 64) -> torch.Tensor:
    """``a @ b`` in fp32 with the K reduction split ``split_k`` ways."""
    del BLOCK_M, BLOCK_N, BLOCK_K  # tile shape is fixed by the tcgen05 kernel
    if split_k < 1:
        raise _lib.ShapeError("split_k must be >= 1")
    return _gemm(a, b, split_k)


def triton_gemm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """``a @ b`` in fp32 (no K split)."""
    return _gemm(a, b, 1)
