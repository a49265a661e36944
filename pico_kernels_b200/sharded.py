"""N-sharded quantized linear layers across the GPUs of one node.

For the Llama-70B-shaped layers (up_proj K=8192, N=28672; down_proj K=28672,
N=8192) each of the p ranks (one process per GPU, ``torch.distributed`` over
NCCL / NVLink) holds a contiguous slice of the output columns: packed int4
weights ``[K, N/(2p)]`` with their group scales ``[K/g, N/p]``, or an e4m3
``[K, N/p]`` slice for the fp8 variant. Every rank computes its ``[M, N/p]``
block with the local kernel, then one ``all_gather_into_tensor`` assembles
``[M, N]`` on every rank. Columns are independent, so this is the only
exchange; for M = 1 the gathered buffer already is the row-major output, for
M > 1 the rank-major blocks are interleaved back into rows.

fp8 scales are per tensor and must be global: callers quantize the whole
activation and weight (or all-reduce the absmax) before slicing, so every
rank's ``out_scale`` equals the unsharded one.

The reference has no multi-GPU path; this is the sharding BASELINE.json's
Llama-70B configuration asks for.
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import gemm_fp8, gemm_int4

__all__ = ["shard_columns", "shard_int4", "gather_columns", "sharded_int4_gemm",
           "sharded_fp8_gemm"]


def shard_columns(n: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """Column range [n0, n1) of ``rank``'s contiguous slice of ``n`` columns."""
    if n % world or (n // world) % align:
        raise ValueError(f"N={n} does not split into {world} slices of a multiple of {align}")
    per = n // world
    return rank * per, (rank + 1) * per


def shard_int4(packed: torch.Tensor, scales: torch.Tensor, world: int, rank: int
               ) -> tuple[torch.Tensor, torch.Tensor]:
    """This rank's packed-weight and scale slices (contiguous copies)."""
    n = scales.shape[1]
    n0, n1 = shard_columns(n, world, rank)
    return packed[:, n0 // 2:n1 // 2].contiguous(), scales[:, n0:n1].contiguous()


def gather_columns(local: torch.Tensor, world: int,
                   group: Optional[dist.ProcessGroup] = None,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """All-gather rank-major column blocks ``[M, N/p]`` into ``[M, N]``."""
    M, n_local = local.shape
    if world == 1:
        return local
    flat = torch.empty((world * M, n_local), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(flat, local.contiguous(), group=group)
    buf = flat.view(world, M, n_local)
    if M == 1:
        y = buf.view(1, world * n_local)
    else:
        y = buf.permute(1, 0, 2).reshape(M, world * n_local)
    if out is not None:
        out.copy_(y)
        return out
    return y


def sharded_int4_gemm(a: torch.Tensor, packed_shard: torch.Tensor, scales_shard: torch.Tensor,
                      group_size: int = 128, world: int = 1,
                      process_group: Optional[dist.ProcessGroup] = None,
                      local_gemm: Optional[Callable] = None, **kw) -> torch.Tensor:
    """``A @ dequant(W)`` for a W4A16 layer whose columns are sharded over ranks.

    ``local_gemm(a, packed, scales, group_size=...)`` defaults to
    ``gemm_int4.int4_gemm`` (the sm_100a kernels); tests may pass another
    implementation to exercise the sharding on CPU ranks.
    """
    fn = local_gemm or gemm_int4.int4_gemm
    y_local = fn(a, packed_shard, scales_shard, group_size=group_size, **kw)
    return gather_columns(y_local, world, process_group)


def sharded_fp8_gemm(a8: torch.Tensor, a_scale: float, b8_shard: torch.Tensor, b_scale: float,
                     world: int = 1, process_group: Optional[dist.ProcessGroup] = None,
                     local_gemm: Optional[Callable] = None, **kw) -> torch.Tensor:
    """Scaled e4m3 GEMM with B's columns sharded over ranks (global scales)."""
    fn = local_gemm or gemm_fp8.fp8_gemm_precast
    y_local = fn(a8, a_scale, b8_shard, b_scale, **kw)
    return gather_columns(y_local, world, process_group)
