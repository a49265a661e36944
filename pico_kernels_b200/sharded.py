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

Where the local kernel is the CUDA-core GEMV (M <= 2), the tensor-core decode
kernel (M <= 32) or the skinny swap-AB kernel (32 < M <= 256 where the library
picks it), a ``PeerExchange`` replaces the all-gather: the kernel writes its
columns straight into every rank's output buffer over NVLink (buffers mapped
with CUDA IPC handles) and ends with a flag barrier, so the layer is one kernel
per rank (``pk_w4a16_gemm_sharded``).

fp8 scales are per tensor and must be global: callers quantize the whole
activation and weight (or all-reduce the absmax) before slicing, so every
rank's ``out_scale`` equals the unsharded one.

The reference has no multi-GPU path; this is the sharding BASELINE.json's
Llama-70B configuration asks for.
"""

from __future__ import annotations

import ctypes
from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib, gemm_fp8, gemm_int4

__all__ = ["shard_columns", "shard_int4", "gather_columns", "sharded_int4_gemm",
           "sharded_fp8_gemm", "PeerExchange"]


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


def _readable(t: torch.Tensor) -> torch.Tensor:
    """``t`` in the layout the sharded kernels read: unit stride along the
    last dimension, a row stride of 16 bytes' multiple and a 16-byte aligned
    start (a fresh copy when the tensor is a view that misses one)."""
    elem = t.element_size()
    if (t.stride(-1) == 1 and (t.stride(0) * elem) % 16 == 0 and t.stride(0) >= t.shape[1]
            and t.data_ptr() % 16 == 0):
        return t
    return t.clone(memory_format=torch.contiguous_format)


class _DeviceArray:
    """Zero-copy view of raw device memory for torch.as_tensor."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


class PeerExchange:
    """Output buffers of an N-sharded layer, mapped on every rank.

    Each rank allocates two ``[max_m, n_full]`` buffers (alternated call by
    call, so a fast rank never overwrites the output a slow rank is still
    reading) and a 32-bit arrival flag, and maps every peer's allocation with
    a CUDA IPC handle (exchanged once with ``all_gather_object``). Collective:
    every rank constructs it, calls ``int4_gemm`` in the same order, and
    ``close``s it. No NCCL runs on the data path.
    """

    def __init__(self, max_m: int, n_full: int, dtype: torch.dtype = torch.float32,
                 group: Optional[dist.ProcessGroup] = None):
        if dtype not in (torch.float32, torch.bfloat16):
            raise _lib.DtypeError("exchange buffers are fp32 or bf16")
        self.lib = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise _lib.ShapeError("the fused exchange covers up to 8 GPUs")
        self.max_m, self.n_full, self.dtype = max_m, n_full, dtype
        self.elem = 4 if dtype == torch.float32 else 2
        self.buf_bytes = (max_m * n_full * self.elem + 255) // 256 * 256
        self.flag_off = 2 * self.buf_bytes
        ptr = ctypes.c_void_p()
        _lib.check(self.lib.pk_shared_alloc(self.flag_off + 256, ctypes.byref(ptr)), "shared alloc")
        self.base = ptr.value
        handle = (ctypes.c_char * 64)()
        _lib.check(self.lib.pk_ipc_get_handle(self.base, ctypes.addressof(handle)), "IPC handle")
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.bases = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.bases.append(self.base)
                continue
            peer = ctypes.c_void_p()
            hbuf = ctypes.create_string_buffer(h, 64)
            _lib.check(self.lib.pk_ipc_open(ctypes.addressof(hbuf), ctypes.byref(peer)), "IPC open")
            self.bases.append(peer.value)
        self.calls = 0  # selects the buffer: calls alternate between the two
        self.device = torch.device("cuda", torch.cuda.current_device())

    def output(self, parity: int, m: int) -> torch.Tensor:
        """This rank's buffer ``parity`` as an ``[m, n_full]`` tensor (no copy)."""
        arr = _DeviceArray(self.base + parity * self.buf_bytes, (m, self.n_full),
                           "<f4" if self.elem == 4 else "<u2")
        t = torch.as_tensor(arr, device=self.device)
        return t if self.elem == 4 else t.view(torch.bfloat16)

    def int4_gemm(self, a: torch.Tensor, packed_shard: torch.Tensor, scales_shard: torch.Tensor,
                  group_size: int = 128) -> Optional[torch.Tensor]:
        """This rank's slice of ``A @ dequant(W)`` written to every rank's buffer.

        Returns ``[M, n_full]`` (valid until two calls later), or None when
        no kernel with the fused exchange covers the shape. Every rank of the
        layer gets the same answer: the library decides from the shape alone
        (``pk_w4a16_gemm_sharded``), and the operands are first brought into
        the layout its kernels read (contiguous, 16-byte aligned, scales in
        A's dtype), so a rank cannot fall back to the all-gather on its own
        while its peers wait in the fused kernel.
        """
        _lib.require_cuda(a, packed_shard, scales_shard)
        for t in (a, packed_shard, scales_shard):
            if t.device != self.device:
                raise _lib.DtypeError(f"operands must be on {self.device} (got {t.device})")
        if a.dtype not in (torch.float16, torch.bfloat16):
            raise _lib.DtypeError(f"a must be fp16 or bf16 (got {a.dtype})")
        if packed_shard.dtype != torch.uint8:
            raise _lib.DtypeError("packed_shard must be uint8")
        if a.dim() != 2 or packed_shard.dim() != 2 or scales_shard.dim() != 2:
            raise _lib.ShapeError("a, packed_shard and scales_shard must be 2-D")
        M, K = a.shape
        n_local = scales_shard.shape[1]
        if packed_shard.shape != (K, n_local // 2) or n_local % 2:
            raise _lib.ShapeError(f"packed_shard must be [{K}, {n_local // 2}] "
                                  f"(got {tuple(packed_shard.shape)})")
        if scales_shard.shape[0] != (K + group_size - 1) // group_size:
            raise _lib.ShapeError(f"scales_shard must have ceil(K / {group_size}) rows")
        if M > self.max_m or n_local * self.world != self.n_full:
            return None
        a = _readable(a)
        packed_shard = _readable(packed_shard)
        scales_shard = _readable(scales_shard if scales_shard.dtype == a.dtype
                                 else scales_shard.to(a.dtype))
        ws_bytes = max(self.lib.pk_w4a16_workspace_size(M, n_local, K, 0), 1 << 16)
        ws = _lib.workspace(a.device, ws_bytes, tag="sharded")
        self.calls += 1
        parity = self.calls & 1
        outs = (ctypes.c_uint64 * self.world)(*[b + parity * self.buf_bytes for b in self.bases])
        flags = (ctypes.c_uint64 * self.world)(*[b + self.flag_off for b in self.bases])
        outs_p, flags_p = ctypes.addressof(outs), ctypes.addressof(flags)
        rc = self.lib.pk_w4a16_gemm_sharded(
            a.data_ptr(), _lib.dtype_code(a.dtype), a.stride(0), packed_shard.data_ptr(),
            scales_shard.data_ptr(), 1.0, group_size, M, n_local, K, _lib.dtype_code(self.dtype),
            self.n_full, self.rank * n_local, self.world, self.rank, outs_p, flags_p,
            ws.data_ptr(), ws.numel(), _lib.stream_of(a))
        if rc == _lib.PK_ERR_UNSUPPORTED:
            self.calls -= 1
            return None
        _lib.check(rc, "sharded int4_gemm")
        return self.output(parity, M)

    def close(self) -> None:
        torch.cuda.synchronize()
        for r, b in enumerate(self.bases):
            if r != self.rank:
                self.lib.pk_ipc_close(b)
        dist.barrier(group=self.group)  # peers unmapped before the memory goes
        self.lib.pk_shared_free(self.base)
        self.bases = []


def sharded_int4_gemm(a: torch.Tensor, packed_shard: torch.Tensor, scales_shard: torch.Tensor,
                      group_size: int = 128, world: int = 1,
                      process_group: Optional[dist.ProcessGroup] = None,
                      local_gemm: Optional[Callable] = None,
                      exchange: Optional[PeerExchange] = None, **kw) -> torch.Tensor:
    """``A @ dequant(W)`` for a W4A16 layer whose columns are sharded over ranks.

    With an ``exchange`` and a shape its kernels cover, the output travels
    inside the local kernel (``PeerExchange``); otherwise each rank computes its block and one NCCL
    all-gather assembles the layer. ``local_gemm(a, packed, scales,
    group_size=...)`` defaults to ``gemm_int4.int4_gemm`` (the sm_100a
    kernels); tests may pass another implementation to exercise the sharding
    on CPU ranks.
    """
    if exchange is not None and local_gemm is None and not kw:
        y = exchange.int4_gemm(a, packed_shard, scales_shard, group_size)
        if y is not None:
            return y
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
