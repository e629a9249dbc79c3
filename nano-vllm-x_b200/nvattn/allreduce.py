"""One-shot all-reduce over NVLink peer memory for the row-parallel linears.

RowParallelLinear.forward (nanovllm/layers/linear.py:152-155) computes
``y = F.linear(x, W_shard)`` on every rank and sums the partials with
``dist.all_reduce(y)`` (NCCL). For decode-sized messages (a few hundred
tokens x hidden) NCCL's per-call latency dominates. Here each rank's GEMM
(cuBLAS, local operands only) writes its partial straight into an IPC-shared
buffer, and one kernel (``nvattn_allreduce``) synchronises with the peers
through flags in those buffers, reads every partial over NVLink and writes the
sum: the same bits on every rank, the single rounded bf16 add of NCCL's sum
at two ranks. Messages larger than the buffer keep NCCL, the reference's own
collective.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

_HEADER_BYTES = 4096
_HANDLE_BYTES = 64


class _DevicePtr:
    """A raw device allocation seen through __cuda_array_interface__."""

    def __init__(self, ptr: int, numel: int):
        self.__cuda_array_interface__ = {"shape": (numel,), "typestr": "<i2",
                                         "data": (ptr, False), "version": 3}


class OneShotAllReduce:
    """Peer-memory all-reduce for one process group (one rank per GPU, up to 8).

    Collective to construct (all ranks at once, outside graph capture).
    ``partial(n)`` is a bf16 view of this rank's first n shared elements (the
    GEMM's output); ``all_reduce(n, out)`` sums the n-element partials of all
    ranks into ``out``. Every rank must call in the same order.
    """

    def __init__(self, capacity_elems: int, group=None, device=None):
        if capacity_elems <= 0:
            raise ValueError("capacity_elems must be positive")
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("the one-shot all-reduce serves up to 8 ranks")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None \
            else torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("nvattn ops need CUDA tensors (no CPU fallback)")
        lib = _lib.load()
        self.capacity = int(capacity_elems)
        self.bytes = int(lib.nvattn_ar_buffer_bytes(self.capacity))
        own = ctypes.c_void_p()
        handle = (ctypes.c_char * _HANDLE_BYTES)()
        with torch.cuda.device(self.device):
            _lib.call("nvattn_ar_alloc", self.bytes, ctypes.addressof(own),
                      ctypes.addressof(handle))
        self._own = own.value
        handles: list = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self._opened: list[int] = []
        bases = []
        with torch.cuda.device(self.device):
            for p, h in enumerate(handles):
                if p == self.rank:
                    bases.append(self._own)
                    continue
                buf = (ctypes.c_char * _HANDLE_BYTES).from_buffer_copy(h)
                peer = ctypes.c_void_p()
                _lib.call("nvattn_ar_open", ctypes.addressof(buf), ctypes.addressof(peer))
                self._opened.append(peer.value)
                bases.append(peer.value)
        self._bases = (ctypes.c_uint64 * self.world)(*bases)
        data = torch.as_tensor(_DevicePtr(self._own + _HEADER_BYTES, self.capacity),
                               device=self.device)
        self._data = data.view(torch.bfloat16)
        self._closed = False

    def partial(self, numel: int) -> torch.Tensor:
        """This rank's shared partial, the first ``numel`` elements (bf16)."""
        if not 0 < numel <= self.capacity:
            raise ValueError(f"{numel} elements outside (0, {self.capacity}]")
        return self._data[:numel]

    def all_reduce(self, numel: int, out: torch.Tensor, status=None) -> torch.Tensor:
        """out[:numel] = sum over ranks of partial(numel)."""
        if self._closed:
            raise RuntimeError("all-reduce buffers already released")
        if out.device != self.device or out.dtype != torch.bfloat16 or not out.is_contiguous() \
                or out.numel() < numel:
            raise ValueError("out must be a contiguous bf16 CUDA tensor of >= numel elements")
        from .ops import _stream, status_tensor
        if status is None:
            status = status_tensor(self.device)
        _lib.call("nvattn_allreduce", ctypes.addressof(self._bases), self.rank, self.world,
                  int(numel), self.capacity, out.data_ptr(),
                  status.data_ptr() if status is not None else None, _stream(self.device))
        return out

    def close(self) -> None:
        """Release the mappings and the buffer (collective: all ranks)."""
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._data = None
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.call("nvattn_ar_close", p)
            dist.barrier(group=self.group)
            _lib.call("nvattn_ar_free", self._own)
        self._opened = []
        self._closed = True


def row_parallel_forward(ar: OneShotAllReduce, x: torch.Tensor, weight: torch.Tensor,
                         bias: torch.Tensor | None, tp_rank: int) -> torch.Tensor | None:
    """RowParallelLinear.forward (linear.py:152-155) through the one-shot
    all-reduce: the GEMM writes the partial into the shared buffer, then one
    kernel sums it across ranks. Returns None when the message exceeds the
    buffer (the caller keeps the reference path)."""
    n_out = weight.shape[0]
    numel = x.numel() // x.shape[-1] * n_out
    if numel == 0 or numel > ar.capacity:
        return None
    part = ar.partial(numel).view(*x.shape[:-1], n_out)
    torch.matmul(x, weight.t(), out=part)
    if bias is not None and tp_rank == 0:
        part.add_(bias)
    out = torch.empty(part.shape, dtype=part.dtype, device=part.device)
    ar.all_reduce(numel, out)
    return out
