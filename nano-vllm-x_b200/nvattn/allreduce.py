"""One-shot all-reduce over NVLink peer memory for the row-parallel linears.

RowParallelLinear.forward (nanovllm/layers/linear.py:152-155) computes
``y = F.linear(x, W_shard)`` on every rank and sums the partials with
``dist.all_reduce(y)`` (NCCL). For decode-sized messages (a few hundred
tokens x hidden) NCCL's per-call latency dominates. Here one kernel
(``nvattn_allreduce``) sums the partials over the ranks' IPC-shared buffers:
small messages are pushed into every peer's receive area with the launch
number beside each 4-byte word (no fence or flag round trip), larger ones are
published in the rank's own buffer behind per-block flags and read by the
peers over NVLink. Either way every rank gets the same bits, the single
rounded bf16 add of NCCL's sum at two ranks. Messages larger than the buffer
keep NCCL, the reference's own collective.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

_HANDLE_BYTES = 64


class OneShotAllReduce:
    """Peer-memory all-reduce for one process group (one rank per GPU, up to 8).

    Collective to construct (all ranks at once, outside graph capture).
    ``all_reduce(x, out)`` sums the bf16 tensor x of every rank into out (x
    itself when out is None: in place). Every rank must call in the same
    order with the same number of elements.
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
        self._closed = False

    def all_reduce(self, x: torch.Tensor, out: torch.Tensor | None = None,
                   status=None) -> torch.Tensor:
        """out = sum over ranks of x (bf16, contiguous, <= capacity elements)."""
        if self._closed:
            raise RuntimeError("all-reduce buffers already released")
        if out is None:
            out = x
        for t in (x, out):
            if t.device != self.device or t.dtype != torch.bfloat16 or not t.is_contiguous():
                raise ValueError("x and out must be contiguous bf16 tensors on this rank's GPU")
        if out.numel() != x.numel():
            raise ValueError("x and out differ in size")
        if x.numel() > self.capacity:
            raise ValueError(f"{x.numel()} elements exceed the capacity {self.capacity}")
        from .ops import _stream, status_tensor
        if status is None:
            status = status_tensor(self.device)
        _lib.call("nvattn_allreduce", ctypes.addressof(self._bases), self.rank, self.world,
                  int(x.numel()), self.capacity, x.data_ptr(), out.data_ptr(),
                  status.data_ptr() if status is not None else None, _stream(self.device))
        return out

    def pushes_words(self, numel: int) -> bool:
        """True when a call of numel elements takes the pushed-words protocol
        (the one faster than NCCL; nvattn_ar_protocol)."""
        return _lib.load().nvattn_ar_protocol(self.world, int(numel), self.capacity) == 1

    def close(self) -> None:
        """Release the mappings and the buffer (collective: all ranks)."""
        if self._closed:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.call("nvattn_ar_close", p)
            dist.barrier(group=self.group)
            _lib.call("nvattn_ar_free", self._own)
        self._opened = []
        self._closed = True


def row_parallel_forward(ar: OneShotAllReduce, x: torch.Tensor, weight: torch.Tensor,
                         bias: torch.Tensor | None, tp_rank: int,
                         pushed_only: bool = False) -> torch.Tensor | None:
    """RowParallelLinear.forward (linear.py:152-155) through the one-shot
    all-reduce: the rank's F.linear partial, then one kernel sums it across
    ranks in place. Returns None when the message exceeds the buffer, or with
    pushed_only when it would not take the pushed-words protocol (the caller
    keeps the reference path)."""
    import torch.nn.functional as F
    n_out = weight.shape[0]
    numel = x.numel() // x.shape[-1] * n_out
    if numel == 0 or numel > ar.capacity:
        return None
    if pushed_only and not ar.pushes_words(numel):
        return None
    y = F.linear(x, weight, bias if tp_rank == 0 else None)
    return ar.all_reduce(y.contiguous())
