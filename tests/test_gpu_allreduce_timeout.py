"""The one-shot all-reduce's bounded wait, made to run out on one GPU.

Two shared buffers are allocated on the same GPU and handed to
nvattn_allreduce as ranks 0 and 1 of a two-rank group. Rank 0 calls alone:
it publishes its chunks and then waits for rank 1's, which nothing sets.
With the wait limit shortened to about a millisecond, the launch must end
by itself and set NVATTN_STATUS_TIMEOUT. No peer GPU is involved, every
address is a local allocation, and the context stays usable.

Rank 1 then calls with its own input: rank 0's part of that launch is
already published (or pushed), so rank 1's waits succeed at once and its
output must be the exact sum of both ranks' inputs. The flags stayed
consistent through the timed-out launch. Both protocols are covered.
"""
from __future__ import annotations

import ctypes
import time

import numpy as np
import pytest
import torch

from nvattn import _lib, ops
from oracle import reference_math as R

pytestmark = pytest.mark.gpu
dev = torch.device("cuda")


def _bits(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


@pytest.mark.parametrize("cap", [300_001, 100_001], ids=["published-halves", "pushed-words"])
def test_wait_on_a_peer_that_never_arrives_times_out(cap):
    """300,001 elements take the protocol whose ranks publish their own half
    and read the peers'; 100,001 the one that pushes every word with the
    launch number into the peers' receive areas."""
    lib = _lib.load()
    nbytes = lib.nvattn_ar_buffer_bytes(cap)
    bufs = []
    try:
        for _ in range(2):
            b, h = ctypes.c_void_p(), (ctypes.c_char * 64)()
            _lib.call("nvattn_ar_alloc", nbytes, ctypes.addressof(b), ctypes.addressof(h))
            bufs.append(b.value)
        bases = (ctypes.c_uint64 * 2)(*bufs)
        status = ops.status_tensor(dev)
        ops.read_status(dev)
        g = torch.Generator(device=dev).manual_seed(3)
        x0 = (torch.randn(cap, generator=g, device=dev) * 3).to(torch.bfloat16)
        x1 = (torch.randn(cap, generator=g, device=dev) * 3).to(torch.bfloat16)
        out0, out1 = torch.empty_like(x0), torch.empty_like(x1)
        stream = torch.cuda.current_stream(dev).cuda_stream
        prev = lib.nvattn_ar_set_wait_limit(2_000_000)  # ~1 ms of SM clocks
        try:
            torch.cuda.synchronize(dev)
            t0 = time.perf_counter()
            _lib.call("nvattn_allreduce", ctypes.addressof(bases), 0, 2, cap, cap,
                      x0.data_ptr(), out0.data_ptr(), status.data_ptr(), stream)
            torch.cuda.synchronize(dev)
            waited = time.perf_counter() - t0
        finally:
            lib.nvattn_ar_set_wait_limit(prev)
        st = ops.read_status(dev)
        print(f"rank 0 alone: status {st:#x} after {waited * 1e3:.1f} ms")
        assert st & 4, "NVATTN_STATUS_TIMEOUT not set"
        assert waited < 5.0
        # rank 1 completes the launch rank 0 published: the exact two-rank sum
        _lib.call("nvattn_allreduce", ctypes.addressof(bases), 1, 2, cap, cap,
                  x1.data_ptr(), out1.data_ptr(), status.data_ptr(), stream)
        torch.cuda.synchronize(dev)
        assert ops.read_status(dev) == 0
        want = R.allreduce_sum(np.stack([_bits(x0), _bits(x1)]))
        assert np.array_equal(_bits(out1), want)
    finally:
        torch.cuda.synchronize(dev)
        for b in bufs:
            lib.nvattn_ar_free(ctypes.c_void_p(b))
