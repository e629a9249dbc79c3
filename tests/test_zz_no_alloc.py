"""The allocation-free decode entry point, nvattn_paged_decode_noalloc.

Some hosts cannot allocate device memory at the moment they run decode: an
engine whose allocator has already handed the free GPU memory to its KV
cache, a path that must avoid cudaMalloc's implicit device synchronisation,
or a foreign-language caller holding only raw pointers. For them the library
keeps the split-K workspace in a fixed 16 MiB device array of its own. These
tests call that entry point through the C ABI and check it against the
workspace-taking nvattn_paged_decode on the same inputs, twice in a row (the
array is shared by every call and keeps the previous call's contents).

This file is named to be collected last, so a run that stops at the first
failure has already run every other test; it also passes on its own.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_close, paged_layout, random_cache
from oracle import reference_math as R

from nvattn import _lib, ops

pytestmark = pytest.mark.gpu
dev = torch.device("cuda")
SCRATCH_BYTES = 16 << 20  # the library's fixed workspace, per device


def _noalloc(q, kc, vc, lens, bt, out):
    num_blocks, block_size, kvh, d = kc.shape
    B, H, _ = q.shape
    _lib.call("nvattn_paged_decode_noalloc", q.data_ptr(), q.stride(0), q.stride(1),
              kc.data_ptr(), vc.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
              lens.data_ptr(), bt.data_ptr(), bt.stride(0), bt.shape[1], num_blocks, block_size,
              B, H, kvh, d, d ** -0.5, None, torch.cuda.current_stream().cuda_stream)


def _case(seed, B, H, KVH, max_len):
    g = torch.Generator().manual_seed(seed)
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, max_len + 1, size=B).tolist()
    nblocks, bt = paged_layout(lens, 256, seed=seed)
    kc = random_cache(nblocks, 256, KVH, g)
    vc = random_cache(nblocks, 256, KVH, g)
    q = torch.randn(B, H, 128, generator=g).to(torch.bfloat16)
    return q, kc, vc, torch.tensor(lens, dtype=torch.int32), bt


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row():
    B, H, KVH = 8, 32, 8
    cases = [_case(101, B, H, KVH, 4000), _case(202, B, H, KVH, 3000)]
    for q, kc, vc, lens, bt in cases:
        # the split-K path must be the one exercised, and it must fit the scratch
        need = ops.decode_workspace_bytes(B, H, KVH, bt.shape[1], 256)
        assert 0 < need <= SCRATCH_BYTES
    outs = []
    for q, kc, vc, lens, bt in cases:  # two calls back to back on one stream
        qd, kd, vd, ld, bd = q.to(dev), kc.to(dev), vc.to(dev), lens.to(dev), bt.to(dev)
        out = torch.empty(B, H, 128, dtype=torch.bfloat16, device=dev)
        _noalloc(qd, kd, vd, ld, bd, out)
        ref_entry = ops.paged_decode(qd, kd, vd, ld, bd, softmax_scale=128 ** -0.5)
        outs.append((out, ref_entry, q, kc, vc, lens, bt))
    torch.cuda.synchronize()
    for out, ref_entry, q, kc, vc, lens, bt in outs:
        assert torch.isfinite(out.float()).all()
        # the same kernels with the same split: only the workspace address
        # differs, so the outputs must be equal bit for bit
        assert torch.equal(out, ref_entry)
        ref = R.decode_attention(q, kc, vc, lens.numpy(), bt.numpy(), 128 ** -0.5)
        assert_close(out, ref, "no-alloc decode vs oracle")
    assert ops.read_status() == 0


def test_noalloc_rejects_batches_beyond_its_scratch():
    # configs[3] at TP1 needs ~34 MB of partials: more than the fixed 16 MiB
    B, H, KVH, width = 128, 64, 8, 128
    assert ops.decode_workspace_bytes(B, H, KVH, width, 256) > SCRATCH_BYTES
    q = torch.zeros(B, H, 128, dtype=torch.bfloat16, device=dev)
    kc = torch.zeros(1, 256, KVH, 128, dtype=torch.bfloat16, device=dev)
    lens = torch.ones(B, dtype=torch.int32, device=dev)
    bt = torch.zeros(B, width, dtype=torch.int32, device=dev)
    out = torch.empty_like(q)
    with pytest.raises(_lib.NvattnError) as ei:
        _noalloc(q, kc, kc, lens, bt, out)
    assert ei.value.code == _lib.ERR_WORKSPACE
    assert "scratch" in str(ei.value)
