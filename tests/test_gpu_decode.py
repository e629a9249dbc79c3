"""Paged split-K decode on the GPU against the oracle (max-abs 1e-2 beyond the
bf16 output rounding, helpers.ATOL)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_close, paged_layout, random_cache
from oracle import reference_math as R

from nvattn import ops

pytestmark = pytest.mark.gpu
dev = torch.device("cuda")


def _run(lens, H, KVH, block_size=256, seed=0, extra_width=0, nan_fill=False):
    g = torch.Generator().manual_seed(seed)
    nblocks, bt = paged_layout(lens, block_size, seed=seed)
    if extra_width:  # block_table wider than needed (CUDA-graph static buffer)
        bt = torch.cat([bt, torch.full((len(lens), extra_width), -1, dtype=torch.int32)], 1)
    kc = random_cache(nblocks, block_size, KVH, g)
    vc = random_cache(nblocks, block_size, KVH, g)
    if nan_fill:
        # stale bytes past each context end: NaN must not leak into the output
        for b, n in enumerate(lens):
            for j in range(int(n), ((int(n) + block_size - 1) // block_size) * block_size):
                blk = int(bt[b, j // block_size])
                kc[blk, j % block_size] = float("nan")
                vc[blk, j % block_size] = float("nan")
    q = torch.randn(len(lens), H, 128, generator=g).to(torch.bfloat16)
    seqlens = torch.tensor(lens, dtype=torch.int32)
    out = ops.paged_decode(q.to(dev), kc.to(dev), vc.to(dev), seqlens.to(dev), bt.to(dev),
                           softmax_scale=128 ** -0.5)
    torch.cuda.synchronize()
    ref = R.decode_attention(q, kc, vc, seqlens.numpy(), bt.numpy(), 128 ** -0.5)
    return out, ref


@pytest.mark.parametrize("H,KVH", [(64, 8), (16, 8), (32, 8), (8, 1), (16, 1), (4, 4)])
def test_group_sizes(H, KVH):
    rng = np.random.default_rng(H + KVH)
    lens = rng.integers(1, 3000, size=6).tolist()
    out, ref = _run(lens, H, KVH, seed=H)
    assert_close(out, ref)
    assert ops.read_status() == 0


def test_block_boundary_lengths():
    lens = [1, 2, 63, 64, 65, 127, 128, 255, 256, 257, 511, 512, 513, 2047, 2048, 2049, 4097]
    out, ref = _run(lens, 32, 8, seed=3)
    assert_close(out, ref)


def test_zero_length_rows_give_zeros():
    # CUDA-graph padding rows: context_lens 0, stale block-table rows
    lens = [0, 300, 0, 5]
    out, ref = _run(lens, 16, 8, seed=4)
    assert torch.all(out[0] == 0) and torch.all(out[2] == 0)
    assert_close(out, ref)


def test_stale_nan_past_context_end_is_ignored():
    out, ref = _run([5, 70, 300], 16, 8, seed=5, nan_fill=True)
    assert torch.isfinite(out.float()).all()
    assert_close(out, ref)


def test_single_split_path():
    # enough (sequence, kv-head) pairs that one split per pair is chosen
    rng = np.random.default_rng(9)
    lens = rng.integers(1, 2048, size=300).tolist()
    assert ops.decode_workspace_bytes(300, 16, 8, 8, 256) == 0
    out, ref = _run(lens, 16, 8, seed=9)
    assert_close(out, ref)


def test_long_context_qwen3_32b_shape():
    # cfg4 shape at reduced batch: 64Q/8KV heads, contexts into the tens of thousands
    rng = np.random.default_rng(11)
    lens = rng.integers(4096, 32768, size=3).tolist()
    out, ref = _run(lens, 64, 8, seed=11)
    assert_close(out, ref)


def test_block_size_512():
    out, ref = _run([100, 600, 1500], 16, 8, block_size=512, seed=12)
    assert_close(out, ref)


def test_wide_block_table_and_graph_capture():
    """Capture decode in a CUDA graph on static buffers, replay with new metadata."""
    g = torch.Generator().manual_seed(13)
    H, KVH, bs, width, B = 16, 8, 256, 16, 8
    nblocks = B * width
    kc = random_cache(nblocks, bs, KVH, g).to(dev)
    vc = random_cache(nblocks, bs, KVH, g).to(dev)
    q = torch.zeros(B, H, 128, dtype=torch.bfloat16, device=dev)
    lens = torch.zeros(B, dtype=torch.int32, device=dev)
    bt = torch.zeros(B, width, dtype=torch.int32, device=dev)
    out = torch.empty(B, H, 128, dtype=torch.bfloat16, device=dev)
    ws = torch.empty(max(1, ops.decode_workspace_bytes(B, H, KVH, width, bs)), dtype=torch.uint8,
                     device=dev)
    ops.status_tensor()  # created before capture
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.paged_decode(q, kc, vc, lens, bt, out=out, workspace=ws)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.paged_decode(q, kc, vc, lens, bt, out=out, workspace=ws)
    for trial in range(3):
        rng = np.random.default_rng(100 + trial)
        new_lens = rng.integers(0, width * bs, size=B).astype(np.int32)
        perm = rng.permutation(nblocks)[:B * width].reshape(B, width).astype(np.int32)
        qn = torch.randn(B, H, 128, generator=g).to(torch.bfloat16)
        q.copy_(qn.to(dev))
        lens.copy_(torch.from_numpy(new_lens).to(dev))
        bt.copy_(torch.from_numpy(perm).to(dev))
        graph.replay()
        torch.cuda.synchronize()
        ref = R.decode_attention(qn, kc.cpu(), vc.cpu(), new_lens, perm, 128 ** -0.5)
        assert_close(out, ref)
    assert ops.read_status() == 0


def test_many_short_sequences_with_empty_rows():
    """1000 sequences of 0-299 keys, 30% of them empty (CUDA-graph padding)."""
    rng = np.random.default_rng(21)
    lens = rng.integers(0, 300, size=1000)
    lens[rng.random(1000) < 0.3] = 0
    out, ref = _run(lens.tolist(), 4, 2, seed=21)
    assert torch.all(out[torch.from_numpy(lens == 0)] == 0)
    assert_close(out, ref)
    assert ops.read_status() == 0


def test_one_long_sequence_group16():
    """One sequence of 60,000 keys, 16 query heads per KV head (both accumulator
    row halves of the MMA carry heads), split over many CTAs."""
    out, ref = _run([60000], 16, 1, seed=23)
    assert_close(out, ref)


def test_wide_block_table_with_partials():
    """64 sequences under a 64-block-wide table: several key splits per pair,
    most of them past their sequence's end."""
    rng = np.random.default_rng(24)
    lens = rng.integers(1, 8000, size=64).tolist()
    width = 64
    assert ops.decode_workspace_bytes(64, 16, 8, width, 256) > 0
    nb = max(1, (max(lens) + 255) // 256)
    out, ref = _run(lens, 16, 8, seed=24, extra_width=width - nb)
    assert_close(out, ref)
    assert ops.read_status() == 0


def test_flash_attn_with_kvcache_signature():
    """The keyword form used at attention.py:72-74 returns (B, 1, H, d)."""
    g = torch.Generator().manual_seed(14)
    lens = [10, 400]
    nblocks, bt = paged_layout(lens, 256, seed=14)
    kc = random_cache(nblocks, 256, 2, g)
    vc = random_cache(nblocks, 256, 2, g)
    q = torch.randn(2, 8, 128, generator=g).to(torch.bfloat16)
    o = ops.flash_attn_with_kvcache(q.to(dev).unsqueeze(1), kc.to(dev), vc.to(dev),
                                    cache_seqlens=torch.tensor(lens, dtype=torch.int32,
                                                               device=dev),
                                    block_table=bt.to(dev), softmax_scale=128 ** -0.5,
                                    causal=True)
    assert o.shape == (2, 1, 8, 128)
    ref = R.decode_attention(q, kc, vc, np.array(lens), bt.numpy(), 128 ** -0.5)
    assert_close(o[:, 0], ref)
