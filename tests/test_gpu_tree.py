"""Tree-verification attention and accepted-path compaction on the GPU."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import bf16_bits
from helpers import assert_close, cu, max_err, paged_layout, random_cache
from oracle import reference_math as R

from nvattn import ops, tree

pytestmark = pytest.mark.gpu
dev = torch.device("cuda")


def _setup(ctx, n_nodes, H, KVH, seed):
    g = torch.Generator().manual_seed(seed)
    total = [c + n for c, n in zip(ctx, n_nodes)]
    nblocks, bt = paged_layout(total, 256, seed=seed)
    kc = random_cache(nblocks, 256, KVH, g)
    vc = random_cache(nblocks, 256, KVH, g)
    q = torch.randn(sum(n_nodes), H, 128, generator=g).to(torch.bfloat16)
    return g, kc, vc, q, bt


def test_eagle_tree_64_nodes_qwen3_8b_shape():
    parents, _ = tree.build_draft_tree((4, 3, 2, 1, 1, 1), 64)
    masks = tree.ancestor_masks(parents)
    ctx = [1024, 255, 256, 3000]
    n = [64] * len(ctx)
    H, KVH = 32, 8
    g, kc, vc, q, bt = _setup(ctx, n, H, KVH, 31)
    # the tree nodes' K/V are scattered into the cache first (positions ctx+i)
    kn = torch.randn(sum(n), KVH, 128, generator=g).to(torch.bfloat16)
    vn = torch.randn(sum(n), KVH, 128, generator=g).to(torch.bfloat16)
    slots = []
    for b, c in enumerate(ctx):
        for i in range(n[b]):
            p = c + i
            slots.append(int(bt[b, p // 256]) * 256 + p % 256)
    slots = torch.tensor(slots, dtype=torch.int32)
    kcd, vcd = kc.to(dev), vc.to(dev)
    ops.store_kvcache(kn.to(dev), vn.to(dev), kcd, vcd, slots.to(dev))
    all_masks = np.concatenate([masks] * len(ctx))
    cq = cu(n)
    ctx_t = torch.tensor(ctx, dtype=torch.int32)
    out = ops.tree_attention(q.to(dev), kcd, vcd, cq.to(dev), ctx_t.to(dev),
                             torch.from_numpy(all_masks.view(np.int64)).to(dev), bt.to(dev), 64,
                             softmax_scale=128 ** -0.5)
    torch.cuda.synchronize()
    R.store_kvcache(kn.view(torch.int16).numpy(), vn.view(torch.int16).numpy(),
                    kc.view(torch.int16).numpy(), vc.view(torch.int16).numpy(), slots.numpy())
    assert torch.equal(kcd.cpu(), kc) and torch.equal(vcd.cpu(), vc)
    ref = R.tree_attention(q, kc, vc, cq.numpy(), ctx, all_masks, bt.numpy(), 128 ** -0.5)
    assert_close(out, ref)
    assert ops.read_status() == 0


def test_chain_draft_equals_paged_prefill_kernel():
    """8-token linear (n-gram) draft: tree kernel == paged causal prefill kernel."""
    ctx = [100, 256, 511, 2000]
    n = [8] * 4
    g, kc, vc, q, bt = _setup(ctx, n, 32, 8, 32)
    masks = np.concatenate([tree.chain_masks(8)] * 4)
    cq = cu(n)
    ck = cu([c + 8 for c in ctx])
    args = (kc.to(dev), vc.to(dev))
    a = ops.tree_attention(q.to(dev), *args, cq.to(dev),
                           torch.tensor(ctx, dtype=torch.int32, device=dev),
                           torch.from_numpy(masks.view(np.int64)).to(dev), bt.to(dev), 8)
    b = ops.varlen_prefill(q.to(dev), *args, cq.to(dev), ck.to(dev), 8, max(ctx) + 8,
                           causal=True, block_table=bt.to(dev))
    torch.cuda.synchronize()
    ref = R.varlen_attention(q, kc, vc, cq.numpy(), ck.numpy(), 128 ** -0.5, True, bt.numpy())
    assert_close(a, ref)
    assert_close(b, ref)
    # same kernel family, same masks: the two paths agree to bf16 rounding
    assert max_err(a, b) <= 2 ** -7 * max(1.0, float(ref.abs().max()))


def test_accepted_path_compaction():
    parents, _ = tree.build_draft_tree((4, 3, 2, 1, 1, 1), 64)
    rng = np.random.default_rng(7)
    ctx = [300, 1000]
    KVH = 8
    g, kc, vc, _, bt = _setup(ctx, [64, 64], 32, KVH, 33)
    srcs, dsts, cuts = [], [], [0]
    for b, c in enumerate(ctx):
        # random root-to-leaf walk
        path, node = [0], 0
        while True:
            kids = [j for j in range(64) if parents[j] == node]
            if not kids or rng.random() < 0.1:
                break
            node = int(rng.choice(kids))
            path.append(node)
        s, d = tree.compaction_moves(c, path, bt[b].tolist(), 256)
        srcs += s
        dsts += d
        cuts.append(len(srcs))
    src = np.array(srcs, np.int32)
    dst = np.array(dsts, np.int32)
    cuts = np.array(cuts, np.int32)
    kcd, vcd = kc.to(dev), vc.to(dev)
    ops.kv_move(kcd, vcd, torch.from_numpy(src).to(dev), torch.from_numpy(dst).to(dev),
                torch.from_numpy(cuts).to(dev))
    torch.cuda.synchronize()
    ek, ev = bf16_bits(kc), bf16_bits(vc)
    R.kv_move(ek, ev, src, dst, cuts)
    assert np.array_equal(bf16_bits(kcd), ek) and np.array_equal(bf16_bits(vcd), ev)


def test_tree_split_and_unsplit_paths():
    """Few sequences: the context is split over CTAs and merged; many (a wave
    or more of CTAs): no split, sequences dispatched longest first."""
    from nvattn import ops as O
    parents, _ = tree.build_draft_tree((4, 3, 2, 1, 1, 1), 64)
    masks = tree.ancestor_masks(parents)
    for nseq, ctx_hi, expect_split in ((3, 5000, True), (80, 300, False)):
        rng = np.random.default_rng(nseq)
        ctx = rng.integers(1, ctx_hi, size=nseq).tolist()
        n = [64] * nseq
        g, kc, vc, q, bt = _setup(ctx, n, 32, 8, 40 + nseq)
        ws = O.tree_workspace_bytes(nseq, 64, sum(n), 32, 8, bt.shape[1], 256)
        order_bytes = (nseq * 4 + 255) // 256 * 256  # the dispatch order, always there
        assert ws >= order_bytes and (ws > order_bytes) == expect_split
        all_masks = np.concatenate([masks] * nseq)
        cq = cu(n)
        out = ops.tree_attention(q.to(dev), kc.to(dev), vc.to(dev), cq.to(dev),
                                 torch.tensor(ctx, dtype=torch.int32, device=dev),
                                 torch.from_numpy(all_masks.view(np.int64)).to(dev), bt.to(dev),
                                 64, softmax_scale=128 ** -0.5)
        torch.cuda.synchronize()
        ref = R.tree_attention(q, kc, vc, cq.numpy(), ctx, all_masks, bt.numpy(), 128 ** -0.5)
        assert_close(out, ref)
    assert ops.read_status() == 0


def test_tree_row_max_growing_in_a_late_tile():
    """Context keys scaled x10 at positions 200, 300 and 470 (the second half of
    key tile 1, the first half of tile 2, the second half of tile 3) make many
    rows' running maxima grow past the rescale threshold after their first
    tile: the single pass must take the two-pass fallback (first half) or wait
    for the first half's P V, rescale and redo the second half."""
    parents, _ = tree.build_draft_tree((4, 3, 2, 1, 1, 1), 64)
    masks = tree.ancestor_masks(parents)
    ctx = [700, 700, 520]
    n = [64] * len(ctx)
    H, KVH = 32, 8
    g, kc, vc, q, bt = _setup(ctx, n, H, KVH, 57)
    for b in range(len(ctx)):
        for pos in (200, 300, 470):
            kc[int(bt[b, pos // 256]), pos % 256] = (kc[int(bt[b, pos // 256]), pos % 256].float()
                                                      * 10).to(torch.bfloat16)
    all_masks = np.concatenate([masks] * len(ctx))
    cq = cu(n)
    out = ops.tree_attention(q.to(dev), kc.to(dev), vc.to(dev), cq.to(dev),
                             torch.tensor(ctx, dtype=torch.int32, device=dev),
                             torch.from_numpy(all_masks.view(np.int64)).to(dev), bt.to(dev), 64,
                             softmax_scale=128 ** -0.5)
    torch.cuda.synchronize()
    ref = R.tree_attention(q, kc, vc, cq.numpy(), ctx, all_masks, bt.numpy(), 128 ** -0.5)
    assert torch.isfinite(out.float()).all()
    assert_close(out, ref, "tree, late max growth")
    assert ops.read_status() == 0
