"""Varlen causal prefill (dense and paged/prefix-cache) on the GPU against
the oracle (max-abs 1e-2 beyond the bf16 output rounding, helpers.ATOL)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_close, cu, paged_layout, random_cache
from oracle import reference_math as R

from nvattn import ops

pytestmark = pytest.mark.gpu
dev = torch.device("cuda")


def _dense(lens_q, H, KVH, lens_k=None, causal=True, seed=0):
    g = torch.Generator().manual_seed(seed)
    lens_k = lens_q if lens_k is None else lens_k
    Nq, Nk = sum(lens_q), sum(lens_k)
    q = torch.randn(Nq, H, 128, generator=g).to(torch.bfloat16)
    # k, v as the engine passes them: k contiguous, v a view into a qkv buffer
    qkv = torch.randn(Nk, (H + 2 * KVH) * 128, generator=g).to(torch.bfloat16)
    k = qkv[:, H * 128:(H + KVH) * 128].contiguous().view(Nk, KVH, 128)
    cq, ck = cu(lens_q), cu(lens_k)
    qkv_d = qkv.to(dev)
    vd = qkv_d[:, (H + KVH) * 128:].view(Nk, KVH, 128)
    out = ops.varlen_prefill(q.to(dev), k.to(dev), vd, cq.to(dev), ck.to(dev), max(lens_q),
                             max(lens_k), softmax_scale=128 ** -0.5, causal=causal)
    torch.cuda.synchronize()
    v = qkv[:, (H + KVH) * 128:].view(Nk, KVH, 128)
    ref = R.varlen_attention(q, k, v, cq.numpy(), ck.numpy(), 128 ** -0.5, causal)
    return out, ref


@pytest.mark.parametrize("H,KVH", [(16, 8), (32, 8), (64, 8), (8, 8), (16, 1)])
def test_dense_causal(H, KVH):
    lens = [1, 2, 63, 64, 65, 300, 1024]
    out, ref = _dense(lens, H, KVH, seed=H * 3 + KVH)
    assert_close(out, ref)
    assert ops.read_status() == 0


def test_dense_non_causal():
    out, ref = _dense([5, 130, 77], 16, 8, causal=False, seed=2)
    assert_close(out, ref)


def test_dense_fewer_keys_than_queries():
    # bottom-right alignment: the first Lq-Lk queries see no key -> zeros
    out, ref = _dense([6, 10], 8, 4, lens_k=[3, 10], seed=3)
    assert torch.all(out[:3] == 0)
    assert_close(out, ref)


def _paged(cached, new, H, KVH, block_size=256, seed=0, shared_prefix=False):
    g = torch.Generator().manual_seed(seed)
    klen = [c + n for c, n in zip(cached, new)]
    nblocks, bt = paged_layout(klen, block_size, seed=seed)
    if shared_prefix:
        # every sequence reuses sequence 0's prefix blocks (prefix-cache hit)
        P = cached[0]
        assert all(c == P for c in cached) and P % block_size == 0
        for b in range(1, len(klen)):
            bt[b, :P // block_size] = bt[0, :P // block_size]
    kc = random_cache(nblocks, block_size, KVH, g)
    vc = random_cache(nblocks, block_size, KVH, g)
    q = torch.randn(sum(new), H, 128, generator=g).to(torch.bfloat16)
    cq, ck = cu(new), cu(klen)
    out = ops.varlen_prefill(q.to(dev), kc.to(dev), vc.to(dev), cq.to(dev), ck.to(dev),
                             max(new), max(klen), softmax_scale=128 ** -0.5, causal=True,
                             block_table=bt.to(dev))
    torch.cuda.synchronize()
    ref = R.varlen_attention(q, kc, vc, cq.numpy(), ck.numpy(), 128 ** -0.5, True, bt.numpy())
    return out, ref


def test_paged_prefix_cache_hit_qwen3_8b_shape():
    # cfg3 shape at reduced batch: 32Q/8KV, shared 2048-token prefix, suffix in [128, 512]
    rng = np.random.default_rng(21)
    new = rng.integers(128, 513, size=4).tolist()
    out, ref = _paged([2048] * 4, new, 32, 8, seed=21, shared_prefix=True)
    assert_close(out, ref)
    assert ops.read_status() == 0


def test_paged_chunked_prefill_continuation():
    # second chunk of a chunked prefill: 1024 cached tokens, 276 new (scheduler.py:42)
    out, ref = _paged([1024, 0, 300], [276, 50, 1], 16, 8, seed=22)
    assert_close(out, ref)


def test_paged_unaligned_prefix_and_block_512():
    out, ref = _paged([100, 700], [33, 64], 16, 4, block_size=512, seed=23)
    assert_close(out, ref)


def test_flash_attn_varlen_func_keyword_form():
    g = torch.Generator().manual_seed(24)
    lens = [17, 40]
    q = torch.randn(57, 8, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(57, 2, 128, generator=g).to(torch.bfloat16)
    v = torch.randn(57, 2, 128, generator=g).to(torch.bfloat16)
    c = cu(lens)
    o = ops.flash_attn_varlen_func(q.to(dev), k.to(dev), v.to(dev), max_seqlen_q=40,
                                   cu_seqlens_q=c.to(dev), max_seqlen_k=40,
                                   cu_seqlens_k=c.to(dev), softmax_scale=128 ** -0.5,
                                   causal=True, block_table=None)
    ref = R.varlen_attention(q, k, v, c.numpy(), c.numpy(), 128 ** -0.5, True)
    assert_close(o, ref)


@pytest.mark.parametrize("paged", [False, True])
def test_row_max_growing_in_a_late_tile(paged):
    """Keys whose scores jump far above everything before them (x10 keys at
    positions 300, 460 and 700: the second half of tile 2, the first and
    second halves of tile 3 and 5) make every row's running max grow past the
    rescale threshold after its first tiles; the single-pass softmax must redo
    those halves and rescale what it already accumulated."""
    g = torch.Generator().manual_seed(31)
    H, KVH, L = 16, 8, 800
    q = torch.randn(L, H, 128, generator=g).to(torch.bfloat16)
    k = torch.randn(L, KVH, 128, generator=g)
    v = torch.randn(L, KVH, 128, generator=g).to(torch.bfloat16)
    k[[300, 460, 700]] *= 10
    k = k.to(torch.bfloat16)
    c = cu([L])
    if paged:
        nblocks, bt = paged_layout([L], 256, seed=31)
        kc = torch.zeros(nblocks, 256, KVH, 128, dtype=torch.bfloat16)
        vc = torch.zeros_like(kc)
        for t in range(L):
            kc[bt[0, t // 256], t % 256] = k[t]
            vc[bt[0, t // 256], t % 256] = v[t]
        # the last 8 of the 800 queries: they see every key
        qn = q[-8:]
        out = ops.varlen_prefill(qn.to(dev), kc.to(dev), vc.to(dev), cu([8]).to(dev), c.to(dev),
                                 8, L, softmax_scale=128 ** -0.5, causal=True,
                                 block_table=bt.to(dev))
        ref = R.varlen_attention(qn, kc, vc, cu([8]).numpy(), c.numpy(), 128 ** -0.5, True,
                                 bt.numpy())
    else:
        out = ops.varlen_prefill(q.to(dev), k.to(dev), v.to(dev), c.to(dev), c.to(dev), L, L,
                                 softmax_scale=128 ** -0.5, causal=False)
        ref = R.varlen_attention(q, k, v, c.numpy(), c.numpy(), 128 ** -0.5, False)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    assert_close(out, ref, f"late max growth ({'paged' if paged else 'dense'})")
    assert ops.read_status() == 0
