"""Seeded attention cases shared by the golden-vector script and the tests.

Inputs are regenerated from torch's CPU generator (deterministic for a given
torch build), so the committed fixtures only hold outputs. Each case mirrors
one call pattern of nanovllm/layers/attention.py:

* dense         — flash_attn_varlen_func without block_table (attention.py:67-70,
                  fresh prefill); k and v are views of a qkv projection, as the
                  engine passes them (qwen3.py:78-81).
* paged_prefix  — flash_attn_varlen_func with block_table: prefix-cache hit,
                  keys gathered from the cache (attention.py:65-66).
* decode        — flash_attn_with_kvcache on q.unsqueeze(1) (attention.py:72-74),
                  block-boundary context lengths, permuted physical blocks.
* chain8        — paged prefill with 8 queries per sequence: the verification
                  batch of a linear (n-gram) draft.
"""
from __future__ import annotations

import numpy as np
import torch

HEAD_DIM = 128


def _paged(gen, lens, nkv, block_size=256, extra_blocks=3):
    """Random caches and permuted block tables holding `lens` tokens per sequence."""
    nblk = [(n + block_size - 1) // block_size for n in lens]
    total = sum(nblk) + extra_blocks
    perm = torch.randperm(total, generator=gen).tolist()
    tables, pos = [], 0
    for n in nblk:
        tables.append(perm[pos:pos + n])
        pos += n
    width = max(nblk)
    bt = torch.tensor([t + [-1] * (width - len(t)) for t in tables], dtype=torch.int32)
    k_cache = torch.randn(total, block_size, nkv, HEAD_DIM, generator=gen).to(torch.bfloat16)
    v_cache = torch.randn(total, block_size, nkv, HEAD_DIM, generator=gen).to(torch.bfloat16)
    return k_cache, v_cache, bt


def make_case(name: str) -> dict:
    seeds = {"dense": 11, "paged_prefix": 12, "decode": 13, "chain8": 14}
    gen = torch.Generator().manual_seed(seeds[name])
    if name == "dense":
        H, KVH = 4, 2
        lens = [1, 37, 150]
        N = sum(lens)
        qkv = torch.randn(N, (H + 2 * KVH) * HEAD_DIM, generator=gen).to(torch.bfloat16)
        q, k, v = qkv.split([H * HEAD_DIM, KVH * HEAD_DIM, KVH * HEAD_DIM], dim=-1)
        q = q.contiguous().view(N, H, HEAD_DIM)
        k = k.contiguous().view(N, KVH, HEAD_DIM)
        v = v.view(N, KVH, HEAD_DIM)
        cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)
        return dict(kind="varlen", q=q, k=k, v=v, cu_q=cu, cu_k=cu.clone(), max_q=max(lens),
                    max_k=max(lens), block_table=None, H=H, KVH=KVH, qkv=qkv)
    if name in ("paged_prefix", "chain8"):
        H, KVH = 4, 1
        if name == "paged_prefix":
            cached, new = [256, 512, 0], [40, 100, 70]
        else:
            cached, new = [100, 256, 300], [8, 8, 8]
        klen = [c + n for c, n in zip(cached, new)]
        k_cache, v_cache, bt = _paged(gen, klen, KVH)
        q = torch.randn(sum(new), H, HEAD_DIM, generator=gen).to(torch.bfloat16)
        cu_q = torch.tensor(np.concatenate([[0], np.cumsum(new)]), dtype=torch.int32)
        cu_k = torch.tensor(np.concatenate([[0], np.cumsum(klen)]), dtype=torch.int32)
        return dict(kind="varlen", q=q, k=k_cache, v=v_cache, cu_q=cu_q, cu_k=cu_k,
                    max_q=max(new), max_k=max(klen), block_table=bt, H=H, KVH=KVH)
    if name == "decode":
        H, KVH = 8, 1
        lens = [1, 63, 64, 255, 257, 700]
        k_cache, v_cache, bt = _paged(gen, lens, KVH)
        q = torch.randn(len(lens), H, HEAD_DIM, generator=gen).to(torch.bfloat16)
        return dict(kind="decode", q=q, k_cache=k_cache, v_cache=v_cache,
                    cache_seqlens=torch.tensor(lens, dtype=torch.int32), block_table=bt,
                    H=H, KVH=KVH)
    raise KeyError(name)


CASES = ("dense", "paged_prefix", "decode", "chain8")
