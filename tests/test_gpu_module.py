"""The drop-in Attention module driven the way ModelRunner drives it.

Single attention layer at the Qwen3-0.6B shape (16 Q heads, 8 KV heads,
head_dim 128, block_size 256): 4 sequences with prompt lengths uniform in
[100, 1024], contiguous block allocation, one prefill then 32 decode steps,
then a prefix-cache prefill of a new sequence that shares sequence 0's first
block. The context is filled with the engine's metadata (restated from
model_runner.py:129-188 and pinned against the reference by
test_oracle.py); after every step the KV cache must equal the oracle's bit for
bit and the outputs must match within 1e-2.
"""
from __future__ import annotations

import random

import numpy as np
import pytest
import torch

from conftest import bf16_bits
from helpers import assert_close
from oracle import reference_math as R

import nvattn
from nvattn import context as ctxmod

pytestmark = pytest.mark.gpu
dev = torch.device("cuda")
H, KVH, D, BS = 16, 8, 128, 256


def _to(t):
    return torch.from_numpy(np.asarray(t)).to(dev) if t is not None else None


def test_prefill_then_32_decode_steps_then_prefix_hit():
    rnd = random.Random(0)
    lens = [rnd.randint(100, 1024) for _ in range(4)]
    steps = 32
    # contiguous blocks, enough for prompt + decode steps (+1 spare block each)
    tables, nxt = [], 0
    for n in lens:
        nb = (n + steps + BS - 1) // BS + 1
        tables.append(list(range(nxt, nxt + nb)))
        nxt += nb
    num_blocks = nxt + 4
    attn = nvattn.Attention(H, D, D ** -0.5, KVH)
    kv = torch.zeros(2, num_blocks, BS, KVH, D, dtype=torch.bfloat16, device=dev)
    attn.k_cache, attn.v_cache = kv[0], kv[1]
    ref_k = np.zeros((num_blocks, BS, KVH, D), np.uint16)
    ref_v = np.zeros_like(ref_k)
    g = torch.Generator().manual_seed(0)

    # ---- prefill (no cache hit: dense attention over the new k/v)
    seqs = [dict(start=0, num_scheduled=n, num_tokens=n, block_table=t[:(n + BS - 1) // BS])
            for n, t in zip(lens, tables)]
    cu_q, cu_k, mq, mk, slots, bt = R.prepare_prefill_metadata(seqs, BS)
    assert bt is None
    N = int(cu_q[-1])
    q = torch.randn(N, H, D, generator=g).to(torch.bfloat16)
    k = torch.randn(N, KVH, D, generator=g).to(torch.bfloat16)
    v = torch.randn(N, KVH, D, generator=g).to(torch.bfloat16)
    ctxmod.set_context(True, _to(cu_q), _to(cu_k), mq, mk, _to(slots), None, None)
    out = attn(q.to(dev), k.to(dev), v.to(dev))
    torch.cuda.synchronize()
    R.store_kvcache(bf16_bits(k), bf16_bits(v), ref_k, ref_v, slots)
    ref = R.varlen_attention(q, k, v, cu_q, cu_k, D ** -0.5, True)
    assert out.shape == (N, H, D)
    assert_close(out, ref)
    assert np.array_equal(bf16_bits(kv[0]), ref_k) and np.array_equal(bf16_bits(kv[1]), ref_v)

    # ---- decode steps
    kc_cpu = lambda: torch.from_numpy(ref_k.view(np.int16)).view(torch.bfloat16)  # noqa: E731
    vc_cpu = lambda: torch.from_numpy(ref_v.view(np.int16)).view(torch.bfloat16)  # noqa: E731
    for step in range(steps):
        dseqs = []
        for n, t in zip(lens, tables):
            total = n + step + 1
            dseqs.append(dict(num_tokens=total, block_table=t[:(total + BS - 1) // BS]))
        slots, ctx_lens, bt = R.prepare_decode_metadata(dseqs, BS)
        B = len(dseqs)
        q = torch.randn(B, H, D, generator=g).to(torch.bfloat16)
        k = torch.randn(B, KVH, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, KVH, D, generator=g).to(torch.bfloat16)
        ctxmod.set_context(False, slot_mapping=_to(slots), context_lens=_to(ctx_lens),
                           block_tables=_to(bt))
        out = attn(q.to(dev), k.to(dev), v.to(dev))
        torch.cuda.synchronize()
        assert out.shape == (B, 1, H, D)
        R.store_kvcache(bf16_bits(k), bf16_bits(v), ref_k, ref_v, slots)
        ref = R.decode_attention(q, kc_cpu(), vc_cpu(), ctx_lens, bt, D ** -0.5)
        assert_close(out[:, 0], ref)
        assert np.array_equal(bf16_bits(kv[0]), ref_k) and np.array_equal(bf16_bits(kv[1]), ref_v)

    # ---- prefix-cache prefill: a new sequence reuses sequence 0's first block
    n_new = 300
    table = [tables[0][0], num_blocks - 2, num_blocks - 1]
    seqs = [dict(start=BS, num_scheduled=n_new - BS + 60, num_tokens=n_new + 60,
                 block_table=table)]
    cu_q, cu_k, mq, mk, slots, bt = R.prepare_prefill_metadata(seqs, BS)
    assert bt is not None  # cu_seqlens_k[-1] > cu_seqlens_q[-1]
    N = int(cu_q[-1])
    q = torch.randn(N, H, D, generator=g).to(torch.bfloat16)
    k = torch.randn(N, KVH, D, generator=g).to(torch.bfloat16)
    v = torch.randn(N, KVH, D, generator=g).to(torch.bfloat16)
    ctxmod.set_context(True, _to(cu_q), _to(cu_k), mq, mk, _to(slots), None, _to(bt))
    out = attn(q.to(dev), k.to(dev), v.to(dev))
    torch.cuda.synchronize()
    R.store_kvcache(bf16_bits(k), bf16_bits(v), ref_k, ref_v, slots)
    ref = R.varlen_attention(q, kc_cpu(), vc_cpu(), cu_q, cu_k, D ** -0.5, True, bt)
    assert_close(out, ref)
    assert np.array_equal(bf16_bits(kv[0]), ref_k)
    ctxmod.reset_context()
    assert nvattn.ops.read_status() == 0


def test_warmup_path_without_cache():
    """ModelRunner.warmup_model runs prefill before the cache is bound
    (model_runner.py:91-101): the store is skipped, dense attention runs."""
    attn = nvattn.Attention(H, D, D ** -0.5, KVH)
    g = torch.Generator().manual_seed(1)
    lens = [128, 128]
    c = torch.tensor([0, 128, 256], dtype=torch.int32)
    q = torch.randn(256, H, D, generator=g).to(torch.bfloat16)
    k = torch.randn(256, KVH, D, generator=g).to(torch.bfloat16)
    ctxmod.set_context(True, c.to(dev), c.to(dev), 128, 128,
                       torch.empty(0, dtype=torch.int32, device=dev), None, None)
    out = attn(q.to(dev), k.to(dev), k.to(dev))
    ref = R.varlen_attention(q, k, k, c.numpy(), c.numpy(), D ** -0.5, True)
    assert_close(out, ref)
    ctxmod.reset_context()
    del lens
