"""Fused q/k RMSNorm + rotary + KV scatter on the GPU.

The kernel uses the oracle's fixed fp32 operation order, so outputs and the
cache are compared bit for bit. Against the reference's own modules (golden
fixture) the same at-most-1-ulp bound as the oracle holds.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN, bf16_bits, from_bits
from oracle import reference_math as R

from nvattn import _lib, ops

pytestmark = pytest.mark.gpu
dev = torch.device("cuda")


def _split(qkv: torch.Tensor, H: int, KVH: int, d: int = 128):
    q, k, v = qkv.split([H * d, KVH * d, KVH * d], dim=-1)
    return q.view(-1, H, d), k.view(-1, KVH, d), v.view(-1, KVH, d)


def test_golden_bit_exact_vs_oracle_and_within_1ulp_of_reference():
    g = np.load(GOLDEN / "qk_norm_rope_ref.npz")
    N, H, KVH, D, max_pos = (int(x) for x in g["meta"])
    qkv = from_bits(g["qkv"]).to(dev)
    q, k, v = _split(qkv, H, KVH, D)
    cache = R.rope_cache(D, max_pos, float(g["theta"])).to(dev)
    pos = torch.from_numpy(g["positions"]).to(dev)
    qw, kw = from_bits(g["q_weight"]).to(dev), from_bits(g["k_weight"]).to(dev)
    q_rot, k_rot = ops.qk_norm_rope_store(pos, q, k, v, qw, kw, cache, float(g["eps"]))
    torch.cuda.synchronize()
    q_np = g["qkv"][:, :H * D].reshape(N, H, D)
    k_np = g["qkv"][:, H * D:(H + KVH) * D].reshape(N, KVH, D)
    eq, ek = R.qk_norm_rope_store(g["positions"], q_np, k_np, None, g["q_weight"], g["k_weight"],
                                  cache.cpu().numpy(), float(g["eps"]))
    assert np.array_equal(bf16_bits(q_rot), eq)
    assert np.array_equal(bf16_bits(k_rot), ek)
    for out, ref in ((q_rot, g["q_rot"]), (k_rot, g["k_rot"])):
        ulp = np.abs(bf16_bits(out).astype(np.int32) - ref.astype(np.int32))
        assert ulp.max() <= 1 and (ulp > 0).mean() <= 1e-4
    assert ops.read_status() == 0


@pytest.mark.parametrize("N,H,KVH,frac_skip", [(1, 16, 8, 0.0), (37, 16, 8, 0.2),
                                               (1000, 32, 8, 0.1), (4096, 64, 8, 0.0),
                                               (300, 2, 1, 0.5), (16384, 16, 8, 0.05)])
def test_random_bit_exact_with_scatter(N, H, KVH, frac_skip):
    gen = torch.Generator().manual_seed(N + 7 * H)
    d, bs = 128, 256
    nb = (N + bs - 1) // bs + 2
    max_pos = 40960
    qkv = (torch.randn(N, (H + 2 * KVH) * d, generator=gen) * 3).to(torch.bfloat16)
    pos = torch.randint(0, max_pos, (N,), generator=gen, dtype=torch.int64)
    slots = torch.randperm(nb * bs, generator=gen)[:N].to(torch.int32)
    slots[torch.rand(N, generator=gen) < frac_skip] = -1
    qw = (1 + 0.1 * torch.randn(d, generator=gen)).to(torch.bfloat16)
    kw = (1 + 0.1 * torch.randn(d, generator=gen)).to(torch.bfloat16)
    kc0 = torch.randn(nb, bs, KVH, d, generator=gen).to(torch.bfloat16)
    vc0 = torch.randn(nb, bs, KVH, d, generator=gen).to(torch.bfloat16)
    cache = R.rope_cache(d, max_pos, 1e6)
    q, k, v = _split(qkv.to(dev), H, KVH)
    kc, vc = kc0.to(dev), vc0.to(dev)
    q_rot, k_rot = ops.qk_norm_rope_store(pos.to(dev), q, k, v, qw.to(dev), kw.to(dev),
                                          cache.to(dev), 1e-6, kc, vc, slots.to(dev))
    torch.cuda.synchronize()
    qn, kn, vn = _split(qkv, H, KVH)
    ek_cache, ev_cache = bf16_bits(kc0), bf16_bits(vc0)
    eq, ek = R.qk_norm_rope_store(pos.numpy(), bf16_bits(qn), bf16_bits(kn), bf16_bits(vn),
                                  bf16_bits(qw), bf16_bits(kw), cache.numpy(), 1e-6,
                                  ek_cache, ev_cache, slots.numpy())
    assert np.array_equal(bf16_bits(q_rot), eq)
    assert np.array_equal(bf16_bits(k_rot), ek)
    assert np.array_equal(bf16_bits(kc), ek_cache)
    assert np.array_equal(bf16_bits(vc), ev_cache)
    assert ops.read_status() == 0


def test_edge_cases_flags_and_optional_outputs():
    d, H, KVH, N = 128, 8, 2, 5
    gen = torch.Generator().manual_seed(3)
    qkv = torch.randn(N, (H + 2 * KVH) * d, generator=gen).to(torch.bfloat16).to(dev)
    q, k, v = _split(qkv, H, KVH)
    cache = R.rope_cache(d, 64, 1e6).to(dev)
    w = torch.ones(d, dtype=torch.bfloat16, device=dev)
    kc = torch.zeros(2, 16, KVH, d, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    ops.read_status()
    # no scatter, no k output
    q_rot, k_rot = ops.qk_norm_rope_store(torch.arange(N, device=dev), q, k, v, w, w, cache, 1e-6,
                                          need_k=False)
    assert k_rot is None and ops.read_status() == 0
    # positions outside the cache are clamped and flagged; bad slots skipped and flagged
    pos = torch.tensor([0, 63, 64, -1, 5], device=dev)
    slots = torch.tensor([0, 31, 32, -1, -7], dtype=torch.int32, device=dev)
    ops.qk_norm_rope_store(pos, q, k, v, w, w, cache, 1e-6, kc, vc, slots)
    st = ops.read_status()
    assert st & _lib.STATUS_BAD_POSITION and st & _lib.STATUS_BAD_SLOT
    assert kc.view(-1, KVH * d)[0].abs().sum() > 0 and kc.view(-1, KVH * d)[31].abs().sum() > 0
    # empty batch
    e = qkv[:0]
    qe, ke, ve = _split(e, H, KVH)
    q0, k0 = ops.qk_norm_rope_store(torch.zeros(0, dtype=torch.int64, device=dev), qe, ke, ve, w, w,
                                    cache, 1e-6, kc, vc, torch.zeros(0, dtype=torch.int32, device=dev))
    assert q0.shape == (0, H, d) and k0.shape == (0, KVH, d)


def test_fused_decode_step_in_cuda_graph():
    """Attention.forward_fused in decode mode captured in a CUDA graph on static
    buffers (as ModelRunner.capture_cudagraph does, model_runner.py:222-257),
    replayed with new tokens, positions, slots and lengths; every replay equals
    the eager fused step, and the rotated K/V land in the cache."""
    import nvattn
    from nvattn import context as C

    H, KVH, d, bs, width, B = 16, 8, 128, 256, 4, 8
    nb = B * width
    gen = torch.Generator().manual_seed(21)
    kc = (torch.randn(nb, bs, KVH, d, generator=gen) * 0.5).to(torch.bfloat16).to(dev)
    vc = (torch.randn(nb, bs, KVH, d, generator=gen) * 0.5).to(torch.bfloat16).to(dev)
    cache = R.rope_cache(d, 4096, 1e6).to(dev)
    qw = (1 + 0.1 * torch.randn(d, generator=gen)).to(torch.bfloat16).to(dev)
    kw = (1 + 0.1 * torch.randn(d, generator=gen)).to(torch.bfloat16).to(dev)
    attn = nvattn.Attention(H, d, d ** -0.5, KVH)
    attn.k_cache, attn.v_cache = kc, vc
    # static graph inputs
    qkv = torch.zeros(B, (H + 2 * KVH) * d, dtype=torch.bfloat16, device=dev)
    pos = torch.zeros(B, dtype=torch.int64, device=dev)
    slots = torch.full((B,), -1, dtype=torch.int32, device=dev)
    lens = torch.zeros(B, dtype=torch.int32, device=dev)
    bt = torch.arange(nb, dtype=torch.int32, device=dev).view(B, width)

    def step():
        q, k, v = _split(qkv, H, KVH)
        return attn.forward_fused(pos, q, k, v, qw, kw, cache, 1e-6)

    saved = nvattn.Attention.__dict__["get_context"]
    try:
        nvattn.Attention.get_context = staticmethod(C.get_context)
        C.set_context(False, slot_mapping=slots, context_lens=lens, block_tables=bt)
        ops.status_tensor()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = step()
        for trial in range(3):
            rng = np.random.default_rng(50 + trial)
            n = rng.integers(1, width * bs, size=B)  # context length including the new token
            qkv.copy_((torch.randn(B, (H + 2 * KVH) * d, generator=gen)).to(torch.bfloat16))
            pos.copy_(torch.from_numpy(n - 1))
            slot_np = (np.arange(B) * width * bs + (n - 1)).astype(np.int32)
            slots.copy_(torch.from_numpy(slot_np))
            lens.copy_(torch.from_numpy(n.astype(np.int32)))
            kc_before = kc.clone()
            graph.replay()
            torch.cuda.synchronize()
            got = out.clone()
            k_graph = kc.clone()
            # eager fused step on the same inputs and the same starting cache
            kc.copy_(kc_before)
            want = step()
            torch.cuda.synchronize()
            assert torch.equal(got, want)
            assert torch.equal(k_graph, kc)
            # the new token's rotated K is in its slot (oracle, bit-exact)
            q_np = bf16_bits(qkv[:, :H * d].reshape(B, H, d))
            k_np = bf16_bits(qkv[:, H * d:(H + KVH) * d].reshape(B, KVH, d))
            _, ek = R.qk_norm_rope_store(n - 1, q_np, k_np, None, bf16_bits(qw), bf16_bits(kw),
                                         cache.cpu().numpy(), 1e-6)
            assert np.array_equal(bf16_bits(kc.view(-1, KVH, d)[torch.from_numpy(slot_np).long()]), ek)
        del graph
    finally:
        C.reset_context()
        nvattn.Attention.get_context = saved
    assert ops.read_status() == 0
