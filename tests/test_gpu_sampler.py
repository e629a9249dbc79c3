"""One-pass sampler on the GPU (Sampler.forward, sampler.py:5-12).

Greedy rows are bit-exact against torch.argmax. Sampled rows follow the
reference's law softmax(logits / T) (chi-square against the exact
probabilities, and against the reference's own Sampler when importable), and
the noise stream is pinned to the Philox4x32-10 oracle: with equal logits the
pick is the column whose noise word is largest.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import reference_math as R

from nvattn import ops

pytestmark = pytest.mark.gpu
dev = torch.device("cuda")


@pytest.mark.parametrize("B,V,strided", [(1, 151936, False), (256, 151936, False),
                                         (7, 1000, False), (33, 4097, True), (5, 3, False)])
def test_greedy_matches_torch_argmax(B, V, strided):
    g = torch.Generator(device=dev).manual_seed(B * 7 + V)
    full = torch.randn(B, V + (5 if strided else 0), generator=g, device=dev).to(torch.bfloat16)
    logits = full[:, 1:V + 1] if strided else full
    # ties: copy each row's max to a later column, and a -inf column
    m = logits.float().argmax(-1)
    for r in range(B):
        j = int(m[r])
        if j + 1 < V:
            logits[r, V - 1] = logits[r, j]
        logits[r, 0] = float("-inf")
    got = ops.sample(logits)
    torch.cuda.synchronize()
    assert torch.equal(got, R.greedy_tokens(logits.cpu()).to(dev))
    t = torch.zeros(B, dtype=torch.float32, device=dev)  # T <= 0 -> greedy too
    assert torch.equal(ops.sample(logits, t), got)


@pytest.mark.parametrize("V", [64, 1003, 151936])
def test_equal_logits_pick_the_largest_noise_word(V):
    B, seed, offset = 6, 0x1234_5678_9abc_def0, 77
    logits = torch.zeros(B, V, dtype=torch.bfloat16, device=dev)
    t = torch.ones(B, dtype=torch.float32, device=dev)
    got = ops.sample(logits, t, seed=seed, offset=offset).cpu().numpy()
    for r in range(B):
        words = R.sample_uniforms(r, V, seed, offset)
        # the kernel keeps the top 23 bits of each word before the monotone
        # Gumbel transform: the pick holds the largest of them
        top = words >> 9
        assert top[got[r]] == top.max()


@pytest.mark.parametrize("T", [0.5, 1.0, 2.0])
def test_sampling_law_chi_square(T):
    torch.manual_seed(0)
    V, B = 12, 200000
    base = torch.tensor([3.0, 2.5, 2.0, 1.0, 0.0, -1.0, 0.5, 1.5, -3.0, 2.9, -10.0, 0.25])
    logits = base.to(torch.bfloat16).to(dev).expand(B, V).contiguous()
    t = torch.full((B,), T, dtype=torch.float32, device=dev)
    picks = ops.sample(logits, t, seed=42, offset=int(T * 10))
    counts = torch.bincount(picks, minlength=V).double().cpu()
    p = R.sample_probs(logits[:1].cpu(), T)[0].double()
    expected = p * B
    keep = expected > 5
    chi2 = (((counts - expected) ** 2) / expected)[keep].sum().item()
    dof = int(keep.sum()) - 1
    # p-value ~1e-6 threshold for chi-square with <= 11 dof
    assert chi2 < 45.0, (chi2, dof)
    assert counts[~keep].sum() < 50


def test_mixed_rows_and_determinism():
    B, V = 64, 5000
    g = torch.Generator(device=dev).manual_seed(9)
    logits = torch.randn(B, V, generator=g, device=dev).to(torch.bfloat16)
    t = torch.rand(B, generator=g, device=dev) + 0.5
    t[::4] = 0.0  # greedy rows
    a = ops.sample(logits, t, seed=5, offset=1)
    b = ops.sample(logits, t, seed=5, offset=1)
    c = ops.sample(logits, t, seed=5, offset=2)
    assert torch.equal(a, b)
    assert torch.equal(a[::4], R.greedy_tokens(logits[::4].cpu()).to(dev))
    assert not torch.equal(a, c)


def test_law_matches_reference_sampler():
    """Against the reference's own Sampler (torch.compile'd, run here)."""
    sampler_mod = pytest.importorskip("nanovllm.layers.sampler")
    V, B, T = 10, 100000, 0.8
    base = torch.tensor([1.0, 0.5, 0.0, 2.0, -1.0, 1.5, 0.2, -0.5, 0.9, 1.2])
    logits = base.to(torch.bfloat16).to(dev).expand(B, V).contiguous()
    t = torch.full((B,), T, dtype=torch.float32, device=dev)
    ours = torch.bincount(ops.sample(logits, t, seed=3, offset=0), minlength=V).double().cpu()
    ref = torch.bincount(sampler_mod.Sampler()(logits, t), minlength=V).double().cpu()
    # two-sample chi-square
    tot = ours + ref
    chi2 = (((ours - ref) ** 2) / tot.clamp_min(1)).sum().item()
    assert chi2 < 40.0, chi2


def _mixed_rows(B, V, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    logits = (torch.randn(B, V, generator=g, device=dev) * 2).to(torch.bfloat16)
    t = torch.rand(B, generator=g, device=dev) + 0.5
    t[::3] = 0.0                      # greedy rows
    if B > 4:
        logits[1] = float("-inf")     # no candidate: column 0
        logits[2, ::2] = float("nan")
        logits[4, V // 2:] = logits[4].max()  # a tie that spans shard borders
    return logits, t


@pytest.mark.parametrize("B,V,cuts", [(256, 151936, [75968]),
                                      (33, 151936, [18992, 37984, 75968, 113952]),
                                      (7, 1003, [1, 498, 998]),      # unaligned: scalar path
                                      (9, 5000, [2504]), (1, 151936, [8, 151928])])
def test_vocab_shards_merge_to_the_whole_row_pick(B, V, cuts):
    """Tensor-parallel LM head (embed_head.py:56-66): each shard's keys,
    merged, give the token the one-pass sampler gives on the gathered row,
    bit for bit, for sampled and greedy rows alike."""
    logits, t = _mixed_rows(B, V, B * 31 + V)
    seed, offset = 0xABCDEF0123, 17
    whole = ops.sample(logits, t, seed=seed, offset=offset)
    bounds = [0] + cuts + [V]
    keys = torch.stack([ops.sample_shard(logits[:, a:b], a, t, seed=seed, offset=offset)
                        for a, b in zip(bounds[:-1], bounds[1:])])
    merged = ops.sample_merge(keys)
    torch.cuda.synchronize()
    assert torch.equal(merged, whole)
    # greedy rows: every shard key equals the oracle's key bit for bit
    gr = (t <= 0).nonzero().flatten().cpu()
    for s, (a, b) in enumerate(zip(bounds[:-1], bounds[1:])):
        want = R.greedy_shard_keys(logits[:, a:b].cpu()[gr], a)
        assert np.array_equal(keys[s].cpu()[gr].numpy().view(np.uint64), want)
    if B > 4:
        assert whole[1].item() == 0
    lf = logits.float()
    greedy_whole = R.greedy_tokens(torch.where(torch.isnan(lf), float("-inf"), lf).cpu())
    assert torch.equal(whole.cpu()[gr], greedy_whole[gr])


@pytest.mark.parametrize("V,cut", [(1000, 504), (151936, 75968), (4099, 2050)])
def test_shard_noise_is_indexed_by_global_column(V, cut):
    B, seed, offset = 4, 0x1234_5678_9abc_def0, 5
    logits = torch.zeros(B, V, dtype=torch.bfloat16, device=dev)
    t = torch.ones(B, dtype=torch.float32, device=dev)
    keys = torch.stack([ops.sample_shard(logits[:, :cut], 0, t, seed=seed, offset=offset),
                        ops.sample_shard(logits[:, cut:], cut, t, seed=seed, offset=offset)])
    got = ops.sample_merge(keys).cpu().numpy()
    for r in range(B):
        top = R.sample_uniforms(r, V, seed, offset) >> 9
        assert top[got[r]] == top.max()


def test_sample_and_merge_capture_in_a_cuda_graph():
    B, V = 64, 151936
    logits, t = _mixed_rows(B, V, 3)
    out = torch.empty(B, dtype=torch.int64, device=dev)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        ops.sample(logits, t, seed=9, offset=1, out=out)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        ops.sample(logits, t, seed=9, offset=1, out=out)
    for trial in range(3):
        new, _ = _mixed_rows(B, V, 100 + trial)
        logits.copy_(new)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ops.sample(logits, t, seed=9, offset=1))
    del graph


def test_skipped_vectors_never_hold_the_pick():
    """Sampled rows skip the noise of any 8-column vector whose largest logit
    / T plus the noise bound is below the thread's best. With 256 rows of
    151,936 columns each thread scans about four vectors. Every 16th column
    is live (logit 0), the rest are at -100: once a thread has seen a live
    column it skips the dead vectors. The pick must be the live column with
    the largest noise word, for the whole row and for shards alike."""
    B, V, cut, seed, offset = 256, 151936, 75968, 77, 3
    logits = torch.full((B, V), -100.0, dtype=torch.bfloat16, device=dev)
    for r in range(B):
        logits[r, r % 16::16] = 0.0
    t = torch.ones(B, dtype=torch.float32, device=dev)
    whole = ops.sample(logits, t, seed=seed, offset=offset).cpu().numpy()
    keys = torch.stack([ops.sample_shard(logits[:, :cut], 0, t, seed=seed, offset=offset),
                        ops.sample_shard(logits[:, cut:], cut, t, seed=seed, offset=offset)])
    merged = ops.sample_merge(keys).cpu().numpy()
    for r in range(B):
        top = R.sample_uniforms(r, V, seed, offset) >> 9
        cols = np.arange(r % 16, V, 16)
        want = cols[top[cols] == top[cols].max()].min()
        assert whole[r] == want and merged[r] == want, r
