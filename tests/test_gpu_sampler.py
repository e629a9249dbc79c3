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
        # the kernel keeps the top 24 bits of each word before the monotone
        # Gumbel transform: the pick holds the largest of them
        top = words >> 8
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
