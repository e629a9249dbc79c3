"""Seeded input builders shared by the GPU parity tests."""
from __future__ import annotations

import numpy as np
import torch

D = 128


def paged_layout(lens, block_size=256, extra_blocks=2, seed=0, permute=True):
    """Block tables (padded with -1) for sequences of `lens` tokens over a
    shared pool of physical blocks; returns (num_blocks, tables int32 tensor)."""
    rng = np.random.default_rng(seed)
    nblk = [max(1, (int(n) + block_size - 1) // block_size) for n in lens]
    total = sum(nblk) + extra_blocks
    ids = rng.permutation(total) if permute else np.arange(total)
    tables, pos = [], 0
    for n in nblk:
        tables.append(ids[pos:pos + n].tolist())
        pos += n
    width = max(nblk)
    bt = np.full((len(lens), width), -1, dtype=np.int32)
    for i, t in enumerate(tables):
        bt[i, :len(t)] = t
    return total, torch.from_numpy(bt)


def random_cache(num_blocks, block_size, nkv, gen, fill_nan=False):
    shape = (num_blocks, block_size, nkv, D)
    if fill_nan:
        return torch.full(shape, float("nan"), dtype=torch.bfloat16)
    return torch.randn(shape, generator=gen).to(torch.bfloat16)


def cu(lens):
    return torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32)


def max_err(a: torch.Tensor, b: torch.Tensor) -> float:
    return (a.float().cpu() - b.float().cpu()).abs().max().item()
