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


# Attention-output tolerance: max-abs 1e-2 between the kernel output and the
# fp32-accumulated reference, beyond the output's own final rounding to bf16:
# |out - ref| <= 1e-2 + half a bf16 ulp of ref. The half ulp is 2^(e-8) for
# |ref| in [2^e, 2^(e+1)): 0.0039 below 2, 0.0078 in [2, 4). Rows with one or
# two visible keys reach |o| of 2-4 (o is then a mix of one or two N(0,1) V
# rows), and there a kernel that feeds P to the tensor cores as bf16 (as
# flash-attn does) differs from the fp32 reference by up to ~2^-9 |v| from P's
# rounding plus the output's half ulp. Every check prints its margin.
ATOL = 1e-2


def half_ulp_bf16(x: torch.Tensor) -> torch.Tensor:
    """Half the spacing of bf16 numbers at |x| (8 significant bits)."""
    ax = x.abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(ax)) - 8)


def excess(a: torch.Tensor, b: torch.Tensor) -> float:
    """max(|a - b| - (ATOL + half_ulp(b))); <= 0 means within tolerance."""
    a = a.float().cpu()
    b = b.float().cpu()
    return ((a - b).abs() - (ATOL + half_ulp_bf16(b))).max().item()


def assert_close(a: torch.Tensor, b: torch.Tensor, what: str = "") -> None:
    err = max_err(a, b)
    ex = excess(a, b)
    print(f"[max-abs] {what or 'attention output'}: {err:.3e} (bound 1e-2 + half ulp; "
          f"margin {-ex:.3e})")
    assert ex <= 0, f"{what}: max-abs error {err:.4g} exceeds 1e-2 + half a bf16 ulp by {ex:.3g}"
