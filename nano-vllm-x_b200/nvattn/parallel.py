"""Head sharding of the attention path across tensor-parallel ranks.

Nano-vLLM-X splits attention by head (nanovllm/models/qwen3.py:29-35): with
tp ranks, rank r owns query heads [r*H/tp, (r+1)*H/tp) and KV heads
[r*KVH/tp, (r+1)*KVH/tp) (the QKV weight loader takes chunk r of each
projection, linear.py:131-149), and its KV cache holds only its KV heads
(model_runner.py:110). Attention itself needs no collective: each rank runs
the kernels on its own shard.

The LM head splits the vocabulary instead (embed_head.py:17-23): rank r
holds logits for columns [r*V/tp, (r+1)*V/tp) and the reference gathers all
of them to rank 0 before sampling (embed_head.py:62-65). Here each rank picks
within its own columns (``nvattn.ops.sample_shard``) and the ranks exchange
one 64-bit key per row; the merge gives the same token as sampling the
gathered row.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def head_shard(num_heads: int, num_kv_heads: int, rank: int, world_size: int):
    """Return ((q_begin, q_end), (kv_begin, kv_end)) for this rank."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("bad rank/world_size")
    if num_heads % world_size or num_kv_heads % world_size:
        raise ValueError("heads must divide evenly across ranks (qwen3.py:31,34)")
    hq = num_heads // world_size
    hk = num_kv_heads // world_size
    return (rank * hq, (rank + 1) * hq), (rank * hk, (rank + 1) * hk)


def vocab_shard(vocab: int, rank: int, world_size: int):
    """Return (begin, end) of this rank's vocabulary columns (embed_head.py:17-23)."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("bad rank/world_size")
    if vocab % world_size:
        raise ValueError("the vocabulary must divide evenly across ranks (embed_head.py:19)")
    n = vocab // world_size
    return rank * n, (rank + 1) * n


def gather_pick_keys(keys: torch.Tensor, group=None) -> torch.Tensor:
    """(B,) int64 pick keys of this rank -> (world, B) keys of every rank,
    with one all-gather of B x 8 bytes (instead of B x V/tp logits)."""
    world = dist.get_world_size(group)
    flat = torch.empty(world * keys.numel(), dtype=keys.dtype, device=keys.device)
    dist.all_gather_into_tensor(flat, keys.contiguous(), group=group)
    return flat.view(world, keys.numel())


def sample_vocab_parallel(logits_local: torch.Tensor, temperatures: torch.Tensor | None = None, *,
                          vocab_offset: int, seed: int, offset: int, group=None) -> torch.Tensor:
    """Tokens for (B, V/tp) bf16 logits of this rank's vocabulary shard.

    Every rank calls it with the same ``seed``, ``offset`` and temperatures;
    every rank gets the (B,) int64 tokens, equal to ``nvattn.ops.sample`` on
    the gathered (B, V) logits with that seed and offset.
    """
    from . import ops
    keys = ops.sample_shard(logits_local, vocab_offset, temperatures, seed=seed, offset=offset)
    return ops.sample_merge(gather_pick_keys(keys, group))
