"""Head sharding of the attention path across tensor-parallel ranks.

Nano-vLLM-X splits attention by head (nanovllm/models/qwen3.py:29-35): with
tp ranks, rank r owns query heads [r*H/tp, (r+1)*H/tp) and KV heads
[r*KVH/tp, (r+1)*KVH/tp) (the QKV weight loader takes chunk r of each
projection, linear.py:131-149), and its KV cache holds only its KV heads
(model_runner.py:110). Attention itself needs no collective: each rank runs
the kernels on its own shard.
"""
from __future__ import annotations


def head_shard(num_heads: int, num_kv_heads: int, rank: int, world_size: int):
    """Return ((q_begin, q_end), (kv_begin, kv_end)) for this rank."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError("bad rank/world_size")
    if num_heads % world_size or num_kv_heads % world_size:
        raise ValueError("heads must divide evenly across ranks (qwen3.py:31,34)")
    hq = num_heads // world_size
    hk = num_kv_heads // world_size
    return (rank * hq, (rank + 1) * hq), (rank * hk, (rank + 1) * hk)
