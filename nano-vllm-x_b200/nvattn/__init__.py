"""nvattn — B200 (sm_100a) paged-KV attention for Nano-vLLM-X.

Drop-in for nanovllm/layers/attention.py: ``Attention`` (same constructor and
``forward(q, k, v)``), the context module mirror, and the operators that
replace the reference's Triton scatter and flash-attn calls. Kernels live in
the in-tree ``libnvattn.so`` (C ABI: include/nvattn.h); build it with
``python -m nvattn.build``.
"""
from .attention import Attention
from .context import Context, get_context, reset_context, set_context
from . import ops, tree, parallel, decode_meta
from .decode_meta import DecodeMetadata
from .ops import (flash_attn_varlen_func, flash_attn_with_kvcache, kv_move, paged_decode,
                  qk_norm_rope_store, sample, sample_merge, sample_shard, store_kvcache,
                  tree_attention, varlen_prefill)

__all__ = [
    "Attention", "Context", "get_context", "set_context", "reset_context", "ops", "tree",
    "parallel", "store_kvcache", "varlen_prefill", "paged_decode", "tree_attention", "kv_move",
    "flash_attn_varlen_func", "flash_attn_with_kvcache", "qk_norm_rope_store", "sample",
    "sample_shard", "sample_merge", "DecodeMetadata", "decode_meta", "install",
]


def install(fuse_qk_norm_rope: bool = False) -> None:
    """Replace Nano-vLLM-X's Attention with nvattn's (see nvattn._engine_hook);
    with ``fuse_qk_norm_rope`` also fuse Qwen3's q/k norm, rotary and KV scatter."""
    from ._engine_hook import install as _install
    _install(fuse_qk_norm_rope)
