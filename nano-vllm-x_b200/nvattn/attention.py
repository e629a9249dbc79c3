"""Drop-in replacement for ``nanovllm.layers.attention.Attention``.

Constructor, attributes and ``forward(q, k, v)`` follow
nanovllm/layers/attention.py:43-75 exactly:

* ``k_cache``/``v_cache`` start as empty tensors and are rebound by
  ``ModelRunner.allocate_kv_cache`` (model_runner.py:117-121), which finds
  the module through ``hasattr(module, "k_cache")``;
* ``forward`` reads only the attention context: it scatters the new K/V into
  the cache when one is bound (attention.py:61-63), then runs varlen prefill
  — over the caches when ``block_tables`` is set, i.e. a prefix-cache hit
  (attention.py:64-70) — or paged decode (attention.py:71-74);
* outputs have the reference's shapes: (N, H, d) for prefill and
  (B, 1, H, d) for decode.

``forward_fused`` is the same step with the producer side folded in: it
takes the raw q/k/v split of the QKV projection plus the RMSNorm weights and
the rotary cache, and one kernel applies q_norm/k_norm and the rotation and
scatters K/V (qwen3.py:82-86 and attention.py:62-63) before the attention.

All steps run libnvattn kernels; there is no other code path.
"""
from __future__ import annotations

import torch
from torch import nn

from . import context as _ctx
from . import ops


class Attention(nn.Module):
    # Source of the per-step context; ``nvattn.install`` points this at the
    # host engine's context module so both read the same global.
    get_context = staticmethod(_ctx.get_context)

    def __init__(self, num_heads, head_dim, scale, num_kv_heads):
        super().__init__()
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.scale = scale
        self.num_kv_heads = num_kv_heads
        self.k_cache = self.v_cache = torch.tensor([])

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor):
        context = self.get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        if k_cache.numel() and v_cache.numel():
            ops.store_kvcache(k, v, k_cache, v_cache, context.slot_mapping)
        return self._attend(context, q, k, v)

    def forward_fused(self, positions: torch.Tensor, q: torch.Tensor, k: torch.Tensor,
                      v: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                      cos_sin_cache: torch.Tensor, eps: float):
        """q_norm/k_norm + rotary_emb + KV scatter in one kernel, then attention.

        q, k, v are the un-normalised split of the QKV projection
        (qwen3.py:79-81); the result equals ``forward`` applied to the
        normalised, rotated q and k (qwen3.py:82-86).
        """
        context = self.get_context()
        k_cache, v_cache = self.k_cache, self.v_cache
        bound = bool(k_cache.numel() and v_cache.numel())
        # the rotated K itself is read only by dense prefill; the other paths
        # read K back from the cache
        need_k = bool(context.is_prefill and context.block_tables is None)
        q, k = ops.qk_norm_rope_store(positions, q, k, v, q_weight, k_weight, cos_sin_cache, eps,
                                      k_cache if bound else None, v_cache if bound else None,
                                      context.slot_mapping if bound else None, need_k=need_k)
        return self._attend(context, q, k, v)

    def _attend(self, context, q: torch.Tensor, k, v):
        k_cache, v_cache = self.k_cache, self.v_cache
        if context.is_prefill:
            if context.block_tables is not None:  # prefix cache
                k, v = k_cache, v_cache
            o = ops.varlen_prefill(q, k, v, context.cu_seqlens_q, context.cu_seqlens_k,
                                   context.max_seqlen_q, context.max_seqlen_k,
                                   softmax_scale=self.scale, causal=True,
                                   block_table=context.block_tables)
        else:  # decode
            o = ops.paged_decode(q, k_cache, v_cache, context.context_lens,
                                 context.block_tables, softmax_scale=self.scale).unsqueeze(1)
        return o
