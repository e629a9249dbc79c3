"""Swap nvattn's Attention into a Nano-vLLM-X installation.

``install()`` replaces ``nanovllm.layers.attention.Attention`` and the name
``Attention`` bound inside ``nanovllm.models.qwen3`` (qwen3.py:7, used at
qwen3.py:64) by ``nvattn.Attention``, and makes it read the engine's own
context (nanovllm/utils/context.py), which ``ModelRunner.prepare_prefill``/
``prepare_decode`` fill. Call it before the engine builds its model.

``install(fuse_qk_norm_rope=True)`` also replaces ``Qwen3Attention.forward``
(qwen3.py:76-88) by a version whose q_norm/k_norm, rotary_emb and KV scatter
run as one nvattn kernel (``Attention.forward_fused``); the QKV and output
projections are the module's own.
"""
from __future__ import annotations

import importlib

from .attention import Attention


def _fused_qwen3_attention_forward(self, positions, hidden_states):
    """Qwen3Attention.forward (qwen3.py:76-88) with steps 82-86 fused."""
    if self.qkv_bias or not isinstance(self.attn, Attention):
        return _ORIGINAL["qwen3_attention_forward"](self, positions, hidden_states)
    qkv = self.qkv_proj(hidden_states)
    q, k, v = qkv.split([self.q_size, self.kv_size, self.kv_size], dim=-1)
    q = q.view(-1, self.num_heads, self.head_dim)
    k = k.view(-1, self.num_kv_heads, self.head_dim)
    v = v.view(-1, self.num_kv_heads, self.head_dim)
    o = self.attn.forward_fused(positions, q, k, v, self.q_norm.weight, self.k_norm.weight,
                                self.rotary_emb.cos_sin_cache, self.q_norm.eps)
    return self.o_proj(o.flatten(1, -1))


_ORIGINAL: dict = {}


def install(fuse_qk_norm_rope: bool = False) -> None:
    ctx_mod = importlib.import_module("nanovllm.utils.context")
    attn_mod = importlib.import_module("nanovllm.layers.attention")
    Attention.get_context = staticmethod(lambda: ctx_mod.get_context())
    attn_mod.Attention = Attention
    try:
        qwen3 = importlib.import_module("nanovllm.models.qwen3")
    except ImportError:
        return
    qwen3.Attention = Attention
    cls = qwen3.Qwen3Attention
    _ORIGINAL.setdefault("qwen3_attention_forward", cls.forward)
    cls.forward = (_fused_qwen3_attention_forward if fuse_qk_norm_rope
                   else _ORIGINAL["qwen3_attention_forward"])
