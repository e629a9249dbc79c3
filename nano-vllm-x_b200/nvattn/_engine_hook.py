"""Swap nvattn's Attention into a Nano-vLLM-X installation.

``install()`` replaces ``nanovllm.layers.attention.Attention`` and the name
``Attention`` bound inside ``nanovllm.models.qwen3`` (qwen3.py:7, used at
qwen3.py:64) by ``nvattn.Attention``, and makes it read the engine's own
context (nanovllm/utils/context.py), which ``ModelRunner.prepare_prefill``/
``prepare_decode`` fill. Call it before the engine builds its model.
"""
from __future__ import annotations

import importlib

from .attention import Attention


def install() -> None:
    ctx_mod = importlib.import_module("nanovllm.utils.context")
    attn_mod = importlib.import_module("nanovllm.layers.attention")
    Attention.get_context = staticmethod(lambda: ctx_mod.get_context())
    attn_mod.Attention = Attention
    try:
        qwen3 = importlib.import_module("nanovllm.models.qwen3")
        qwen3.Attention = Attention
    except ImportError:
        pass
