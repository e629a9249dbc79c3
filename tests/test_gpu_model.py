"""nvattn inside the reference's own Qwen3 model (configs[1] architecture).

The model (nanovllm/models/qwen3.py) is built once with random weights and
run three times on the same token sequences: with the reference's attention
(Triton scatter + flash-attn), with nvattn.Attention swapped into every
layer, and with q/k RMSNorm + rotary + scatter also fused into one nvattn
kernel (``install(fuse_qk_norm_rope=True)``). Decode steps are teacher-forced with the reference's greedy tokens, so
both runs see identical inputs and differences cannot cascade. Per step the
logits must agree: cosine similarity > 0.999, and the greedy token must match
wherever the reference's top-2 margin exceeds the bf16 noise of the logits.

Skipped when the reference engine is not importable (it lives in
baseline/_ref when installed).
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
nanovllm = pytest.importorskip("nanovllm")
pytest.importorskip("flash_attn")


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_teacher_forced_logits_match_reference_attention():
    import torch.distributed as dist
    from transformers import Qwen3Config

    import nvattn
    from nanovllm.layers.attention import Attention as RefAttention
    from nanovllm.models.qwen3 import Qwen3ForCausalLM
    from nanovllm.utils.context import reset_context, set_context
    from oracle import reference_math as R

    own_pg = not dist.is_initialized()
    if own_pg:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        os.environ["MASTER_PORT"] = str(_port())
        dist.init_process_group("gloo", rank=0, world_size=1)
    dev = torch.device("cuda")
    cfg = Qwen3Config(hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                      num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                      vocab_size=151936, max_position_embeddings=40960, rms_norm_eps=1e-6,
                      rope_theta=1000000.0, tie_word_embeddings=True, attention_bias=False,
                      dtype="bfloat16")
    prev_dtype = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    torch.set_default_device(dev)
    try:
        model = Qwen3ForCausalLM(cfg)
    finally:
        torch.set_default_device("cpu")
        torch.set_default_dtype(prev_dtype)
    g = torch.Generator(device=dev).manual_seed(0)
    with torch.no_grad():
        for name, prm in model.named_parameters():
            if prm.dim() == 1:
                prm.copy_(1.0 + 0.1 * torch.randn(prm.shape, generator=g, device=dev))
            else:
                prm.copy_(0.02 * torch.randn(prm.shape, generator=g, device=dev))

    BS, L, KVH, D = 256, 28, 8, 128
    rng = np.random.default_rng(0)
    lens = [37, 200, 513, 1024]
    steps = 16
    prompts = [rng.integers(0, 10000, size=n).tolist() for n in lens]
    tables, nxt = [], 0
    for n in lens:
        nb = (n + steps + BS - 1) // BS
        tables.append(list(range(nxt, nxt + nb)))
        nxt += nb
    kv = torch.zeros(2, L, nxt, BS, KVH, D, dtype=torch.bfloat16, device=dev)
    attn_modules = [m for m in model.modules() if isinstance(m, RefAttention)]
    assert len(attn_modules) == L
    for i, m in enumerate(attn_modules):
        m.k_cache, m.v_cache = kv[0, i], kv[1, i]

    def to(x):
        return torch.as_tensor(np.asarray(x), device=dev)

    def run(forced):
        """Prefill + `steps` decode steps; returns per-step logits (fp32, cpu)."""
        kv.zero_()
        out = []
        seqs = [dict(start=0, num_scheduled=n, num_tokens=n, block_table=t[:(n + BS - 1) // BS])
                for n, t in zip(lens, tables)]
        cu_q, cu_k, mq, mk, slots, _ = R.prepare_prefill_metadata(seqs, BS)
        ids = torch.tensor(sum(prompts, []), dtype=torch.int64, device=dev)
        pos = torch.tensor(sum([list(range(n)) for n in lens], []), dtype=torch.int64,
                           device=dev)
        with torch.inference_mode():
            set_context(True, to(cu_q), to(cu_k), mq, mk, to(slots), None, None)
            out.append(model.compute_logits(model(ids, pos)).float().cpu())
            for s in range(steps):
                toks = forced[s] if forced is not None else out[-1].argmax(-1).tolist()
                seqs_d = [dict(num_tokens=n + s + 1, block_table=t[:(n + s + 1 + BS - 1) // BS])
                          for n, t in zip(lens, tables)]
                slots, ctx_lens, bt = R.prepare_decode_metadata(seqs_d, BS)
                set_context(False, slot_mapping=to(slots), context_lens=to(ctx_lens),
                            block_tables=to(bt))
                ids = torch.tensor(toks, dtype=torch.int64, device=dev)
                pos = torch.tensor([n + s for n in lens], dtype=torch.int64, device=dev)
                out.append(model.compute_logits(model(ids, pos)).float().cpu())
        reset_context()
        return out

    ref = run(None)
    forced = [ref[s].argmax(-1).tolist() for s in range(steps)]
    saved_ctx = nvattn.Attention.__dict__["get_context"]  # the staticmethod object
    nvattn.install()  # nvattn.Attention reads the engine's context
    try:
        for m in attn_modules:
            m.__class__ = nvattn.Attention
        ours = run(forced)
        # q/k norm + rotary + KV scatter fused into one kernel (qwen3.py:82-86)
        nvattn.install(fuse_qk_norm_rope=True)
        fused = run(forced)
    finally:
        nvattn.install(fuse_qk_norm_rope=False)
        nvattn.Attention.get_context = saved_ctx
    # the fused kernel rounds the RMSNorm reduction in its own fixed order, so
    # fused and unfused runs differ like any two reduction orders (28 layers)
    for a, b in zip(ours, fused):
        assert torch.nn.functional.cosine_similarity(a, b, dim=-1).min() > 0.999
    _check_against_reference(ref, fused, steps, lens)
    _check_against_reference(ref, ours, steps, lens)
    assert nvattn.ops.read_status() == 0
    if own_pg:
        dist.destroy_process_group()


def _check_against_reference(ref, ours, steps, lens):
    checked = 0
    for s, (a, b) in enumerate(zip(ref, ours)):
        cos = torch.nn.functional.cosine_similarity(a, b, dim=-1)
        assert cos.min() > 0.999, (s, cos.min().item())
        top2 = a.topk(2, dim=-1).values
        margin = top2[:, 0] - top2[:, 1]
        # logits are bf16 (the LM head runs in bf16): 4 ulps of the largest one
        noise = a.abs().amax(dim=-1) * 2.0 ** -6
        decisive = margin > noise
        checked += int(decisive.sum())
        assert torch.equal(a.argmax(-1)[decisive], b.argmax(-1)[decisive]), s
    print(f"decisive rows checked: {checked} of {(steps + 1) * len(lens)}; min cosine "
          f"{min(torch.nn.functional.cosine_similarity(a, b, dim=-1).min().item() for a, b in zip(ref, ours)):.6f}")
    assert checked >= (steps + 1) * len(lens) // 4
