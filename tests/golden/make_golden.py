"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run in a container where the reference source tree is readable (it is NOT
needed afterwards: tests read only the committed fixtures):

    python tests/golden/make_golden.py --reference <path-to-Nano-vLLM-X>

Produces, next to this script:

* store_kvcache_triton.npz — the reference's own Triton kernel
  ``store_kvcache_kernel`` (nanovllm/layers/attention.py:10-40) executed
  with TRITON_INTERPRET=1 on seeded bf16 inputs: K contiguous, V a strided
  view of a qkv projection (as in qwen3.py:78-81), random unique slots with
  two -1 entries. Inputs and the resulting caches (raw uint16 bit patterns).
* engine_metadata.json — attention contexts produced by the reference's own
  Scheduler + BlockManager (prefix cache, chunked prefill) and
  ModelRunner.prepare_prefill / prepare_decode (model_runner.py:129-188),
  with the sequence states that produced them. torch's pin_memory/.cuda()
  are neutralised for the CPU; nothing else of the reference is changed.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def make_store_fixture(seed: int = 1234) -> None:
    import torch
    import nanovllm.layers.attention as A  # noqa: E402  (reference)

    g = torch.Generator().manual_seed(seed)
    N, H, KVH, d = 40, 4, 2, 128
    nb, bs = 2, 256
    qkv = torch.randn(N, (H + 2 * KVH) * d, generator=g).to(torch.bfloat16)
    q, k, v = qkv.split([H * d, KVH * d, KVH * d], dim=-1)
    k = k.contiguous().view(N, KVH, d)          # k is contiguous after k_norm/RoPE
    v = v.view(N, KVH, d)                       # v stays a strided view of qkv
    assert v.stride(0) == (H + 2 * KVH) * d
    perm = torch.randperm(nb * bs, generator=g)[:N].to(torch.int32)
    perm[5] = -1
    perm[17] = -1
    k_cache = torch.zeros(nb, bs, KVH, d, dtype=torch.bfloat16)
    v_cache = torch.zeros(nb, bs, KVH, d, dtype=torch.bfloat16)
    A.store_kvcache(k, v, k_cache, v_cache, perm)
    np.savez_compressed(
        HERE / "store_kvcache_triton.npz",
        qkv=qkv.view(torch.int16).numpy().view(np.uint16),
        slot_mapping=perm.numpy(),
        k_cache=k_cache.view(torch.int16).numpy().view(np.uint16),
        v_cache=v_cache.view(torch.int16).numpy().view(np.uint16),
        shape=np.array([N, H, KVH, d, nb, bs], dtype=np.int64),
    )


def make_metadata_fixture(seed: int = 7) -> None:
    import random

    import torch
    from transformers import Qwen3Config

    from nanovllm.config import Config
    from nanovllm.engine.model_runner import ModelRunner
    from nanovllm.engine.scheduler import Scheduler
    from nanovllm.engine.sequence import Sequence
    from nanovllm.sampling_params import SamplingParams
    from nanovllm.utils.context import get_context, reset_context

    # CPU stand-ins for the pinned-memory H2D copies in prepare_* (values untouched).
    real_tensor = torch.tensor
    torch.tensor = lambda *a, pin_memory=False, **k: real_tensor(*a, **k)
    torch.Tensor.cuda = lambda self, *a, **k: self

    class Runner:  # only what prepare_* reads: block_size and prepare_block_tables
        block_size = 256
        prepare_block_tables = ModelRunner.prepare_block_tables

    rnd = random.Random(seed)
    with tempfile.TemporaryDirectory() as tmp:
        Qwen3Config(hidden_size=64, num_attention_heads=4, num_key_value_heads=2, head_dim=16,
                    num_hidden_layers=1, intermediate_size=128, vocab_size=1000,
                    max_position_embeddings=8192).save_pretrained(tmp)
        cfg = Config(tmp, max_num_batched_tokens=1024, max_num_seqs=8, max_model_len=4096)
        cfg.num_kvcache_blocks = 24
        cfg.eos = -1
        sched = Scheduler(cfg)
        prefix = [rnd.randrange(1000) for _ in range(600)]
        prompts = [
            prefix,                                                  # A
            prefix[:512] + [rnd.randrange(1000) for _ in range(100)],  # B: 2 shared blocks
            [rnd.randrange(1000) for _ in range(300)],               # C
            [rnd.randrange(1000) for _ in range(1300)],              # D: chunked
        ]
        sp = SamplingParams(temperature=1.0, max_tokens=260, ignore_eos=True)
        seqs = [Sequence(p, sp) for p in prompts]
        steps = []
        # A alone first so its blocks are hashed before B arrives (prefix hit).
        sched.add(seqs[0])
        pending = seqs[1:]
        step = 0
        while not sched.is_finished() and step < 300:
            if step == 1:
                for s in pending:
                    sched.add(s)
            batch, is_prefill = sched.schedule()
            states = [dict(num_tokens=len(s), start=s.num_cached_tokens,
                           num_scheduled=s.num_scheduled_tokens,
                           block_table=list(s.block_table)) for s in batch]
            if is_prefill:
                ModelRunner.prepare_prefill(Runner(), batch)
            else:
                ModelRunner.prepare_decode(Runner(), batch)
            c = get_context()
            rec = dict(is_prefill=is_prefill, seqs=states,
                       slot_mapping=c.slot_mapping.tolist(),
                       block_tables=None if c.block_tables is None else c.block_tables.tolist())
            if is_prefill:
                rec.update(cu_seqlens_q=c.cu_seqlens_q.tolist(),
                           cu_seqlens_k=c.cu_seqlens_k.tolist(),
                           max_seqlen_q=c.max_seqlen_q, max_seqlen_k=c.max_seqlen_k)
            else:
                rec.update(context_lens=c.context_lens.tolist())
            # keep the fixture small: every prefill, and decode steps around block edges
            if is_prefill or step % 37 == 0 or any(st["num_tokens"] % 256 in (0, 1, 255)
                                                    for st in states):
                steps.append(rec)
            reset_context()
            sched.postprocess(batch, [rnd.randrange(1000) for _ in batch], is_prefill)
            step += 1
    (HERE / "engine_metadata.json").write_text(json.dumps(dict(block_size=256, steps=steps)))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the Nano-vLLM-X source tree")
    args = ap.parse_args()
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(Path(args.reference).resolve()))
    make_store_fixture()
    make_metadata_fixture()
    print("wrote", sorted(p.name for p in HERE.iterdir() if p.suffix in (".npz", ".json")))


if __name__ == "__main__":
    main()
