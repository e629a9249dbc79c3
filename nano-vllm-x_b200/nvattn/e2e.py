"""End-to-end generation through the reference engine with nvattn attention.

the reference's own engine (Nano-vLLM-X: LLM ->
LLMEngine -> Scheduler/BlockManager -> ModelRunner with CUDA-graph decode)
generates for bench.py's workload (random.seed(0); 256 requests of random
token ids, input and output lengths uniform in [100, 1024], ignore_eos;
bench.py:8-24) with a random-init Qwen3-0.6B: 28 layers, hidden 1024,
16 Q / 8 KV heads, head_dim 128, vocab 151936, RMSNorm, RoPE theta 1e6,
bf16. Greedy decoding.

The engine is used unchanged except for what this environment lacks:

* weights: seeded random bf16 tensors written as safetensors next to a
  written config.json (no checkpoint is available offline);
* tokenizer: the workload is token ids only, so AutoTokenizer is replaced
  by a stub (no tokenizer files are available);
* sampler: the reference forbids temperature 0 (sampling_params.py:11) and
  samples stochastically (sampler.py:11); greedy decoding takes the argmax
  of the same logits;
* attention: ``--attn nvattn`` swaps nanovllm.layers.attention.Attention for
  nvattn.Attention in every engine process (tensor-parallel workers are
  spawned, so the swap runs in ModelRunner's constructor); ``--attn
  nvattn-fused`` also fuses Qwen3's q/k RMSNorm, rotary and KV scatter into
  one kernel (``nvattn.install(fuse_qk_norm_rope=True)``) and takes the greedy
  token with nvattn's sampler kernel (``nvattn.ops.sample``); at TP > 1 the
  LM head no longer gathers its logits to rank 0 (embed_head.py:62-65):
  every rank picks within its own vocabulary shard and the ranks exchange
  one 64-bit key per row (``nvattn.parallel.sample_vocab_parallel``); and
  each decode step's metadata comes from one packed host record and one
  kernel writing the CUDA graph's inputs in place
  (``nvattn.DecodeMetadata``, replacing prepare_decode and run_model's
  copies, model_runner.py:172-188, 204-210); and at TP > 1 the row-parallel
  linears' all-reduce (linear.py:152-155) runs through nvattn's peer-memory
  kernel (``nvattn.allreduce``) for the messages it pushes word by word
  (decode steps), NCCL keeping the larger ones (``--nccl-allreduce`` keeps
  NCCL for all; ``--oneshot-allreduce`` is the default, kept as a flag);
  ``--attn reference`` keeps the engine's own flash-attn / Triton path.

    python -m nvattn.e2e --tp 1 --attn nvattn [--num-seqs 256] [--out ids.npz] [--record]
    python -m nvattn.e2e --compare reference.npz nvattn.npz

Prints one JSON line: output tokens, seconds, tok/s. With ``--record`` rank 0
also keeps, for every generated token, the top-2 logits (values and ids) of
the row it was picked from; ``--out`` saves them beside the token ids.
``--compare`` reads two such files (the first is the reference arm) and gives,
per request, whether the ids are identical, the first divergent step, and the
reference's top-1 minus top-2 logit margin at that step in bf16 ulps of its
top logit. Needs the reference package importable (e.g. ``pip install
--no-deps --target baseline/_ref``).
"""
from __future__ import annotations

import argparse
import json
import os
import random
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

QWEN3_0_6B = dict(hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                  num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                  vocab_size=151936, max_position_embeddings=40960, rms_norm_eps=1e-6,
                  rope_theta=1000000.0, tie_word_embeddings=True, hidden_act="silu",
                  attention_bias=False, dtype="bfloat16")


def write_model(path: Path, seed: int = 0, **overrides) -> None:
    """config.json + seeded random weights (HF parameter names) as safetensors."""
    from safetensors.torch import save_file
    from transformers import Qwen3Config

    cfg = dict(QWEN3_0_6B, **overrides)
    Qwen3Config(**cfg).save_pretrained(path)
    g = torch.Generator().manual_seed(seed)
    h, inter, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    nh, nkv, d, V = (cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"],
                     cfg["vocab_size"])

    def w(*shape, std=0.02):
        return (torch.randn(*shape, generator=g) * std).to(torch.bfloat16)

    def norm(n):
        return (1.0 + 0.1 * torch.randn(n, generator=g)).to(torch.bfloat16)

    tensors = {"model.embed_tokens.weight": w(V, h), "model.norm.weight": norm(h)}
    for i in range(L):
        p = f"model.layers.{i}."
        tensors.update({
            p + "input_layernorm.weight": norm(h),
            p + "post_attention_layernorm.weight": norm(h),
            p + "self_attn.q_proj.weight": w(nh * d, h),
            p + "self_attn.k_proj.weight": w(nkv * d, h),
            p + "self_attn.v_proj.weight": w(nkv * d, h),
            p + "self_attn.o_proj.weight": w(h, nh * d),
            p + "self_attn.q_norm.weight": norm(d),
            p + "self_attn.k_norm.weight": norm(d),
            p + "mlp.gate_proj.weight": w(inter, h),
            p + "mlp.up_proj.weight": w(inter, h),
            p + "mlp.down_proj.weight": w(h, inter),
        })
    save_file(tensors, str(path / "model.safetensors"))


class _TokenizerStub:
    """Token-id workloads need no tokenizer; decode() is only used for text."""

    eos_token_id = -1

    @classmethod
    def from_pretrained(cls, *args, **kwargs):
        return cls()

    def encode(self, text):
        raise ValueError("the e2e harness takes token-id prompts only")

    def decode(self, token_ids):
        return ""


def _greedy_forward(self, logits, temperatures):
    return logits.float().argmax(dim=-1)


def _nvattn_greedy_forward(self, logits, temperatures):
    from nvattn import ops
    return ops.sample(logits)  # T <= 0 path: greedy argmax, first index on ties


def _lm_head_local_forward(self, x):
    """ParallelLMHead.forward (embed_head.py:53-66) without the gather: each
    rank returns the logits of its own vocabulary shard."""
    import torch.nn.functional as F
    from nanovllm.utils.context import get_context
    context = get_context()
    if context.is_prefill:
        x = x[context.cu_seqlens_q[1:] - 1].contiguous()
    return F.linear(x, self.weight)


_ONESHOT = None
_ONESHOT_CAPACITY = 512 * 4096  # decode graphs up to 512 tokens x hidden 4096


def _row_parallel_oneshot_forward(self, x):
    """RowParallelLinear.forward (linear.py:152-155) at TP > 1 through
    nvattn's peer-memory all-reduce for the messages it pushes word by word
    (decode steps); larger ones keep the reference's F.linear +
    dist.all_reduce."""
    global _ONESHOT
    if self.tp_size == 1:
        return self._reference_forward(x)
    if _ONESHOT is None:  # first call: warm-up, all ranks together, outside capture
        from nvattn.allreduce import OneShotAllReduce
        _ONESHOT = OneShotAllReduce(_ONESHOT_CAPACITY)
    from nvattn.allreduce import row_parallel_forward
    y = row_parallel_forward(_ONESHOT, x, self.weight, self.bias, self.tp_rank, pushed_only=True)
    return y if y is not None else self._reference_forward(x)


def patch_engine(attn: str) -> None:
    """Apply the substitutions listed in the module docstring (idempotent)."""
    import nanovllm.engine.llm_engine as llm_engine
    import nanovllm.engine.model_runner as model_runner
    import nanovllm.layers.sampler as sampler

    sampler.Sampler.forward = _nvattn_greedy_forward if attn == "nvattn-fused" else _greedy_forward
    model_runner.Sampler = sampler.Sampler
    llm_engine.AutoTokenizer = _TokenizerStub
    llm_engine.ModelRunner = E2EModelRunner
    if attn in ("nvattn", "nvattn-fused"):
        import nvattn
        nvattn.install(fuse_qk_norm_rope=(attn == "nvattn-fused"))
    if attn == "nvattn-fused":
        import nanovllm.layers.embed_head as embed_head
        import nanovllm.layers.linear as linear
        embed_head.ParallelLMHead.forward = _lm_head_local_forward
        if os.environ.get("NVATTN_E2E_ONESHOT_AR") == "1":
            if not hasattr(linear.RowParallelLinear, "_reference_forward"):
                linear.RowParallelLinear._reference_forward = linear.RowParallelLinear.forward
            linear.RowParallelLinear.forward = _row_parallel_oneshot_forward


class _RecordingSampler:
    """Wraps rank 0's sampler: before sampling, keeps the top-2 logits of
    every row that yields a token this step (a partial prefill chunk yields
    none, scheduler.py postprocess), keyed by sequence id."""

    def __init__(self, inner, runner):
        self.inner = inner
        self.runner = runner

    def __call__(self, logits, temperatures):
        top = logits.float().topk(2, dim=-1)
        vals = top.values.cpu().numpy()
        ids = top.indices.cpu().numpy()
        for row, (seq_id, keep) in enumerate(self.runner._step_rows):
            if keep:
                self.runner._record.setdefault(seq_id, []).append(
                    (vals[row, 0], vals[row, 1], ids[row, 0], ids[row, 1]))
        return self.inner(logits, temperatures)


def _runner_base():
    import nanovllm.engine.model_runner as model_runner
    return model_runner.ModelRunner


def _make_runner_class():
    base = _runner_base()

    class Runner(base):
        """ModelRunner that re-applies the substitutions in its own process
        (tensor-parallel workers are started with the spawn method)."""

        def __init__(self, config, rank, event):
            self._attn = os.environ.get("NVATTN_E2E_ATTN", "nvattn")
            self._sample_step = 0
            # top-2 logits per generated token, on rank 0 where the whole row
            # is sampled (not in the fused arm at TP > 1: shards only)
            self._recording = (os.environ.get("NVATTN_E2E_RECORD") == "1" and rank == 0 and
                               not (self._attn == "nvattn-fused" and
                                    config.tensor_parallel_size > 1))
            self._record: dict[int, list] = {}
            self._step_rows: list = []
            patch_engine(self._attn)
            super().__init__(config, rank, event)  # workers (rank > 0) loop in here
            if self._recording:
                self.sampler = _RecordingSampler(self.sampler, self)

        def prepare_decode(self, seqs):
            """ModelRunner.prepare_decode (model_runner.py:172-188). In the
            fused arm: one packed record, one copy, one kernel; on the graph
            path the kernel writes the graph's static inputs directly, so
            run_model only replays."""
            if self._attn != "nvattn-fused":
                return super().prepare_decode(seqs)
            from nanovllm.utils.context import set_context
            from nvattn.decode_meta import DecodeMetadata
            dev = torch.device("cuda", torch.cuda.current_device())
            if getattr(self, "_decode_meta", None) is None:
                max_w = (self.config.max_model_len + self.block_size - 1) // self.block_size
                self._decode_meta = DecodeMetadata(max(self.config.max_num_seqs, 512), max_w,
                                                   self.block_size, dev)
            meta = self._decode_meta
            B, W = meta.pack(seqs)
            gv = getattr(self, "graph_vars", None)
            if self.enforce_eager or B > 512 or gv is None:
                ids = torch.empty(B, dtype=torch.int64, device=dev)
                pos = torch.empty(B, dtype=torch.int64, device=dev)
                slots = torch.empty(B, dtype=torch.int32, device=dev)
                lens = torch.empty(B, dtype=torch.int32, device=dev)
                tables = torch.empty(B, W, dtype=torch.int32, device=dev)
                meta.launch(B, input_ids=ids, positions=pos, slot_mapping=slots,
                            context_lens=lens, block_tables=tables)
                set_context(False, slot_mapping=slots, context_lens=lens, block_tables=tables)
                return ids, pos
            meta.launch(gv["slot_mapping"].numel(), input_ids=gv["input_ids"],
                        positions=gv["positions"], slot_mapping=gv["slot_mapping"],
                        context_lens=gv["context_lens"], block_tables=gv["block_tables"])
            self._graph_inputs_ready = True
            set_context(False, slot_mapping=gv["slot_mapping"][:B],
                        context_lens=gv["context_lens"][:B],
                        block_tables=gv["block_tables"][:B, :W])
            return gv["input_ids"][:B], gv["positions"][:B]

        def exit(self):
            """ModelRunner.exit (model_runner.py:40-49); with the one-shot
            all-reduce, first gathers every rank's nvattn status word to rank 0
            (all ranks run exit together, so the collective is matched)."""
            if os.environ.get("NVATTN_E2E_ONESHOT_AR") == "1" and self.world_size > 1:
                import torch.distributed as dist
                from nvattn import ops
                dev = torch.device("cuda", torch.cuda.current_device())
                st = ops.status_tensor(dev).view(1)
                every = torch.zeros(self.world_size, dtype=torch.int32, device=dev)
                dist.all_gather_into_tensor(every, st)
                bits = 0
                for v in every.tolist():
                    bits |= int(v)
                self._final_status = bits
            return super().exit()

        @torch.inference_mode()
        def run_model(self, input_ids, positions, is_prefill):
            """ModelRunner.run_model (model_runner.py:196-212); the graph's
            inputs are already in place when prepare_decode wrote them."""
            if is_prefill or not getattr(self, "_graph_inputs_ready", False):
                return super().run_model(input_ids, positions, is_prefill)
            self._graph_inputs_ready = False
            bs = input_ids.size(0)
            self.graphs[next(x for x in self.graph_bs if x >= bs)].replay()
            return self.model.compute_logits(self.graph_vars["outputs"][:bs])

        def run(self, seqs, is_prefill):
            """ModelRunner.run (model_runner.py:214-220); in the fused arm at
            TP > 1 every rank samples its vocabulary shard and rank 0
            returns the merged tokens."""
            if self._recording:
                self._step_rows = [
                    (seq.seq_id, not is_prefill or
                     seq.num_cached_tokens + seq.num_scheduled_tokens == seq.num_tokens)
                    for seq in seqs]
            if self._attn != "nvattn-fused" or self.world_size == 1:
                return super().run(seqs, is_prefill)
            from nanovllm.utils.context import reset_context
            from nvattn.parallel import sample_vocab_parallel
            input_ids, positions = (self.prepare_prefill(seqs) if is_prefill
                                    else self.prepare_decode(seqs))
            logits = self.run_model(input_ids, positions, is_prefill)
            tokens = sample_vocab_parallel(logits, None,  # greedy, as the harness decodes
                                           vocab_offset=self.model.lm_head.vocab_start_idx,
                                           seed=0, offset=self._sample_step)
            self._sample_step += 1
            token_ids = tokens.tolist() if self.rank == 0 else None
            reset_context()
            return token_ids

    Runner.__module__ = __name__
    Runner.__qualname__ = "E2EModelRunner"
    return Runner


def __getattr__(name):  # module-level lazy class (needs the reference importable)
    if name == "E2EModelRunner":
        cls = _make_runner_class()
        globals()["E2EModelRunner"] = cls
        return cls
    raise AttributeError(name)


def bench_workload(num_seqs: int = 256, max_input_len: int = 1024, max_output_len: int = 1024):
    """bench.py's draw order under random.seed(0) (bench.py:8-14)."""
    random.seed(0)
    prompts = [[random.randint(0, 10000) for _ in range(random.randint(100, max_input_len))]
               for _ in range(num_seqs)]
    max_tokens = [random.randint(100, max_output_len) for _ in range(num_seqs)]
    return prompts, max_tokens


def peer_memory_allreduce(attn: str, tp: int, requested: bool | None) -> bool:
    """Whether a run routes its decode-sized row-parallel all-reduces through
    nvattn's peer-memory kernel: only the fused arm at TP > 1 can, and it does
    unless the caller asked for NCCL (requested False); None is the default."""
    if attn != "nvattn-fused" or tp <= 1:
        return False
    return True if requested is None else bool(requested)


def run(tp: int, attn: str, num_seqs: int, max_input_len: int, max_output_len: int,
        enforce_eager: bool, model_dir: str | None = None, out: str | None = None,
        oneshot_allreduce: bool | None = None, record: bool = False,
        max_num_seqs: int | None = None) -> dict:
    oneshot_allreduce = peer_memory_allreduce(attn, tp, oneshot_allreduce)
    os.environ["NVATTN_E2E_ATTN"] = attn
    os.environ["NVATTN_E2E_ONESHOT_AR"] = "1" if oneshot_allreduce else "0"
    os.environ["NVATTN_E2E_RECORD"] = "1" if record else "0"
    import nanovllm.engine.llm_engine as llm_engine  # noqa: F401  (reference)
    global E2EModelRunner
    E2EModelRunner = _make_runner_class()
    patch_engine(attn)
    from nanovllm import LLM, SamplingParams

    tmp = None
    if model_dir is None:
        tmp = tempfile.TemporaryDirectory()
        model_dir = tmp.name
        write_model(Path(model_dir))
    prompts, max_tokens = bench_workload(num_seqs, max_input_len, max_output_len)
    extra = {} if max_num_seqs is None else {"max_num_seqs": max_num_seqs}
    llm = LLM(model_dir, enforce_eager=enforce_eager, max_model_len=4096, tensor_parallel_size=tp,
              **extra)
    sps = [SamplingParams(temperature=1.0, ignore_eos=True, max_tokens=m) for m in max_tokens]
    llm.generate([[1, 2, 3]], SamplingParams(max_tokens=4), use_tqdm=False)  # warm-up
    torch.cuda.synchronize()
    runner = llm.model_runner
    if getattr(runner, "_recording", False):
        runner._record = {}
    t = time.time()
    outs = llm.generate(prompts, sps, use_tqdm=False)
    dt = time.time() - t
    total = sum(max_tokens)
    res = {"metric": "e2e out tok/s", "attn": attn, "tp": tp, "num_seqs": num_seqs,
           "output_tokens": total, "seconds": round(dt, 3), "value": round(total / dt, 1),
           "unit": "tok/s", "enforce_eager": enforce_eager,
           "model": "random-init Qwen3-0.6B (28 layers, 16Q/8KV, d128, vocab 151936, bf16)",
           "decoding": "greedy", "oneshot_allreduce": oneshot_allreduce}
    if max_num_seqs is not None:
        res["max_num_seqs"] = max_num_seqs
    arrays = {f"r{i}": np.array(o["token_ids"], np.int32) for i, o in enumerate(outs)}
    if getattr(runner, "_recording", False):
        # requests were added in order, so the i-th smallest sequence id is request i
        for i, seq_id in enumerate(sorted(runner._record)):
            arrays[f"m{i}"] = np.array(runner._record[seq_id], np.float32).reshape(-1, 4)
        res["recorded"] = True
    if out:
        np.savez_compressed(out, **arrays)
    # Stop the engine's workers now (its atexit hook would do the same later).
    import atexit
    atexit.unregister(llm.exit)
    llm.exit()
    if oneshot_allreduce and tp > 1:
        # A flag wait of the peer-memory all-reduce that gave up (NVATTN_STATUS_TIMEOUT)
        # means that launch summed partials a peer may not have finished writing: its
        # tokens are not valid, and neither is the measurement. Every rank's status word
        # was gathered to rank 0 when the engine exited.
        st = getattr(runner, "_final_status", None)
        res["status"] = st
        if st:
            raise RuntimeError(f"nvattn status word {st:#x} on some rank after generate "
                               "(one-shot all-reduce wait timed out, or a bad slot or block): "
                               "the run is invalid")
    if tmp is not None:
        tmp.cleanup()
    return res


def _bf16_ulp(x: np.ndarray) -> np.ndarray:
    """Spacing of bf16 numbers (8 significant bits) at |x|."""
    ax = np.maximum(np.abs(x.astype(np.float64)), 2.0 ** -126)
    return np.exp2(np.floor(np.log2(ax)) - 7)


def compare(ref_path: str, ours_path: str, k_ulps: float = 4.0) -> dict:
    """Per-request comparison of two ``--out`` files; the first is the
    reference arm and must carry ``--record``'s top-2 logits.

    For a request whose ids differ, the first divergent step s is the first
    index where the two id lists differ. Up to s both arms saw the same
    tokens, so at s they sampled from the same context; the reference's
    margin there, (top1 - top2) / ulp(top1), says how close its own choice was
    to a tie. Returns a summary with every request's record."""
    a, b = np.load(ref_path), np.load(ours_path)
    n = len([key for key in a.files if key.startswith("r")])
    rows, all_margins = [], []
    for i in range(n):
        ra, rb = a[f"r{i}"], b[f"r{i}"]
        m = a[f"m{i}"] if f"m{i}" in a.files else None
        if m is not None:
            all_margins.append((m[:, 0] - m[:, 1]) / _bf16_ulp(m[:, 0]))
        same = ra.shape == rb.shape and np.array_equal(ra, rb)
        row = {"request": i, "tokens": int(len(ra)), "identical": bool(same)}
        if not same:
            length = min(len(ra), len(rb))
            diff = np.nonzero(ra[:length] != rb[:length])[0]
            s = int(diff[0]) if len(diff) else length
            row["first_divergence"] = s
            if m is not None and s < len(m):
                row["ref_margin_ulps"] = float((m[s, 0] - m[s, 1]) / _bf16_ulp(m[s, 0]))
                row["ref_top2_ids"] = [int(m[s, 2]), int(m[s, 3])]
                row["ours_token"] = int(rb[s]) if s < len(rb) else None
            mb = b[f"m{i}"] if f"m{i}" in b.files else None
            if mb is not None and s < len(mb):
                row["ours_margin_ulps"] = float((mb[s, 0] - mb[s, 1]) / _bf16_ulp(mb[s, 0]))
        rows.append(row)
    div = [r for r in rows if not r["identical"]]
    margins = np.array([r["ref_margin_ulps"] for r in div if "ref_margin_ulps" in r])
    allm = np.concatenate(all_margins) if all_margins else np.zeros(0)
    summary = {"requests": n, "identical": n - len(div), "diverged": len(div),
               "k_ulps": k_ulps,
               "diverged_within_k": int((margins <= k_ulps).sum()),
               "max_ref_margin_at_divergence_ulps": float(margins.max()) if len(margins) else None,
               "median_first_divergence_frac": float(np.median(
                   [r["first_divergence"] / max(1, r["tokens"]) for r in div])) if div else None,
               "all_steps_margin_median_ulps": float(np.median(allm)) if len(allm) else None,
               "all_steps_frac_within_k": float((allm <= k_ulps).mean()) if len(allm) else None,
               "margin_histogram_at_divergence": {
                   str(lo): int(((margins >= lo) & (margins < hi)).sum())
                   for lo, hi in ((0, 1), (1, 2), (2, 4), (4, 8), (8, 16), (16, 1e9))},
               "rows": rows}
    return summary


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__,
                                 formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--attn", choices=("nvattn", "nvattn-fused", "reference"), default="nvattn")
    ap.add_argument("--num-seqs", type=int, default=256)
    ap.add_argument("--max-input-len", type=int, default=1024)
    ap.add_argument("--max-output-len", type=int, default=1024)
    ap.add_argument("--enforce-eager", action="store_true")
    ap.add_argument("--model-dir", default=None, help="reuse a written model directory")
    ap.add_argument("--write-model", default=None, help="only write the model to this dir")
    ap.add_argument("--out", default=None, help="save generated token ids (npz)")
    ar = ap.add_mutually_exclusive_group()
    ar.add_argument("--oneshot-allreduce", dest="oneshot", action="store_true", default=None,
                    help="fused arm at TP > 1: row-parallel all-reduce of decode-sized "
                         "messages through nvattn's peer-memory kernel (the default)")
    ar.add_argument("--nccl-allreduce", dest="oneshot", action="store_false",
                    help="fused arm at TP > 1: keep NCCL for every row-parallel all-reduce")
    ap.add_argument("--record", action="store_true",
                    help="keep the top-2 logits of every generated token (saved by --out)")
    ap.add_argument("--max-num-seqs", type=int, default=None,
                    help="engine's max_num_seqs (reference default 512)")
    ap.add_argument("--compare", nargs=2, metavar=("REF_NPZ", "OURS_NPZ"),
                    help="compare two --out files (the first from the reference arm)")
    ap.add_argument("--k-ulps", type=float, default=4.0)
    args = ap.parse_args()
    if args.compare:
        summary = compare(*args.compare, k_ulps=args.k_ulps)
        rows = summary.pop("rows")
        print(json.dumps(summary))
        for r in rows:
            if not r["identical"]:
                print(json.dumps(r))
        return
    if args.write_model:
        Path(args.write_model).mkdir(parents=True, exist_ok=True)
        write_model(Path(args.write_model))
        return
    res = run(args.tp, args.attn, args.num_seqs, args.max_input_len, args.max_output_len,
              args.enforce_eager, args.model_dir, args.out, args.oneshot, args.record,
              args.max_num_seqs)
    print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
