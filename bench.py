"""Benchmark of the B200 paged-KV attention path (nvattn).

Headline (the first part of BASELINE.json's metric, "paged decode-attn HBM
GB/s"): configs[3], long-context paged decode at the Qwen3-32B attention shape
(64 Q / 8 KV heads, head_dim 128, bf16 cache, 256-token blocks, 128 sequences,
context lengths uniform in [4096, 32768], physical blocks randomly permuted).
One step = one decode-mode ``Attention.forward`` (nanovllm/layers/attention.py
:59-75): KV scatter of the new token + split-K paged decode (+ combine).
Heads are sharded across ranks like the engine's tensor parallelism
(qwen3.py:29-35): with N GPUs each rank owns 8/N KV heads and 64/N Q heads of
the same batch (strong scaling: the total work is fixed).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl nvattn|reference]

Rank 0 prints one JSON line. ``value`` is the whole-job algorithmic HBM
throughput (bytes all ranks must move / max-over-ranks device time) with
inputs resident in HBM; ``e2e`` is the same metric through the public API
with the step's inputs copied from pinned host memory and the output copied
back inside the timed region. Secondary lines in the same JSON: prefill
TFLOP/s at configs[2] (prefix-cached prefill, Qwen3-8B shape) and tree
verification at configs[4].

``--impl reference`` times the reference's attention math as a CPU
restatement (the oracle; the reference's own attention is flash-attn CUDA
code with no CPU path) on all host cores, on a bounded sample of the same
workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "nano-vllm-x_b200"))

H_TOTAL, KVH_TOTAL, D, BS = 64, 8, 128, 256
BATCH, CTX_LO, CTX_HI = 128, 4096, 32768
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
METRIC = "paged decode-attn HBM GB/s"
WORKLOAD = ("configs[3] long-context paged decode, Qwen3-32B attention: 64Q/8KV heads, d128, "
            "bf16 KV cache, 256-token blocks, 128 seqs, ctx U[4096,32768], permuted blocks; "
            "step = Attention.forward decode (KV scatter + split-K decode + combine)")


# ----------------------------------------------------------------- workload

def decode_workload(seed: int = 0, batch: int = BATCH):
    rng = np.random.default_rng(seed)
    lens = rng.integers(CTX_LO, CTX_HI + 1, size=batch).astype(np.int32)
    nblk = (lens + BS - 1) // BS
    total = int(nblk.sum())
    perm = rng.permutation(total).astype(np.int32)
    width = int(nblk.max())
    bt = np.full((batch, width), -1, np.int32)
    pos = 0
    for b in range(batch):
        bt[b, :nblk[b]] = perm[pos:pos + nblk[b]]
        pos += nblk[b]
    return lens, bt, total


def decode_bytes(lens, kvh, h):
    """Algorithmic HBM bytes of one decode step on one rank."""
    kv_read = int(lens.astype(np.int64).sum()) * kvh * D * 2 * 2
    qo = 2 * len(lens) * h * D * 2
    scatter = 2 * len(lens) * kvh * D * 2 * 2  # read new k/v + write to the cache
    meta = len(lens) * 4 * 2 + int(((lens + BS - 1) // BS).sum()) * 4
    return kv_read + qo + scatter + meta


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        j = json.loads(p.read_text())
        return float(j["hbm_gbs"]), float(j["bf16_tflops"]), float(
            j.get("bf16_tflops_sustained", j["bf16_tflops"])), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


# ------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi sampling of SM clock + throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines: list[str] = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.index), "-lms", "100"], stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread:
            self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "samples": len(sm),
                "reasons": sorted(reasons)}


# -------------------------------------------------------------- distributed

def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
        _gloo_group()  # collective: every rank creates it here, in the same order
    else:
        torch.cuda.set_device(0)
    return rank, world, local


_GLOO = None


def _gloo_group():
    """A CPU process group with a long timeout, for ranks that wait while rank 0
    runs the end-to-end engine (minutes)."""
    global _GLOO
    if _GLOO is None:
        import datetime

        import torch.distributed as dist
        _GLOO = dist.new_group(backend="gloo", timeout=datetime.timedelta(seconds=3600))
    return _GLOO


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(x: float, world: int, device: str = "cuda") -> float:
    """Job time = the slowest rank's time (every rank calls this, same order)."""
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x: float, world: int, device: str = "cuda") -> float:
    """Whole-job work = the sum of every rank's work."""
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def reference_on_path() -> None:
    """Make the reference package (installed into baseline/_ref) importable."""
    ref_dir = REPO / "baseline" / "_ref"
    if ref_dir.is_dir() and str(ref_dir) not in sys.path:
        sys.path.append(str(ref_dir))


# ------------------------------------------------------------- nvattn arm

def timed(fn, steps, stream):
    """Device time (ms) of `steps` calls of fn on `stream`, CUDA events."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    return start.elapsed_time(end)


def graph_timed(fn, steps, dev, per_graph=10):
    """Device time (ms) of one call of fn: `per_graph` calls captured in one
    CUDA graph, the graph replayed `steps` times between CUDA events (no
    host launch gaps between the calls, which a short kernel would show)."""
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(s):
        fn()
    torch.cuda.current_stream(dev).wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for _ in range(per_graph):
            fn()
    graph.replay()
    stream = torch.cuda.current_stream(dev)
    ms = timed(graph.replay, steps, stream) / (steps * per_graph)
    del graph
    return ms


def run_nvattn(args):
    import nvattn
    from nvattn import context as ctxmod
    from nvattn import ops
    from nvattn.parallel import head_shard

    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    (q0, q1), (k0, k1) = head_shard(H_TOTAL, KVH_TOTAL, rank, world)
    H, KVH = q1 - q0, k1 - k0
    hbm_peak, tf_peak, tf_sus, peak_src = load_peaks()

    BATCH = args.batch  # noqa: N806  (configs[3] uses 128; smaller only for profiling)
    lens, bt_np, nblocks = decode_workload(0, BATCH)
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    kv = torch.empty(2, nblocks, BS, KVH, D, dtype=torch.bfloat16, device=dev)
    kv.normal_(generator=g)
    k_cache, v_cache = kv[0], kv[1]
    attn = nvattn.Attention(H, D, D ** -0.5, KVH)
    attn.k_cache, attn.v_cache = k_cache, v_cache

    # decode inputs: the new token of every sequence sits at position len-1
    ctx_lens = lens.copy()
    slots = np.array([bt_np[b, (n - 1) // BS] * BS + (n - 1) % BS for b, n in enumerate(lens)],
                     np.int32)
    q = torch.randn(BATCH, H, D, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(BATCH, KVH, D, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(BATCH, KVH, D, generator=g, device=dev).to(torch.bfloat16)
    slot_d = torch.from_numpy(slots).to(dev)
    lens_d = torch.from_numpy(ctx_lens).to(dev)
    bt_d = torch.from_numpy(bt_np).to(dev)
    ws = torch.empty(max(1, ops.decode_workspace_bytes(BATCH, H, KVH, bt_np.shape[1], BS)),
                     dtype=torch.uint8, device=dev)
    ops.status_tensor(dev)
    stream = torch.cuda.current_stream(dev)

    def step():
        ctxmod.set_context(False, slot_mapping=slot_d, context_lens=lens_d, block_tables=bt_d)
        attn(q, k, v)

    def decode_only():
        ops.paged_decode(q, k_cache, v_cache, lens_d, bt_d, softmax_scale=D ** -0.5,
                         workspace=ws)

    nsplit_launches = 2 if ops.decode_workspace_bytes(BATCH, H, KVH, bt_np.shape[1], BS) else 1
    bytes_rank = decode_bytes(lens, KVH, H)
    bytes_decode = bytes_rank - 2 * BATCH * KVH * D * 2 * 2  # without the scatter

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)

    sampler = ClockSampler(local)
    sampler.start()
    time.sleep(0.5)  # let nvidia-smi start sampling before the timed region
    barrier(world)
    ms = timed(step, args.steps, stream)
    barrier(world)
    ms_dec = timed(decode_only, args.steps, stream)
    clocks = sampler.stop()
    st = ops.read_status(dev)
    if st:
        raise SystemExit(f"kernel status word {st} (bad slot/block or timeout)")

    # ---- e2e through the public API with host buffers
    pin = lambda a: torch.from_numpy(a).pin_memory()  # noqa: E731
    q_h = q.cpu().pin_memory()
    k_h = k.cpu().pin_memory()
    v_h = v.cpu().pin_memory()
    slot_h, lens_h, bt_h = pin(slots), pin(ctx_lens), pin(bt_np)
    out_h = torch.empty(BATCH, 1, H, D, dtype=torch.bfloat16).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (q_h, k_h, v_h, slot_h, lens_h, bt_h))
    d2h = out_h.numel() * out_h.element_size()

    def e2e_step():
        qd = q_h.to(dev, non_blocking=True)
        kd = k_h.to(dev, non_blocking=True)
        vd = v_h.to(dev, non_blocking=True)
        ctxmod.set_context(False, slot_mapping=slot_h.to(dev, non_blocking=True),
                           context_lens=lens_h.to(dev, non_blocking=True),
                           block_tables=bt_h.to(dev, non_blocking=True))
        o = attn(qd, kd, vd)
        out_h.copy_(o, non_blocking=True)

    for _ in range(max(1, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    barrier(world)
    ms_e2e = timed(e2e_step, args.steps, stream)
    ctxmod.reset_context()

    t_step = max_over_ranks(ms / args.steps, world)
    t_dec = max_over_ranks(ms_dec / args.steps, world)
    t_e2e = max_over_ranks(ms_e2e / args.steps, world)
    total_bytes = sum_over_ranks(bytes_rank, world)
    value = total_bytes / (t_step * 1e-3) / 1e9
    e2e_value = total_bytes / (t_e2e * 1e-3) / 1e9
    achieved = bytes_decode / (t_dec * 1e-3) / 1e9

    secondary = {}
    if not args.skip_secondary:
        del kv, k_cache, v_cache
        attn.k_cache = attn.v_cache = torch.tensor([])
        torch.cuda.empty_cache()
        secondary["prefill_cfg3"] = bench_prefill(dev, rank, world, args, tf_peak)
        secondary["tree_verify_cfg5"] = bench_tree(dev, rank, world, args, tf_peak, hbm_peak)
        secondary["qk_norm_rope_store"] = bench_qknorm(dev, rank, world, args, hbm_peak)
        if world == 1:
            secondary["store_kvcache"] = bench_store_kvcache(dev, args, hbm_peak)
            secondary["sampler"] = bench_sampler(dev, args, hbm_peak)
            try:
                secondary["layer_cfg0"] = bench_layer_cfg0(dev, args)
            except Exception as e:  # noqa: BLE001  (a secondary line never sinks the headline)
                secondary["layer_cfg0"] = {"error": f"{e!r}"[:200]}
            try:
                secondary["decode_prepare"] = bench_decode_prepare(dev, args)
            except Exception as e:  # noqa: BLE001
                secondary["decode_prepare"] = {"error": f"{e!r}"[:200]}
        if rank == 0 and world == 1:
            secondary["flash_attn_decode_cfg4"] = bench_flash_attn_decode(dev, args, H, KVH)
            secondary["decode_e2e_shape"] = bench_decode_e2e_shape(dev, args, hbm_peak)

    traffic = None
    prof = REPO / "profiles" / "paged_decode_cfg4.json"
    if prof.exists():
        try:
            traffic = json.loads(prof.read_text()).get(f"traffic_bytes_per_launch_tp{world}")
        except (ValueError, OSError):
            traffic = None

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        cpu = cpu_decode_sample(args.cpu_seconds)

    if not args.skip_e2e:
        # every rank frees its memory; rank 0 runs the engine at TP = world over all
        # GPUs while the others wait (a gloo barrier: no NCCL call stays pending)
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        if rank == 0:
            secondary["e2e_cfg1"] = bench_e2e(args, world)
        if world > 1:
            import torch.distributed as dist
            dist.barrier(group=_gloo_group())

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(t_step, 4),
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": None,
            "dtype": "bf16",
            "data": "synthetic (seeded N(0,1) bf16 K/V/Q; numpy seed 0 lengths and block permutation)",
            "config": {"workload": WORKLOAD if BATCH == 128 else WORKLOAD + f" (batch {BATCH})",
                       "global_batch": BATCH, "num_heads": H_TOTAL,
                       "num_kv_heads": KVH_TOTAL, "head_dim": D, "block_size": BS,
                       "ctx_range": [CTX_LO, CTX_HI], "parallelism": f"tp{world} (head-sharded)",
                       "l2": "inputs larger than L2 (KV cache >= 1.2 GB per rank vs 126 MB L2)"},
            "frac_of_nominal_8tbs": round(value / world / NOMINAL_HBM_GBS, 4),
            "roofline": {"kernel": "paged_decode (split-K kernel + combine)", "bound": "hbm",
                         "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "peak_source": peak_src,
                         "traffic": traffic,
                         "algorithmic_bytes_per_launch": bytes_decode,
                         "ms_per_launch": round(t_dec, 4)},
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(t_e2e, 4)},
            "gpu_launches": args.steps * (1 + nsplit_launches),
            "clocks": clocks,
            "cpu_baseline": cpu,
            "secondary": secondary,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def bench_prefill(dev, rank, world, args, tf_peak):
    """64 seqs share a 2048-token prefix (8 cached blocks), suffix U[128,512]."""
    from nvattn import ops
    from nvattn.parallel import head_shard
    (q0, q1), (k0, k1) = head_shard(32, 8, rank, world)
    H, KVH = q1 - q0, k1 - k0
    rng = np.random.default_rng(3)
    B, P = 64, 2048
    suf = rng.integers(128, 513, size=B).astype(np.int64)
    klen = P + suf
    pre_blocks = P // BS
    own = (suf + BS - 1) // BS
    nblocks = pre_blocks + int(own.sum())
    width = pre_blocks + int(own.max())
    bt = np.full((B, width), -1, np.int32)
    pos = pre_blocks
    for b in range(B):
        bt[b, :pre_blocks] = np.arange(pre_blocks)
        bt[b, pre_blocks:pre_blocks + own[b]] = np.arange(pos, pos + own[b])
        pos += own[b]
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    kc = torch.randn(nblocks, BS, KVH, D, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(nblocks, BS, KVH, D, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(int(suf.sum()), H, D, generator=g, device=dev).to(torch.bfloat16)
    cq = torch.tensor(np.concatenate([[0], np.cumsum(suf)]), dtype=torch.int32, device=dev)
    ck = torch.tensor(np.concatenate([[0], np.cumsum(klen)]), dtype=torch.int32, device=dev)
    btd = torch.from_numpy(bt).to(dev)
    out = torch.empty_like(q)
    flops = float(sum(4 * D * H * (P + i + 1) for s in suf for i in range(int(s))))

    def fn():
        ops.varlen_prefill(q, kc, vc, cq, ck, int(suf.max()), int(klen.max()),
                           softmax_scale=D ** -0.5, causal=True, block_table=btd, out=out)

    for _ in range(args.warmup):
        fn()
    barrier(world)
    # eager launches: GPU-bound at every N (a call is >= 0.1 ms per rank); under
    # graph replay the back-to-back calls reach the power cap sooner
    ms = max_over_ranks(timed(fn, args.steps, torch.cuda.current_stream(dev)) / args.steps,
                        world)
    total = sum_over_ranks(flops, world)
    tfs = total / (ms * 1e-3) / 1e12
    res = {"metric": "prefill attn TFLOP/s", "value": round(tfs, 1), "unit": "TFLOP/s",
           "ms_per_step": round(ms, 4),
           "frac_of_measured_bf16_peak_per_gpu": round(tfs / world / tf_peak, 4),
           "frac_of_measured_bf16_sustained_peak_per_gpu": round(tfs / world / load_peaks()[2], 4),
           "flops_per_step": total,
           "timing": "CUDA events around back-to-back eager calls, max over ranks",
           "workload": "configs[2]: 64 seqs, 2048-token shared prefix (8 blocks), suffix "
                       "U[128,512], 32Q/8KV, d128, causal over prefix+suffix"}
    if world == 1:
        # the reference's own GPU prefill on the same cache: flash_attn_varlen_func as
        # attention.py:64-70 calls it on a prefix-cache hit (block_table set)
        try:
            from flash_attn import flash_attn_varlen_func

            def fa():
                flash_attn_varlen_func(q, kc, vc, max_seqlen_q=int(suf.max()), cu_seqlens_q=cq,
                                       max_seqlen_k=int(klen.max()), cu_seqlens_k=ck,
                                       softmax_scale=D ** -0.5, causal=True, block_table=btd)

            for _ in range(args.warmup):
                fa()
            ms_fa = timed(fa, args.steps, torch.cuda.current_stream(dev)) / args.steps
            res["flash_attn_varlen_func"] = {
                "impl": "flash-attn (reference GPU path, attention.py:64-70)",
                "value": round(flops / (ms_fa * 1e-3) / 1e12, 1), "unit": "TFLOP/s",
                "ms_per_step": round(ms_fa, 4)}
        except Exception as e:  # noqa: BLE001  (a comparison line never sinks the bench)
            res["flash_attn_varlen_func"] = {"unavailable": f"{e!r}"[:200]}
    return res


def bench_tree(dev, rank, world, args, tf_peak, hbm_peak):
    """32 seqs, ctx U[1024,8192], 64-node EAGLE tree (depth 6)."""
    from nvattn import ops, tree
    from nvattn.parallel import head_shard
    (q0, q1), (k0, k1) = head_shard(32, 8, rank, world)
    H, KVH = q1 - q0, k1 - k0
    rng = np.random.default_rng(5)
    B, N = 32, 64
    ctx = rng.integers(1024, 8193, size=B).astype(np.int64)
    parents, depths = tree.build_draft_tree((4, 3, 2, 1, 1, 1), N)
    masks = tree.ancestor_masks(parents)
    tot = ctx + N
    nblk = (tot + BS - 1) // BS
    nblocks = int(nblk.sum())
    perm = rng.permutation(nblocks).astype(np.int32)
    bt = np.full((B, int(nblk.max())), -1, np.int32)
    pos = 0
    for b in range(B):
        bt[b, :nblk[b]] = perm[pos:pos + nblk[b]]
        pos += nblk[b]
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    kc = torch.randn(nblocks, BS, KVH, D, generator=g, device=dev).to(torch.bfloat16)
    vc = torch.randn(nblocks, BS, KVH, D, generator=g, device=dev).to(torch.bfloat16)
    q = torch.randn(B * N, H, D, generator=g, device=dev).to(torch.bfloat16)
    cq = torch.arange(0, (B + 1) * N, N, dtype=torch.int32, device=dev)
    ctx_d = torch.from_numpy(ctx.astype(np.int32)).to(dev)
    m_d = torch.from_numpy(np.tile(masks, B).view(np.int64)).to(dev)
    btd = torch.from_numpy(bt).to(dev)
    out = torch.empty_like(q)
    n_anc = np.array([bin(int(x)).count("1") for x in masks])
    flops = float(sum(4 * D * H * (int(c) + int(a)) for c in ctx for a in n_anc))
    nbytes = float(int(tot.sum()) * KVH * D * 2 * 2 + 2 * B * N * H * D * 2)

    def fn():
        ops.tree_attention(q, kc, vc, cq, ctx_d, m_d, btd, N, softmax_scale=D ** -0.5, out=out)

    for _ in range(args.warmup):
        fn()
    barrier(world)
    ms = max_over_ranks(graph_timed(fn, max(3, args.steps // 10), dev),
                        world)
    tf = sum_over_ranks(flops, world) / (ms * 1e-3) / 1e12
    gbs = sum_over_ranks(nbytes, world) / (ms * 1e-3) / 1e9

    # configs[4] also runs an n-gram linear draft of 8 tokens per sequence:
    # the same contexts, a chain mask (node i sees nodes 0..i)
    NL = 8
    ql = torch.randn(B * NL, H, D, generator=g, device=dev).to(torch.bfloat16)
    cql = torch.arange(0, (B + 1) * NL, NL, dtype=torch.int32, device=dev)
    ml = torch.from_numpy(np.tile(tree.chain_masks(NL), B).view(np.int64)).to(dev)
    outl = torch.empty_like(ql)
    flops_l = float(sum(4 * D * H * (int(c) + i + 1) for c in ctx for i in range(NL)))

    def fn_l():
        ops.tree_attention(ql, kc, vc, cql, ctx_d, ml, btd, NL, softmax_scale=D ** -0.5, out=outl)

    for _ in range(args.warmup):
        fn_l()
    barrier(world)
    ms_l = max_over_ranks(graph_timed(fn_l, max(3, args.steps // 10), dev),
                          world)
    nbytes_l = float(int(ctx.sum() + B * NL) * KVH * D * 2 * 2)
    return {"metric": "tree-verify attn TFLOP/s", "value": round(tf, 1), "unit": "TFLOP/s",
            "GB_per_s": round(gbs, 1), "ms_per_step": round(ms, 4),
            "frac_of_measured_bf16_peak_per_gpu": round(tf / world / tf_peak, 4),
            "frac_of_measured_bf16_sustained_peak_per_gpu": round(tf / world / load_peaks()[2], 4),
            "frac_of_measured_hbm_per_gpu": round(gbs / world / hbm_peak, 4),
            "timing": "device time per call: 10 calls per CUDA graph, max over ranks",
            "workload": "configs[4]: 32 seqs, ctx U[1024,8192], 64-node tree (branching "
                        "[4,3,2,1,1,1], depth 6), 32Q/8KV, d128",
            "linear_draft_8": {
                "ms_per_step": round(ms_l, 4),
                "TFLOP_per_s": round(sum_over_ranks(flops_l, world) / (ms_l * 1e-3) / 1e12, 1),
                "GB_per_s": round(sum_over_ranks(nbytes_l, world) / (ms_l * 1e-3) / 1e9, 1),
                "frac_of_measured_hbm_per_gpu": round(
                    sum_over_ranks(nbytes_l, world) / (ms_l * 1e-3) / 1e9 / world / hbm_peak, 4),
                "workload": "same 32 contexts, 8-token n-gram chain per sequence"}}


def bench_store_kvcache(dev, args, hbm_peak):
    """The KV scatter alone (attention.py:10-40) at the Qwen3-0.6B shape
    (8 KV heads, d128, 256-token blocks): a 16,384-token prefill chunk
    (max_num_batched_tokens; slots in runs of whole blocks, blocks permuted,
    as prepare_prefill lays them out) and a 256-row decode batch (one random
    slot per sequence). K and V are strided views of a qkv projection
    (16Q/8KV), as Qwen3Attention passes them. Beside it the reference's own
    Triton kernel (store_kvcache) on the same inputs."""
    from nvattn import ops
    reference_on_path()
    try:
        from nanovllm.layers.attention import store_kvcache as ref_store
    except Exception as e:  # noqa: BLE001
        ref_store, ref_err = None, f"reference package not importable: {e!r}"[:200]
    H, KVH = 16, 8
    g = torch.Generator(device=dev).manual_seed(31)
    res = {"metric": "store_kvcache GB/s", "unit": "GB/s",
           "bytes": "2*N*KVH*d*2 read + the same written + 4N of slots",
           "timing": "10 calls per CUDA graph, device time per call (both implementations); "
                     "4 input sets and caches in turn (prefill: 4 x 201 MB, larger than L2)"}
    for name, n in (("prefill_chunk_16384", 16384), ("decode_batch_256", 256)):
        nb = max(64, (n + BS - 1) // BS * 2)
        sets = []
        for _ in range(4):
            qkv = torch.randn(n, (H + 2 * KVH) * D, generator=g, device=dev).to(torch.bfloat16)
            _, k, v = qkv.split([H * D, KVH * D, KVH * D], dim=-1)
            k, v = k.view(n, KVH, D), v.view(n, KVH, D)
            kc = torch.zeros(nb, BS, KVH, D, dtype=torch.bfloat16, device=dev)
            vc = torch.zeros_like(kc)
            if name.startswith("prefill"):
                blocks = torch.randperm(nb, generator=g, device=dev)[:(n + BS - 1) // BS]
                slots = (blocks[:, None] * BS + torch.arange(BS, device=dev)[None]).flatten()[:n]
            else:  # decode: one new token per sequence, each in its own block
                slots = torch.randperm(nb * BS, generator=g, device=dev)[:n]
            sets.append((qkv, k, v, kc, vc, slots.to(torch.int32)))
        nbytes = float(2 * n * KVH * D * 2 * 2 + 4 * n)
        turn = [0]

        def nxt():
            turn[0] = (turn[0] + 1) % len(sets)
            return sets[turn[0]]

        def nv_fn():
            _, k, v, kc, vc, sl = nxt()
            ops.store_kvcache(k, v, kc, vc, sl)

        for _ in range(args.warmup):
            nv_fn()
        ms = graph_timed(nv_fn, args.steps, dev)
        row = {"value": round(nbytes / (ms * 1e-3) / 1e9, 1), "us_per_call": round(ms * 1e3, 2),
               "frac_of_measured_hbm": round(nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 4),
               "bytes_per_call": nbytes}
        if ref_store is None:
            row["reference_triton"] = {"unavailable": ref_err}
        else:
            try:
                def ref_fn():
                    _, k, v, kc, vc, sl = nxt()
                    ref_store(k, v, kc, vc, sl)

                for _ in range(max(args.warmup, 3)):
                    ref_fn()
                ms_ref = graph_timed(ref_fn, args.steps, dev)
                row["reference_triton"] = {
                    "impl": "reference store_kvcache (Triton, attention.py:10-40)",
                    "value": round(nbytes / (ms_ref * 1e-3) / 1e9, 1),
                    "us_per_call": round(ms_ref * 1e3, 2)}
                # both wrote the same caches from the same inputs: check one set bit for bit
                _, k, v, kc, vc, sl = sets[0]
                ref_store(k, v, kc, vc, sl)
                kc2, vc2 = torch.zeros_like(kc), torch.zeros_like(vc)
                ops.store_kvcache(k, v, kc2, vc2, sl)
                kc3, vc3 = torch.zeros_like(kc), torch.zeros_like(vc)
                ref_store(k, v, kc3, vc3, sl)
                row["caches_identical_to_reference"] = bool(torch.equal(kc2, kc3) and
                                                            torch.equal(vc2, vc3))
            except Exception as e:  # noqa: BLE001
                row["reference_triton"] = {"unavailable": f"{e!r}"[:200]}
        res[name] = row
        del sets
        torch.cuda.empty_cache()
    res["value"] = res["prefill_chunk_16384"]["value"]
    return res


# Variables torchrun sets for its workers. A process started from a worker
# must not see them: with TORCHELASTIC_USE_AGENT_STORE set, every rank of a
# new tcp:// process group (the reference engine's, model_runner.py:26)
# connects as a client to a store nobody serves, and waits for the timeout.
_LAUNCHER_VARS = ("RANK", "LOCAL_RANK", "WORLD_SIZE", "LOCAL_WORLD_SIZE", "GROUP_RANK",
                  "GROUP_WORLD_SIZE", "ROLE_RANK", "ROLE_WORLD_SIZE", "ROLE_NAME",
                  "MASTER_ADDR", "MASTER_PORT")


def engine_env(base) -> dict:
    """The environment for an engine process started from a bench rank: no
    launcher variables, and the package, repository and reference install on
    PYTHONPATH."""
    env = {k: v for k, v in base.items()
           if k not in _LAUNCHER_VARS and not k.startswith("TORCHELASTIC_")}
    env["PYTHONPATH"] = os.pathsep.join([str(REPO / "nano-vllm-x_b200"), str(REPO),
                                         str(REPO / "baseline" / "_ref"),
                                         env.get("PYTHONPATH", "")])
    return env


def bench_store_sweep(dev, args):
    """The scatter at 64..16,384 tokens (one random slot each) beside the
    reference's Triton kernel: device time per call, 10 calls per CUDA graph,
    4 input sets and caches in turn."""
    from nvattn import ops
    reference_on_path()
    try:
        from nanovllm.layers.attention import store_kvcache as ref_store
    except Exception:  # noqa: BLE001
        ref_store = None
    H, KVH = 16, 8
    g = torch.Generator(device=dev).manual_seed(1)
    res = {"metric": "store_kvcache us per call", "unit": "us", "higher_is_better": False}
    for n in (64, 256, 1024, 2048, 4096, 16384):
        nb = max(64, (n + BS - 1) // BS * 2)
        sets = []
        for _ in range(4):
            qkv = torch.randn(n, (H + 2 * KVH) * D, generator=g, device=dev).to(torch.bfloat16)
            _, k, v = qkv.split([H * D, KVH * D, KVH * D], dim=-1)
            kc = torch.zeros(nb, BS, KVH, D, dtype=torch.bfloat16, device=dev)
            sl = torch.randperm(nb * BS, generator=g, device=dev)[:n].to(torch.int32)
            sets.append((k.view(n, KVH, D), v.view(n, KVH, D), kc, torch.zeros_like(kc), sl))
        turn = [0]

        def nxt():
            turn[0] = (turn[0] + 1) % len(sets)
            return sets[turn[0]]

        def nv():
            k, v, kc, vc, sl = nxt()
            ops.store_kvcache(k, v, kc, vc, sl)

        def rf():
            k, v, kc, vc, sl = nxt()
            ref_store(k, v, kc, vc, sl)

        # both implementations warmed up (the Triton kernel compiled) before either is timed
        for _ in range(max(args.warmup, 3)):
            nv()
            if ref_store is not None:
                rf()
        row = {"nvattn": round(graph_timed(nv, args.steps, dev) * 1e3, 2)}
        if ref_store is not None:
            row["reference_triton"] = round(graph_timed(rf, args.steps, dev) * 1e3, 2)
        res[f"tokens_{n}"] = row
        del sets
        torch.cuda.empty_cache()
    return res


def bench_e2e(args, world):
    """configs[1] end to end (the third part of the metric; the reference's
    bench.py:8-28 workload through its own engine): nvattn.e2e runs the fused
    nvattn arm and the reference arm at TP = world size, each in a fresh
    process, on the full 256-request workload, greedy. Returns tok/s, seconds
    and the number of requests whose ids are identical between the arms."""
    import tempfile
    reference_on_path()
    try:
        import nanovllm  # noqa: F401
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference engine not importable: {e!r}"[:200]}
    env = engine_env(os.environ)
    res = {"metric": "e2e out tok/s", "unit": "tok/s", "tp": world,
           "workload": "configs[1]: 256 requests (bench.py draw order, random.seed(0)), input and "
                       "output lengths U[100,1024], ignore_eos, greedy; random-init Qwen3-0.6B, "
                       "CUDA-graph decode; each arm in a fresh engine process",
           "timing": "wall clock of llm.generate after one warm-up request (engine set-up and "
                     "graph capture excluded), as the reference's bench.py times it"}
    with tempfile.TemporaryDirectory() as tmp:
        model_dir = Path(tmp) / "model"
        r = subprocess.run([sys.executable, "-m", "nvattn.e2e", "--write-model", str(model_dir)],
                           env=env, capture_output=True, text=True, timeout=600)
        if r.returncode != 0:
            return dict(res, error=r.stderr[-300:])
        outs = {}
        for arm in ("nvattn-fused", "reference"):
            out = Path(tmp) / f"{arm}.npz"
            cmd = [sys.executable, "-m", "nvattn.e2e", "--tp", str(world), "--attn", arm,
                   "--model-dir", str(model_dir), "--out", str(out)]
            try:
                r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=900)
            except subprocess.TimeoutExpired:
                res[arm] = {"error": "timed out after 900 s"}
                continue
            if r.returncode != 0:
                res[arm] = {"error": r.stderr[-300:]}
                continue
            line = json.loads(r.stdout.strip().splitlines()[-1])
            res[arm] = {"value": line["value"], "seconds": line["seconds"],
                        "output_tokens": line["output_tokens"]}
            if arm == "nvattn-fused" and world > 1:
                # decode-sized row-parallel all-reduces through nvattn's peer-memory kernel
                res[arm]["peer_memory_allreduce"] = bool(line.get("oneshot_allreduce"))
            outs[arm] = out
        if len(outs) == 2:
            sys.path.insert(0, str(REPO / "nano-vllm-x_b200"))
            from nvattn.e2e import compare
            cmp = compare(str(outs["reference"]), str(outs["nvattn-fused"]))
            res["identical_requests"] = cmp["identical"]
            res["requests"] = cmp["requests"]
            res["median_first_divergence_frac"] = cmp["median_first_divergence_frac"]
    if "value" in res.get("nvattn-fused", {}):
        res["value"] = res["nvattn-fused"]["value"]
    if "value" in res.get("reference", {}) and "value" in res:
        res["speedup_vs_reference"] = round(res["value"] / res["reference"]["value"], 3)
    return res


def bench_layer_cfg0(dev, args):
    """one attention layer at the Qwen3-0.6B shape (16Q/8KV, d128,
    block 256) through nvattn.Attention: 4 sequences with prompt lengths
    U[100,1024] (numpy seed 0), contiguous blocks, one prefill then 32 decode
    steps. Reports the latency of the whole sequence of calls."""
    import nvattn
    from nvattn import context as C
    H, KVH = 16, 8
    rng = np.random.default_rng(0)
    lens = rng.integers(100, 1025, size=4)
    steps = 32
    nblk = (lens + steps + BS - 1) // BS
    starts = np.concatenate([[0], np.cumsum(nblk)[:-1]])
    nb = int(nblk.sum())
    g = torch.Generator(device=dev).manual_seed(0)
    attn = nvattn.Attention(H, D, D ** -0.5, KVH)
    attn.k_cache = torch.zeros(nb, BS, KVH, D, dtype=torch.bfloat16, device=dev)
    attn.v_cache = torch.zeros_like(attn.k_cache)
    saved = nvattn.Attention.__dict__["get_context"]
    nvattn.Attention.get_context = staticmethod(C.get_context)
    N = int(lens.sum())
    q = torch.randn(N, H, D, generator=g, device=dev).to(torch.bfloat16)
    k = torch.randn(N, KVH, D, generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn(N, KVH, D, generator=g, device=dev).to(torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device=dev)
    slots_p = torch.tensor(np.concatenate([starts[b] * BS + np.arange(lens[b])
                                           for b in range(4)]), dtype=torch.int32, device=dev)
    bt = torch.tensor(np.minimum(np.stack([starts + i for i in range(int(nblk.max()))], axis=1),
                                 nb - 1), dtype=torch.int32, device=dev)
    qd = torch.randn(steps, 4, H, D, generator=g, device=dev).to(torch.bfloat16)
    kd = torch.randn(steps, 4, KVH, D, generator=g, device=dev).to(torch.bfloat16)
    vd = torch.randn(steps, 4, KVH, D, generator=g, device=dev).to(torch.bfloat16)
    dec = [(torch.tensor(starts * BS + lens + s, dtype=torch.int32, device=dev),
            torch.tensor(lens + s + 1, dtype=torch.int32, device=dev)) for s in range(steps)]

    def fn():
        C.set_context(True, cu, cu, int(lens.max()), int(lens.max()), slots_p, None, None)
        attn(q, k, v)
        for s in range(steps):
            C.set_context(False, slot_mapping=dec[s][0], context_lens=dec[s][1], block_tables=bt)
            attn(qd[s], kd[s], vd[s])
        C.reset_context()

    try:
        for _ in range(args.warmup):
            fn()
        ms = timed(fn, min(args.steps, 20), torch.cuda.current_stream(dev)) / min(args.steps, 20)
    finally:
        nvattn.Attention.get_context = saved
    return {"metric": "configs[0] layer latency", "value": round(ms, 4), "unit": "ms",
            "higher_is_better": False,
            "workload": "configs[0]: 1 attention layer, Qwen3-0.6B shape, 4 seqs U[100,1024], "
                        "prefill + 32 decode steps (eager, host launch included)"}


def bench_qknorm(dev, rank, world, args, hbm_peak):
    """q/k RMSNorm + rotary + KV scatter (qwen3.py:82-86) for one prefill chunk of
    the e2e model (Qwen3-0.6B: 16Q/8KV heads, 16384 tokens = max_num_batched_tokens),
    fused into one launch; beside it the reference's own four-launch sequence
    (compiled RMSNorm x2, compiled rotary, Triton store_kvcache) when the
    reference package is importable."""
    from nvattn import ops
    from nvattn.parallel import head_shard
    (q0, q1), (k0, k1) = head_shard(16, 8, rank, world)
    H, KVH, N, max_pos = q1 - q0, k1 - k0, 16384, 40960
    g = torch.Generator(device=dev).manual_seed(11 + rank)
    qkv = torch.randn(N, (H + 2 * KVH) * D, generator=g, device=dev).to(torch.bfloat16)
    q, k, v = qkv.split([H * D, KVH * D, KVH * D], dim=-1)
    q, k, v = q.view(N, H, D), k.view(N, KVH, D), v.view(N, KVH, D)
    pos = torch.randint(0, 4096, (N,), generator=g, device=dev)
    nb = N // BS + 4
    slots = torch.randperm(nb * BS, generator=g, device=dev)[:N].to(torch.int32)
    kc = torch.zeros(nb, BS, KVH, D, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    w = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).to(torch.bfloat16)
    inv_freq = 1.0 / (1e6 ** (torch.arange(0, D, 2, dtype=torch.float) / D))
    freqs = torch.einsum("i,j -> ij", torch.arange(max_pos, dtype=torch.float), inv_freq)
    cos_sin = torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1).to(dev)
    q_out = torch.empty(N, H, D, dtype=torch.bfloat16, device=dev)
    k_out = torch.empty(N, KVH, D, dtype=torch.bfloat16, device=dev)
    # algorithmic bytes: q/k/v rows read, q/k written, K/V cache rows written,
    # plus positions, slots and each token's cos/sin row
    nbytes = float(N * (H + 2 * KVH) * D * 2 + N * (H + KVH) * D * 2 + 2 * N * KVH * D * 2
                   + N * (8 + 4 + D * 4))

    def fn():
        ops.qk_norm_rope_store(pos, q, k, v, w, w, cos_sin, 1e-6, kc, vc, slots,
                               q_out=q_out, k_out=k_out)

    for _ in range(args.warmup):
        fn()
    barrier(world)
    ms = max_over_ranks(graph_timed(fn, max(3, args.steps // 10), dev),
                        world)
    gbs = sum_over_ranks(nbytes, world) / (ms * 1e-3) / 1e9
    res = {"metric": "fused q/k-norm+rotary+KV-scatter GB/s", "value": round(gbs, 1),
           "unit": "GB/s", "ms_per_step": round(ms, 4),
           "frac_of_measured_hbm_per_gpu": round(gbs / world / hbm_peak, 4),
           "bytes_per_step": sum_over_ranks(nbytes, world),
           "timing": "device time per call: 10 calls per CUDA graph, max over ranks",
           "workload": "Qwen3-0.6B prefill chunk: 16384 tokens, 16Q/8KV, d128, random slots"}
    if world == 1:
        res["reference_four_launch"] = _reference_qknorm(dev, args, pos, q, k, v, w, cos_sin, kc,
                                                         vc, slots, nbytes)
    return res


def _reference_qknorm(dev, args, pos, q, k, v, w, cos_sin, kc, vc, slots, nbytes):
    """The reference's modules on the same inputs: RMSNorm (layernorm.py:16-26,
    torch.compile), RotaryEmbedding (rotary_embedding.py:37-48, torch.compile)
    and the Triton store_kvcache (attention.py:10-40)."""
    reference_on_path()
    try:
        from nanovllm.layers.attention import store_kvcache
        from nanovllm.layers.layernorm import RMSNorm
        from nanovllm.layers.rotary_embedding import RotaryEmbedding
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference package not importable: {e!r}"[:200]}
    try:
        qn, kn = RMSNorm(D, 1e-6).to(dev), RMSNorm(D, 1e-6).to(dev)
        with torch.no_grad():
            qn.weight.copy_(w.float())
            kn.weight.copy_(w.float())
        qn, kn = qn.to(torch.bfloat16), kn.to(torch.bfloat16)
        rope = RotaryEmbedding(D, D, cos_sin.shape[0], 1e6).to(dev)

        def fn():
            with torch.no_grad():
                qq, kk = rope(pos, qn(q), kn(k))
                store_kvcache(kk, v, kc, vc, slots)

        for _ in range(max(args.warmup, 3)):
            fn()
        ms = timed(fn, args.steps, torch.cuda.current_stream(dev)) / args.steps
        return {"impl": "reference modules (compiled RMSNorm x2 + rotary, Triton scatter)",
                "value": round(nbytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                "ms_per_step": round(ms, 4)}
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference modules did not run: {e!r}"[:200]}


def bench_sampler(dev, args, hbm_peak):
    """One decode step's sampling for the e2e batch: 256 rows of Qwen3 logits
    (vocab 151936, bf16). nvattn's one-pass kernel, sampled (T = 1) and greedy,
    beside the reference's Sampler (sampler.py:5-12, torch.compile) and
    torch.argmax when available."""
    from nvattn import ops
    B, V = 256, 151936
    g = torch.Generator(device=dev).manual_seed(21)
    # four logits buffers (311 MB) used in turn, so no call reads logits that
    # the previous calls left in the 126 MB L2
    bufs = [(torch.randn(B, V, generator=g, device=dev) * 3).to(torch.bfloat16) for _ in range(4)]
    logits = bufs[0]
    turn = [0]

    def next_logits():
        turn[0] = (turn[0] + 1) % len(bufs)
        return bufs[turn[0]]

    t = torch.ones(B, dtype=torch.float32, device=dev)
    out = torch.empty(B, dtype=torch.int64, device=dev)
    nbytes = float(B * V * 2)
    res = {"metric": "sampler logits GB/s", "unit": "GB/s",
           "workload": "256 rows x 151936 bf16 logits (Qwen3 vocab), T = 1 and greedy",
           "l2": "4 logits buffers (311 MB) in turn, larger than L2"}
    res["timing"] = ("nvattn: 10 calls per CUDA graph, device time per call (3 launches: key "
                     "reset, chunk kernel, merge); reference and argmax: eager calls")
    for name, fn in (("sampled", lambda: ops.sample(next_logits(), t, seed=1, offset=0, out=out)),
                     ("greedy", lambda: ops.sample(next_logits(), out=out))):
        for _ in range(args.warmup):
            fn()
        ms = graph_timed(fn, args.steps, dev)
        res[name] = {"value": round(nbytes / (ms * 1e-3) / 1e9, 1), "ms_per_step": round(ms, 4),
                     "frac_of_measured_hbm": round(nbytes / (ms * 1e-3) / 1e9 / hbm_peak, 4)}
        if args.warmup:
            ms_eager = timed(fn, args.steps, torch.cuda.current_stream(dev)) / args.steps
            res[name]["ms_per_call_eager"] = round(ms_eager, 4)
    res["value"] = res["sampled"]["value"]
    # one rank's share of vocabulary-parallel sampling at TP2: the pick keys of
    # its 75,968 columns and the merge of both ranks' keys (the 4 KB all-gather
    # between them needs a second GPU and is not in this number)
    keys2 = torch.zeros(2, B, dtype=torch.int64, device=dev)

    def shard_fn():
        ops.sample_shard(next_logits()[:, :V // 2], 0, t, seed=1, offset=0, out=keys2[0])
        ops.sample_merge(keys2, out=out)

    for _ in range(args.warmup):
        shard_fn()
    ms = graph_timed(shard_fn, args.steps, dev)
    res["tp2_rank_shard_sampled"] = {"value": round(nbytes / 2 / (ms * 1e-3) / 1e9, 1),
                                     "ms_per_step": round(ms, 4)}
    reference_on_path()
    try:
        from nanovllm.layers.sampler import Sampler
        sampler = Sampler()

        def ref_fn():
            sampler(next_logits(), t)

        for _ in range(max(args.warmup, 3)):
            ref_fn()
        ms = timed(ref_fn, args.steps, torch.cuda.current_stream(dev)) / args.steps
        res["reference_sampler"] = {"impl": "reference Sampler (torch.compile)",
                                    "value": round(nbytes / (ms * 1e-3) / 1e9, 1),
                                    "ms_per_step": round(ms, 4)}
    except Exception as e:  # noqa: BLE001
        res["reference_sampler"] = {"unavailable": f"{e!r}"[:200]}

    def argmax_fn():
        torch.argmax(next_logits(), dim=-1)

    for _ in range(args.warmup):
        argmax_fn()
    ms = timed(argmax_fn, args.steps, torch.cuda.current_stream(dev)) / args.steps
    res["torch_argmax"] = {"value": round(nbytes / (ms * 1e-3) / 1e9, 1), "ms_per_step": round(ms, 4)}
    return res


def bench_decode_prepare(dev, args):
    """One decode step's metadata for the e2e batch: 256 sequences of
    U[100, 2048] tokens in 256-token blocks, written into CUDA-graph inputs of
    512 rows x 16 blocks. The reference arm runs the reference's own
    ModelRunner.prepare_decode and run_model (model_runner.py:172-188,
    196-212) on a stand-in runner whose graph replay and logits are no-ops;
    nvattn packs one record and launches nvattn_decode_prepare. Host wall
    time per step with a synchronisation after each step, as the engine
    synchronises on its sampled tokens."""
    import random
    import time
    from types import SimpleNamespace

    from nvattn.decode_meta import DecodeMetadata
    reference_on_path()
    try:
        from nanovllm.engine.model_runner import ModelRunner
        from nanovllm.engine.sequence import Sequence
        from nanovllm.sampling_params import SamplingParams
        from nanovllm.utils.context import reset_context
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference engine not importable: {e!r}"[:200]}
    rnd = random.Random(0)
    seqs = []
    for i in range(256):
        s = Sequence([rnd.randint(0, 10000) for _ in range(rnd.randint(100, 2048))],
                     SamplingParams(ignore_eos=True, max_tokens=64))
        s.block_table = list(range(i * 16, i * 16 + (len(s) + 255) // 256))
        seqs.append(s)
    rows, width = 512, 16

    def graph_vars():
        return dict(input_ids=torch.zeros(rows, dtype=torch.int64, device=dev),
                    positions=torch.zeros(rows, dtype=torch.int64, device=dev),
                    slot_mapping=torch.zeros(rows, dtype=torch.int32, device=dev),
                    context_lens=torch.zeros(rows, dtype=torch.int32, device=dev),
                    block_tables=torch.zeros(rows, width, dtype=torch.int32, device=dev),
                    outputs=torch.zeros(rows, 8, device=dev))

    fake = SimpleNamespace(block_size=256, enforce_eager=False, graph_bs=[256, 512],
                           graphs={256: SimpleNamespace(replay=lambda: None),
                                   512: SimpleNamespace(replay=lambda: None)},
                           graph_vars=graph_vars(),
                           model=SimpleNamespace(compute_logits=lambda x: None))
    fake.prepare_block_tables = lambda ss: ModelRunner.prepare_block_tables(fake, ss)

    def ref_step():
        ids, pos = ModelRunner.prepare_decode(fake, seqs)
        ModelRunner.run_model(fake, ids, pos, False)
        reset_context()

    meta = DecodeMetadata(512, width, 256, dev)
    gv = graph_vars()
    del gv["outputs"]

    def nv_step():
        meta.pack(seqs)
        meta.launch(rows, **gv)

    def wall(fn):
        for _ in range(args.warmup):
            fn()
            torch.cuda.synchronize(dev)
        n = max(args.steps, 20)
        t = time.perf_counter()
        for _ in range(n):
            fn()
            torch.cuda.synchronize(dev)
        return (time.perf_counter() - t) / n * 1e3

    ms_ref = wall(ref_step)
    ms_nv = wall(nv_step)
    # the same outputs from both paths
    same = all(torch.equal(fake.graph_vars[k], gv[k]) for k in gv)
    return {"metric": "decode-step metadata, host wall ms per step", "unit": "ms",
            "higher_is_better": False, "value": round(ms_nv, 4),
            "reference_prepare_decode_and_copies": round(ms_ref, 4),
            "outputs_identical": bool(same), "gpu_launches_per_step": 1,
            "workload": "256 sequences, U[100, 2048] tokens, 256-token blocks; graph inputs "
                        "512 rows x 16 blocks; synchronised each step"}


def bench_decode_e2e_shape(dev, args, hbm_peak, batches=(16, 64, 256)):
    """Paged decode at the e2e model's shape (Qwen3-0.6B: 16Q/8KV, d128, 256-token
    blocks) for batches of 16/64/256 sequences with contexts U[100,2048]
    (numpy seed = batch), physical blocks permuted; flash-attn's decode on the
    same caches beside it. Device time per call, 10 calls per CUDA graph;
    caches used in turn so that >= 200 MB is touched between two reads of one."""
    from nvattn import ops
    try:
        from flash_attn import flash_attn_with_kvcache
    except Exception:  # noqa: BLE001
        flash_attn_with_kvcache = None
    H, KVH = 16, 8
    res = {"metric": "paged decode GB/s at the e2e shape", "unit": "GB/s",
           "workload": "16Q/8KV, d128, ctx U[100,2048], permuted 256-token blocks",
           "timing": "10 calls per CUDA graph, device time per call; several caches in turn"}
    for B in batches:
        rng = np.random.default_rng(B)
        lens = rng.integers(100, 2049, size=B).astype(np.int32)
        nblk = (lens + BS - 1) // BS
        tot = int(nblk.sum())
        perm = rng.permutation(tot).astype(np.int32)
        bt = np.full((B, int(nblk.max())), -1, np.int32)
        pos = 0
        for b in range(B):
            bt[b, :nblk[b]] = perm[pos:pos + nblk[b]]
            pos += nblk[b]
        nbytes = int(lens.astype(np.int64).sum()) * KVH * D * 4
        g = torch.Generator(device=dev).manual_seed(B)
        sets = []
        for _ in range(max(1, min(4, int(200e6 // nbytes) + 1))):
            kc = torch.randn(tot, BS, KVH, D, generator=g, device=dev).to(torch.bfloat16)
            vc = torch.randn(tot, BS, KVH, D, generator=g, device=dev).to(torch.bfloat16)
            sets.append((kc, vc))
        q = torch.randn(B, H, D, generator=g, device=dev).to(torch.bfloat16)
        ld, bd = torch.from_numpy(lens).to(dev), torch.from_numpy(bt).to(dev)
        ws = torch.empty(max(1, ops.decode_workspace_bytes(B, H, KVH, bt.shape[1], BS)),
                         dtype=torch.uint8, device=dev)
        out = torch.empty(B, H, D, dtype=torch.bfloat16, device=dev)
        turn = [0]

        def nxt():
            turn[0] = (turn[0] + 1) % len(sets)
            return sets[turn[0]]

        def nv():
            kc, vc = nxt()
            ops.paged_decode(q, kc, vc, ld, bd, softmax_scale=D ** -0.5, workspace=ws, out=out)

        for _ in range(args.warmup):
            nv()
        ms = graph_timed(nv, args.steps, dev)
        row = {"us": round(ms * 1e3, 2), "value": round(nbytes / ms / 1e6, 1),
               "frac_of_measured_hbm": round(nbytes / ms / 1e6 / hbm_peak, 4), "kv_bytes": nbytes}
        if flash_attn_with_kvcache is not None:
            q4 = q.unsqueeze(1)

            def fa():
                kc, vc = nxt()
                flash_attn_with_kvcache(q4, kc, vc, cache_seqlens=ld, block_table=bd,
                                        softmax_scale=D ** -0.5, causal=True)

            for _ in range(args.warmup):
                fa()
            ms_fa = graph_timed(fa, args.steps, dev)
            row["flash_attn"] = {"us": round(ms_fa * 1e3, 2), "value": round(nbytes / ms_fa / 1e6, 1)}
        res[f"batch_{B}"] = row
        del sets
        torch.cuda.empty_cache()
    return res


def bench_flash_attn_decode(dev, args, H, KVH):
    """The reference's own GPU decode call (flash-attn, attention.py:72-74) on the
    same workload, for comparison; reports why if it cannot run."""
    try:
        from flash_attn import flash_attn_with_kvcache
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"flash-attn import failed: {e!r}"[:200]}
    try:
        lens, bt_np, nblocks = decode_workload(0)
        g = torch.Generator(device=dev).manual_seed(5)
        kc = torch.randn(nblocks, BS, KVH, D, generator=g, device=dev).to(torch.bfloat16)
        vc = torch.randn(nblocks, BS, KVH, D, generator=g, device=dev).to(torch.bfloat16)
        q = torch.randn(BATCH, 1, H, D, generator=g, device=dev).to(torch.bfloat16)
        lens_d = torch.from_numpy(lens).to(dev)
        bt_d = torch.from_numpy(bt_np).to(dev)

        def fn():
            flash_attn_with_kvcache(q, kc, vc, cache_seqlens=lens_d, block_table=bt_d,
                                    softmax_scale=D ** -0.5, causal=True)

        for _ in range(args.warmup):
            fn()
        ms = timed(fn, args.steps, torch.cuda.current_stream(dev)) / args.steps
        nbytes = decode_bytes(lens, KVH, H) - 2 * BATCH * KVH * D * 2 * 2
        return {"impl": "flash-attn (reference GPU path)", "value": round(nbytes / ms / 1e6, 1),
                "unit": "GB/s", "ms_per_step": round(ms, 4)}
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"flash-attn did not run: {e!r}"[:200]}


# ---------------------------------------------------------- CPU baseline

_POOL = None


def _cpu_pool():
    global _POOL
    if _POOL is None:
        lens, _, _ = decode_workload(0)
        gen = torch.Generator().manual_seed(4321)
        nb_max = int((lens.max() + BS - 1) // BS)
        kc = torch.randn(nb_max, BS, KVH_TOTAL, D, generator=gen).to(torch.bfloat16)
        vc = torch.randn(nb_max, BS, KVH_TOTAL, D, generator=gen).to(torch.bfloat16)
        q = torch.randn(1, H_TOTAL, D, generator=gen).to(torch.bfloat16)
        bt = np.arange(nb_max, dtype=np.int32).reshape(1, nb_max)
        _POOL = (lens, kc, vc, q, bt)
    return _POOL


CPU_SAMPLE_SEQS = 32  # the CPU sample: the workload's first 32 sequences, all heads


def _cpu_impl():
    sys.path.insert(0, str(REPO))
    from oracle import reference_math as R
    lens, kc, vc, q, bt = _cpu_pool()
    # the C restatement (OpenMP over sequence x KV head) when built, else torch's
    impl, how = R.decode_attention_c, "C restatement (oracle/decode_ref.c), OpenMP"
    try:
        impl(q, kc, vc, np.array([1]), bt, D ** -0.5)
    except OSError:
        impl, how = R.decode_attention, "torch fp32 restatement (oracle)"
    return impl, how


def cpu_decode_pass(impl, nseq: int = CPU_SAMPLE_SEQS):
    """One oracle decode call over the workload's first `nseq` sequences (all
    64Q/8KV heads; OpenMP over the nseq x 8 (sequence, KV head) pairs, so every
    host thread works). The oracle's cost does not depend on the values, so
    one random KV pool is generated once and every sequence reads its first
    ceil(ctx/256) blocks of it. Returns (algorithmic KV bytes, seconds)."""
    lens, kc, vc, q, bt = _cpu_pool()
    sl = lens[:nseq].astype(np.int32)
    qb = q.expand(nseq, -1, -1).contiguous()
    btb = np.repeat(bt, nseq, axis=0)
    t0 = time.perf_counter()
    impl(qb, kc, vc, sl, btb, D ** -0.5)
    dt = time.perf_counter() - t0
    return int(sl.astype(np.int64).sum()) * KVH_TOTAL * D * 2 * 2, dt


def cpu_decode_sample(budget_s: float):
    """The CPU baseline: passes of cpu_decode_pass over the same sample until
    `budget_s` seconds of CPU time (at least two); all host threads."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    impl, how = _cpu_impl()
    cpu_decode_pass(impl, 2)  # warm-up (page in the pool)
    done_bytes, t_total, n = 0, 0.0, 0
    while n < 2 or t_total < budget_s:
        nb, dt = cpu_decode_pass(impl)
        done_bytes += nb
        t_total += dt
        n += 1
    return {"value": round(done_bytes / t_total / 1e9, 3), "unit": "GB/s", "cores": threads,
            "kind": "port",
            "sample": f"the workload's first {CPU_SAMPLE_SEQS} of {BATCH} sequences (all "
                      f"64Q/8KV heads) per pass, {n} passes, {t_total:.2f} s of CPU time, {how}, "
                      f"{threads} threads"}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return  # the CPU reference runs on rank 0 only
    # each step: one pass of the oracle over the same bounded sample as cpu_baseline
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    impl, how = _cpu_impl()
    for _ in range(args.warmup):
        cpu_decode_pass(impl, 2)
    vals, total_s = [], 0.0
    for _ in range(max(1, args.steps)):
        nb, dt = cpu_decode_pass(impl)
        vals.append(nb / dt / 1e9)
        total_s += dt
    value = round(statistics.median(vals), 3)
    sample = (f"the workload's first {CPU_SAMPLE_SEQS} of {BATCH} sequences (all 64Q/8KV heads) "
              f"per step, {how}, {threads} threads")
    line = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_s * 1e3 / max(1, args.steps), 2),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD, "global_batch": BATCH, "num_heads": H_TOTAL,
                   "num_kv_heads": KVH_TOTAL, "head_dim": D, "block_size": BS,
                   "parallelism": "cpu (host cores)"},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads,
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_only(args):
    """One secondary workload alone (used to profile its kernel)."""
    rank, world, local = dist_setup(args.gpus)
    dev = torch.device("cuda", local)
    hbm_peak, tf_peak, _, _ = load_peaks()
    if args.only == "prefill":
        res = bench_prefill(dev, rank, world, args, tf_peak)
    elif args.only == "qknorm":
        res = bench_qknorm(dev, rank, world, args, hbm_peak)
    elif args.only == "sampler":
        res = bench_sampler(dev, args, hbm_peak)
    elif args.only == "layer":
        res = bench_layer_cfg0(dev, args)
    elif args.only == "prep":
        res = bench_decode_prepare(dev, args)
    elif args.only == "store":
        res = bench_store_kvcache(dev, args, hbm_peak)
    elif args.only == "store_sweep":
        res = bench_store_sweep(dev, args)
    elif args.only == "decode_small":
        res = bench_decode_e2e_shape(dev, args, hbm_peak, batches=(args.batch,))
    elif args.only == "e2e":
        torch.cuda.empty_cache()
        res = bench_e2e(args, world) if rank == 0 else None
        if world > 1:
            import torch.distributed as dist
            dist.barrier(group=_gloo_group())
    else:
        res = bench_tree(dev, rank, world, args, tf_peak, hbm_peak)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("nvattn", "reference"), default="nvattn")
    ap.add_argument("--batch", type=int, default=BATCH,
                    help="decode batch (configs[3] = 128; smaller values only for ncu captures)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--skip-secondary", action="store_true")
    ap.add_argument("--only", choices=("prefill", "tree", "qknorm", "sampler", "layer", "prep",
                                       "store", "store_sweep", "e2e", "decode_small"),
                    default=None,
                    help="run just one secondary workload and print its line (for profiling)")
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--skip-e2e", action="store_true",
                    help="leave out the end-to-end generation leg (configs[1])")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.only:
        run_only(args)
    else:
        run_nvattn(args)


if __name__ == "__main__":
    main()
