"""Vocabulary-parallel sampling over NCCL on two GPUs.

Each rank holds its half of the LM head's logits (embed_head.py:56-61),
picks within it (nvattn_sample_shard) and the ranks all-gather one 64-bit
key per row; the merged tokens must equal the one-GPU sampler on the whole
row, bit for bit, on every rank. Skipped with fewer than two GPUs.
"""
from __future__ import annotations

import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.multiprocessing as mp

from conftest import REPO, PROJECT

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, paths, result_q):
    import sys
    for p in paths:
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok = True
    try:
        from nvattn import ops
        from nvattn.parallel import sample_vocab_parallel, vocab_shard
        dev = torch.device("cuda", rank)
        for B, V, seed in ((256, 151936, 5), (3, 1000, 6), (64, 151936, 7)):
            g = torch.Generator(device=dev).manual_seed(seed)  # same logits on every rank
            logits = (torch.randn(B, V, generator=g, device=dev) * 2).to(torch.bfloat16)
            t = torch.rand(B, generator=g, device=dev) + 0.5
            t[::2] = 0.0
            whole = ops.sample(logits, t, seed=99, offset=seed)
            a, b = vocab_shard(V, rank, world)
            got = sample_vocab_parallel(logits[:, a:b], t, vocab_offset=a, seed=99, offset=seed)
            torch.cuda.synchronize()
            ok = ok and torch.equal(got, whole)
        result_q.put((rank, ok))
    except Exception:
        result_q.put((rank, False))
        raise
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_vocab_parallel_sampling_two_gpus_equals_one():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    result_q = ctx.Queue()
    port = _free_port()
    paths = [str(REPO), str(PROJECT)]
    procs = [ctx.Process(target=_worker, args=(r, 2, port, paths, result_q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        results = dict(result_q.get(timeout=240) for _ in range(2))
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: True, 1: True}
