"""Multi-rank host logic on CPU (gloo, world size 2).

The attention path shards by head across tensor-parallel ranks with no
collective inside attention (qwen3.py:29-35, model_runner.py:110). These
tests run two gloo ranks on the CPU: each rank computes the oracle on its own
head shard (nvattn.parallel.head_shard), the shards are gathered, and the
result must equal the unsharded computation; the bench's max-over-ranks /
sum-over-ranks reductions are checked the same way. The vocabulary-parallel
sampler's exchange (nvattn.parallel.gather_pick_keys) runs on oracle keys of
each rank's vocabulary shard and must give the gathered row's argmax.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import REPO  # noqa: F401  (sets import paths)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q, result_q):
    import sys
    for p in q["paths"]:
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from nvattn.parallel import head_shard
        from oracle import reference_math as R
        import bench
        (q0, q1), (k0, k1) = head_shard(q["H"], q["KVH"], rank, world)
        # decode on this rank's shard of the paged cache
        out = R.decode_attention(q["q"][:, q0:q1], q["kc"][:, :, k0:k1], q["vc"][:, :, k0:k1],
                                 q["lens"], q["bt"], 128 ** -0.5)
        parts = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(parts, out)
        # prefill on the shard (dense varlen)
        pf = R.varlen_attention(q["pq"][:, q0:q1], q["pk"][:, k0:k1], q["pv"][:, k0:k1],
                                q["cu"], q["cu"], 128 ** -0.5, True)
        pparts = [torch.empty_like(pf) for _ in range(world)]
        dist.all_gather(pparts, pf)
        # vocabulary-parallel sampling: each rank's pick keys over its own
        # columns, exchanged with one all-gather of B x 8 bytes, merged
        from nvattn.parallel import gather_pick_keys, vocab_shard
        v0, v1 = vocab_shard(q["logits"].shape[1], rank, world)
        keys = torch.from_numpy(R.greedy_shard_keys(q["logits"][:, v0:v1], v0).view(np.int64))
        all_keys = gather_pick_keys(keys)
        toks = R.merge_pick_keys(all_keys.numpy().view(np.uint64))
        mx = bench.max_over_ranks(float(rank + 1), world, device="cpu")
        sm = bench.sum_over_ranks(float(rank + 1), world, device="cpu")
        if rank == 0:
            result_q.put((torch.cat(parts, dim=1).numpy(), torch.cat(pparts, dim=1).numpy(), mx, sm,
                          toks, tuple(all_keys.shape)))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_head_sharded_attention_equals_unsharded_world2():
    g = torch.Generator().manual_seed(0)
    H, KVH, BS = 16, 8, 256
    lens = np.array([5, 300, 700], np.int32)
    nblk = (lens + BS - 1) // BS
    bt = np.full((3, int(nblk.max())), -1, np.int32)
    pos = 0
    for b, n in enumerate(nblk):
        bt[b, :n] = np.arange(pos, pos + n)
        pos += n
    kc = torch.randn(pos, BS, KVH, 128, generator=g).bfloat16()
    vc = torch.randn(pos, BS, KVH, 128, generator=g).bfloat16()
    q = torch.randn(3, H, 128, generator=g).bfloat16()
    plens = [7, 40]
    cu = np.concatenate([[0], np.cumsum(plens)]).astype(np.int32)
    pq = torch.randn(47, H, 128, generator=g).bfloat16()
    pk = torch.randn(47, KVH, 128, generator=g).bfloat16()
    pv = torch.randn(47, KVH, 128, generator=g).bfloat16()
    logits = (torch.randn(5, 1000, generator=g) * 3).round().bfloat16()  # ties across the border
    logits[0, 500] = logits[0, 499] = 50.0
    from conftest import GOLDEN, PROJECT
    payload = dict(H=H, KVH=KVH, q=q, kc=kc, vc=vc, lens=lens, bt=bt, pq=pq, pk=pk, pv=pv, cu=cu,
                   logits=logits,
                   paths=[str(REPO), str(PROJECT), str(GOLDEN)])
    ctx = mp.get_context("spawn")
    result_q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, payload, result_q)) for r in range(2)]
    for p in procs:
        p.start()
    dec, pre, mx, sm, toks, kshape = result_q.get()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    dec, pre = torch.from_numpy(dec), torch.from_numpy(pre)
    from oracle import reference_math as R
    full_dec = R.decode_attention(q, kc, vc, lens, bt, 128 ** -0.5)
    full_pre = R.varlen_attention(pq, pk, pv, cu, cu, 128 ** -0.5, True)
    assert torch.allclose(dec, full_dec, atol=1e-6)
    assert torch.allclose(pre, full_pre, atol=1e-6)
    assert mx == 2.0 and sm == 3.0
    assert kshape == (2, 5)
    assert np.array_equal(toks, R.greedy_tokens(logits).numpy()) and toks[0] == 499


def test_engine_env_lets_a_child_set_up_its_own_process_group():
    """bench.py runs the end-to-end engine in a child of a torchrun rank. The
    child's environment (bench.engine_env) must carry none of torchrun's
    variables: with TORCHELASTIC_USE_AGENT_STORE inherited, a tcp:// process
    group never finds its store and waits out its timeout."""
    import subprocess
    import sys

    import bench
    port = _free_port()
    rank_env = dict(os.environ, RANK="0", LOCAL_RANK="0", WORLD_SIZE="2", MASTER_ADDR="127.0.0.1",
                    MASTER_PORT=str(_free_port()), TORCHELASTIC_USE_AGENT_STORE="True",
                    TORCHELASTIC_RESTART_COUNT="0", TORCHELASTIC_RUN_ID="x", GROUP_RANK="0")
    env = bench.engine_env(rank_env)
    assert not [k for k in env if k.startswith("TORCHELASTIC_")]
    assert "RANK" not in env and "MASTER_PORT" not in env
    assert str(REPO / "nano-vllm-x_b200") in env["PYTHONPATH"].split(os.pathsep)
    probe = ("import datetime, torch.distributed as dist; "
             f"dist.init_process_group('gloo', 'tcp://127.0.0.1:{port}', world_size=1, rank=0, "
             "timeout=datetime.timedelta(seconds=20)); print('ok'); dist.destroy_process_group()")
    r = subprocess.run([sys.executable, "-c", probe], env=env, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stderr[-500:]
