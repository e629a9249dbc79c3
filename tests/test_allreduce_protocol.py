"""The one-shot all-reduce's flag protocol, emulated on the CPU.

allreduce_oneshot_kernel (csrc/allreduce.cu) synchronises ranks through
flags in each rank's shared buffer: announce the launch count e to every
rank, wait until every rank announced e, sum the partials, count finished
blocks, and let the last block announce "finished reading e", wait for
every rank's end flag and record e. Here each rank is a sequence of launches
whose blocks are Python threads running those steps on shared arrays, with
random delays to shuffle the interleavings; between launches the rank's
"GEMM" overwrites its partial (stream order: only after its previous launch
has completed). Every launch's output must be the sum of that launch's
partials. A planted mistake, the end barrier left out, must be caught: a
fast rank then overwrites its partial while a slow peer still reads it.
"""
from __future__ import annotations

import random
import threading
import time

import numpy as np


class _Rank:
    def __init__(self, n):
        self.start = np.zeros(8, np.int64)
        self.end = np.zeros(8, np.int64)
        self.epoch = 0
        self.done = 0
        self.lock = threading.Lock()
        self.data = np.zeros(n, np.int64)


def _wait(cond, limit=30.0):
    t0 = time.monotonic()
    while not cond():
        if time.monotonic() - t0 > limit:
            return False
        time.sleep(0)
    return True


def _run(world, blocks, launches, n, end_barrier=True, seed=0):
    ranks = [_Rank(n) for _ in range(world)]
    rng = random.Random(seed)
    delays = [[rng.random() * 2e-4 for _ in range(launches)] for _ in range(world)]
    outputs = [[None] * launches for _ in range(world)]
    timeouts = []

    def partial(r, k):
        return np.arange(n, dtype=np.int64) * (k + 1) + 1000 * r

    def block(r, b, k, out):
        me = ranks[r]
        e = me.epoch + 1
        for p in range(world):                        # announce
            ranks[p].start[r] = e
        for p in range(world):                        # wait for every rank's announcement
            if not _wait(lambda: ranks[r].start[p] >= e):
                timeouts.append(("start", r, k))
        time.sleep(delays[r][k] * rng.random())
        for i in range(b, n, blocks):                 # this block's slice, rank order
            acc = 0
            for p in range(world):
                acc += int(ranks[p].data[i])
                time.sleep(0)
            out[i] = acc
        with me.lock:                                 # count finished blocks
            prev = me.done
            me.done += 1
        if prev == blocks - 1:                        # the last block
            if end_barrier:
                for p in range(world):
                    ranks[p].end[r] = e
                for p in range(world):
                    if not _wait(lambda: ranks[r].end[p] >= e):
                        timeouts.append(("end", r, k))
            me.done = 0
            me.epoch = e

    def stream(r):
        for k in range(launches):
            ranks[r].data[:] = partial(r, k)           # the GEMM before the launch
            time.sleep(delays[r][k])
            out = np.zeros(n, np.int64)
            threads = [threading.Thread(target=block, args=(r, b, k, out)) for b in range(blocks)]
            for t in threads:
                t.start()
            for t in threads:
                t.join()                               # the launch completes
            outputs[r][k] = out

    streams = [threading.Thread(target=stream, args=(r,)) for r in range(world)]
    for t in streams:
        t.start()
    for t in streams:
        t.join()
    want = [sum(partial(r, k) for r in range(world)) for k in range(launches)]
    correct = all(np.array_equal(outputs[r][k], want[k])
                  for r in range(world) for k in range(launches))
    return correct, timeouts


def test_protocol_gives_every_launch_its_own_sum():
    for world, blocks, seed in ((2, 3, 0), (3, 2, 1), (4, 3, 2)):
        ok, timeouts = _run(world, blocks, launches=12, n=24, seed=seed)
        assert ok and not timeouts, (world, blocks, timeouts)


def test_protocol_without_the_end_barrier_is_caught():
    caught = False
    for seed in range(6):
        ok, _ = _run(2, 2, launches=12, n=24, end_barrier=False, seed=seed)
        caught = caught or not ok
        if caught:
            break
    assert caught
