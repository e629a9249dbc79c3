"""The one-shot all-reduce's flag protocol, emulated on the CPU.

allreduce_oneshot_kernel (csrc/allreduce.cu) cuts the message into one chunk
per block. In launch e, block b of every rank copies its chunk of the rank's
input into half e % 2 of the rank's shared buffer, publishes e into
flag[rank][b] of every rank, waits until flag[p][b] of its own buffer has
reached e for every rank p, sums chunk b of half e % 2 over the ranks, and
the last block to finish records e. There is no closing barrier: the two
halves stand in for it.

Here each rank is a sequence of launches whose blocks are Python threads
running those steps on shared arrays, with random delays to shuffle the
interleavings; a launch completes when all its blocks have (stream order).
Every launch's output must be the sum of that launch's inputs. A planted
mistake, one data half instead of two, must be caught: a fast rank then
overwrites its chunk while a slow peer still reads the previous launch's.
"""
from __future__ import annotations

import random
import threading
import time

import numpy as np


class _Rank:
    def __init__(self, world, blocks, n):
        self.flag = np.zeros((world, blocks), np.int64)
        self.epoch = 0
        self.done = 0
        self.lock = threading.Lock()
        self.data = np.zeros((2, n), np.int64)


def _wait(cond, limit=30.0):
    t0 = time.monotonic()
    while not cond():
        if time.monotonic() - t0 > limit:
            return False
        time.sleep(0)
    return True


def _run(world, blocks, launches, n, halves=2, seed=0):
    ranks = [_Rank(world, blocks, n) for _ in range(world)]
    rng = random.Random(seed)
    # rank r waits up to (r + 1) ms before its sum and 50 us before a launch, so
    # low ranks tend to run ahead of high ranks' reads
    delays = [[rng.random() * 1e-3 * (r + 1) for _ in range(launches)] for r in range(world)]
    outputs = [[None] * launches for _ in range(world)]
    timeouts = []
    per = (n + blocks - 1) // blocks

    def given(r, k):
        return np.arange(n, dtype=np.int64) * (k + 1) + 1000 * r

    def block(r, b, k, x, out):
        me = ranks[r]
        e = me.epoch + 1
        h = e % halves
        lo, hi = b * per, min(n, (b + 1) * per)
        for i in range(lo, hi):                        # copy this rank's chunk in
            me.data[h, i] = x[i]
            time.sleep(0)
        for p in range(world):                         # publish chunk b of launch e
            ranks[p].flag[r, b] = e
        for p in range(world):                         # every rank's chunk b is in
            if not _wait(lambda: ranks[r].flag[p, b] >= e):
                timeouts.append((r, b, k))
        time.sleep(delays[r][k] * rng.random())
        for i in range(lo, hi):                        # sum in rank order
            acc = 0
            for p in range(world):
                acc += int(ranks[p].data[h, i])
                time.sleep(0)
            out[i] = acc
        with me.lock:                                  # the last block records e
            prev = me.done
            me.done += 1
            if prev == blocks - 1:
                me.done = 0
                me.epoch = e

    def stream(r):
        for k in range(launches):
            x = given(r, k)                            # the launch's input
            time.sleep(delays[r][k] * 0.05)
            out = np.zeros(n, np.int64)
            threads = [threading.Thread(target=block, args=(r, b, k, x, out))
                       for b in range(blocks)]
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
    want = [sum(given(r, k) for r in range(world)) for k in range(launches)]
    correct = all(np.array_equal(outputs[r][k], want[k])
                  for r in range(world) for k in range(launches))
    return correct, timeouts


def test_protocol_gives_every_launch_its_own_sum():
    for world, blocks, seed in ((2, 3, 0), (3, 2, 1), (4, 3, 2), (2, 1, 3)):
        ok, timeouts = _run(world, blocks, launches=12, n=24, seed=seed)
        assert ok and not timeouts, (world, blocks, timeouts)


def test_protocol_with_one_data_half_is_caught():
    caught = False
    for seed in range(8):
        ok, _ = _run(2, 2, launches=12, n=24, halves=1, seed=seed)
        caught = caught or not ok
        if caught:
            break
    assert caught


# --------------------------------------------------------------------------
# The LL protocol (allreduce_ll_kernel): launch e of rank r pushes each word
# of its input, tagged with e, into slot r of half e % 2 of every peer's
# receive area, then waits for every peer's words of the same lines in its
# own area to carry tag e, and sums in rank order. No flags and no fences:
# a word is valid when it is seen with its launch's tag.

class _LLRank:
    def __init__(self, world, n, halves):
        self.area = np.zeros((halves, world, n, 2), np.int64)  # (word, tag)
        self.epoch = 0
        self.done = 0
        self.lock = threading.Lock()


def _run_ll(world, blocks, launches, n, halves=2, seed=0, limit=2.0):
    ranks = [_LLRank(world, n, halves) for _ in range(world)]
    rng = random.Random(seed)
    delays = [[rng.random() * 1e-3 * (r + 1) for _ in range(launches)] for r in range(world)]
    outputs = [[None] * launches for _ in range(world)]
    timeouts = []
    per = (n + blocks - 1) // blocks

    def given(r, k):
        return np.arange(n, dtype=np.int64) * (k + 1) + 1000 * r

    def block(r, b, k, x, out):
        me = ranks[r]
        e = me.epoch + 1
        h = e % halves
        lo, hi = b * per, min(n, (b + 1) * per)
        for i in range(lo, hi):                        # push, tagged with e
            for p in range(world):
                if p != r:
                    ranks[p].area[h, r, i] = (x[i], e)  # one atomic 64-bit store
            time.sleep(0)
        time.sleep(delays[r][k] * rng.random())
        for i in range(lo, hi):                        # gather in rank order
            acc = 0
            for p in range(world):
                if p == r:
                    acc += int(x[i])
                    continue
                cell = me.area[h, p, i]
                if not _wait(lambda: cell[1] == e, limit):
                    timeouts.append((r, b, k))
                    return
                acc += int(cell[0])
                time.sleep(0)
            out[i] = acc
        with me.lock:
            prev = me.done
            me.done += 1
            if prev == blocks - 1:
                me.done = 0
                me.epoch = e

    def stream(r):
        for k in range(launches):
            x = given(r, k)
            time.sleep(delays[r][k] * 0.05)
            out = np.zeros(n, np.int64)
            threads = [threading.Thread(target=block, args=(r, b, k, x, out)) for b in range(blocks)]
            for t in threads:
                t.start()
            for t in threads:
                t.join()
            outputs[r][k] = out

    streams = [threading.Thread(target=stream, args=(r,)) for r in range(world)]
    for t in streams:
        t.start()
    for t in streams:
        t.join()
    want = [sum(given(r, k) for r in range(world)) for k in range(launches)]
    correct = all(np.array_equal(outputs[r][k], want[k])
                  for r in range(world) for k in range(launches))
    return correct, timeouts


def test_ll_protocol_gives_every_launch_its_own_sum():
    for world, blocks, seed in ((2, 3, 0), (3, 2, 1), (4, 2, 2), (2, 1, 3)):
        ok, timeouts = _run_ll(world, blocks, launches=10, n=16, seed=seed)
        assert ok and not timeouts, (world, blocks, timeouts)


def test_ll_protocol_with_one_half_is_caught():
    # A rank that runs a launch ahead overwrites words a slow peer still
    # waits for: the peer never sees its launch's tag (or sums wrong words).
    caught = False
    for seed in range(8):
        ok, timeouts = _run_ll(2, 2, launches=10, n=16, halves=1, seed=seed, limit=0.3)
        caught = caught or not ok or bool(timeouts)
        if caught:
            break
    assert caught
