"""Decode-step metadata on the GPU (nvattn_decode_prepare): every output,
including the graph's padding rows and the regions the reference leaves
alone, bit for bit against the oracle of ModelRunner.prepare_decode + the
graph-input copies (model_runner.py:172-188, 204-210)."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import reference_math as R

from nvattn import _lib, ops
from nvattn.decode_meta import DecodeMetadata

pytestmark = pytest.mark.gpu
dev = torch.device("cuda")


def _graph_buffers(rows, cols, seed):
    g = torch.Generator().manual_seed(seed)
    return dict(input_ids=torch.randint(-9, 9, (rows,), generator=g, dtype=torch.int64),
                positions=torch.randint(-9, 9, (rows,), generator=g, dtype=torch.int64),
                slot_mapping=torch.randint(-9, 9, (rows,), generator=g, dtype=torch.int32),
                context_lens=torch.randint(-9, 9, (rows,), generator=g, dtype=torch.int32),
                block_tables=torch.randint(-9, 9, (rows, cols), generator=g, dtype=torch.int32))


def _run_and_check(meta, seqs, bs, rows, cols, seed):
    prev = _graph_buffers(rows, cols, seed)
    bufs = {k: v.to(dev) for k, v in prev.items()}
    meta.pack_lists([s["last_token"] for s in seqs], [s["num_tokens"] for s in seqs],
                    [s["block_table"] for s in seqs])
    meta.launch(rows, **bufs)
    torch.cuda.synchronize()
    want = R.decode_graph_inputs(seqs, bs, rows, {k: v.numpy() for k, v in prev.items()})
    for k, v in bufs.items():
        assert np.array_equal(v.cpu().numpy(), want[k]), k
    return bufs


def test_reference_engine_steps_bit_exact():
    fix = json.loads((GOLDEN / "engine_metadata.json").read_text())
    bs = fix["block_size"]
    meta = DecodeMetadata(512, 16, bs, dev)
    n = 0
    for st in fix["steps"]:
        if st["is_prefill"]:
            continue
        seqs = st["seqs"]
        for i, s in enumerate(seqs):
            s["last_token"] = 151000 + i
        bufs = _run_and_check(meta, seqs, bs, 512, 16, n)
        B = len(seqs)
        assert bufs["slot_mapping"][:B].tolist() == st["slot_mapping"]
        assert bufs["context_lens"][:B].tolist() == st["context_lens"]
        n += 1
    assert n >= 5 and ops.read_status() == 0


@pytest.mark.parametrize("B,max_w,bs,rows", [(512, 160, 256, 512), (1, 1, 256, 1),
                                             (300, 16, 256, 512), (77, 40, 16, 96)])
def test_random_batches_bit_exact(B, max_w, bs, rows):
    rng = np.random.default_rng(B * 31 + bs)
    nb_total = B * max_w + 5
    perm = rng.permutation(nb_total)
    seqs, pos = [], 0
    for i in range(B):
        n = int(rng.integers(1, max_w * bs + 1))
        nblk = (n + bs - 1) // bs
        seqs.append(dict(last_token=int(rng.integers(0, 151936)), num_tokens=n,
                         block_table=perm[pos:pos + nblk].tolist()))
        pos += nblk
    meta = DecodeMetadata(max(B, 8), max_w, bs, dev)
    _run_and_check(meta, seqs, bs, rows, max_w + 3, B)
    assert ops.read_status() == 0
    # the same object again, with a new batch of the same shape (buffer reuse)
    for s in seqs:
        s["num_tokens"] = min(s["num_tokens"] + 1, len(s["block_table"]) * bs)
    _run_and_check(meta, seqs, bs, rows, max_w + 3, B + 1)


def test_records_without_a_slot_are_flagged_and_skipped():
    meta = DecodeMetadata(8, 4, 256, dev)
    ops.read_status()
    # a table too short for its length, and a negative block id
    meta.pack_lists([1, 2, 3], [600, 10, 5], [[4, 5], [-3], [9]])
    slots = torch.full((4,), 99, dtype=torch.int32, device=dev)
    lens = torch.full((4,), 99, dtype=torch.int32, device=dev)
    meta.launch(4, slot_mapping=slots, context_lens=lens)
    assert slots.tolist() == [-1, -1, 9 * 256 + 4, -1]
    assert lens.tolist() == [600, 10, 5, 0]
    assert ops.read_status() & _lib.STATUS_BAD_SLOT
