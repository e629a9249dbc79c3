"""Decode-step metadata, host side (CPU): the packed record and the oracle of
the decode graph's inputs, both on the reference engine's own decode steps
(tests/golden/engine_metadata.json: Scheduler + BlockManager +
ModelRunner.prepare_decode, model_runner.py:172-188)."""
from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import GOLDEN
from oracle import reference_math as R

from nvattn import decode_meta


def _decode_steps():
    fix = json.loads((GOLDEN / "engine_metadata.json").read_text())
    steps = [s for s in fix["steps"] if not s["is_prefill"]]
    assert len(steps) >= 5
    for st in steps:
        for i, s in enumerate(st["seqs"]):
            s["last_token"] = 1000 + 7 * i  # the fixture has no token ids
    return fix["block_size"], steps


def test_packed_record_holds_the_reference_block_tables():
    bs, steps = _decode_steps()
    buf = np.zeros(1 << 16, np.uint8)
    for st in steps:
        seqs = st["seqs"]
        B, W = decode_meta.pack_record(buf, [s["last_token"] for s in seqs],
                                       [s["num_tokens"] for s in seqs],
                                       [s["block_table"] for s in seqs], 512, 16)
        tok, lens, tl, flat = decode_meta.record_views(buf, B, W)
        assert flat.reshape(B, W).tolist() == st["block_tables"]
        assert lens.tolist() == st["context_lens"]
        assert tl.tolist() == [len(s["block_table"]) for s in seqs]
        assert tok.tolist() == [s["last_token"] for s in seqs]


def test_graph_inputs_oracle_matches_reference_steps():
    bs, steps = _decode_steps()
    rows, cols = 64, 16
    for st in steps:
        prev = dict(input_ids=np.full(rows, 77, np.int64), positions=np.full(rows, 78, np.int64),
                    slot_mapping=np.full(rows, 79, np.int32), context_lens=np.full(rows, 80, np.int32),
                    block_tables=np.full((rows, cols), 81, np.int32))
        out = R.decode_graph_inputs(st["seqs"], bs, rows, prev)
        B, W = len(st["seqs"]), len(st["block_tables"][0])
        assert out["slot_mapping"][:B].tolist() == st["slot_mapping"]
        assert out["context_lens"][:B].tolist() == st["context_lens"]
        assert out["block_tables"][:B, :W].tolist() == st["block_tables"]
        assert (out["positions"][:B] == np.array(st["context_lens"]) - 1).all()
        assert (out["slot_mapping"][B:] == -1).all() and (out["context_lens"][B:] == 0).all()
        # left as they were, as run_model leaves them (model_runner.py:204-210)
        assert (out["input_ids"][B:] == 77).all() and (out["positions"][B:] == 78).all()
        assert (out["block_tables"][B:] == 81).all() and (out["block_tables"][:B, W:] == 81).all()


def test_pack_record_rejects_bad_batches():
    buf = np.zeros(4096, np.uint8)
    with pytest.raises(ValueError):
        decode_meta.pack_record(buf, [], [], [], 8, 4)
    with pytest.raises(ValueError):
        decode_meta.pack_record(buf, [1], [1, 2], [[0]], 8, 4)
    with pytest.raises(ValueError, match="max_table_width"):
        decode_meta.pack_record(buf, [1], [1], [[0, 1, 2, 3, 4]], 8, 4)
    with pytest.raises(ValueError, match="max_seqs"):
        decode_meta.pack_record(buf, [1] * 9, [1] * 9, [[0]] * 9, 8, 4)


def test_decode_metadata_refuses_cpu():
    with pytest.raises(ValueError, match="CUDA"):
        decode_meta.DecodeMetadata(8, 4, 256, "cpu")
