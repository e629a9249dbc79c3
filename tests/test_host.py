"""Host-side checks that need no GPU: the C ABI library, argument validation,
tree bookkeeping and head sharding."""
from __future__ import annotations

import ctypes
import re

import numpy as np
import pytest
import torch

from conftest import REPO

import nvattn
from nvattn import _lib, ops, parallel, tree


def _header_symbols():
    text = (REPO / "include" / "nvattn.h").read_text()
    return sorted(set(re.findall(r"NVATTN_API\s+[\w\s\*]+?\b(nvattn_\w+)\s*\(", text)))


def test_library_exports_every_header_symbol():
    lib = _lib.load()
    names = _header_symbols()
    assert len(names) >= 8
    for n in names:
        assert hasattr(lib, n), n
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature"
    assert _lib.version()[0] == 1


def test_c_abi_rejects_bad_arguments_before_any_launch():
    lib = _lib.load()
    # NULL pointers with work to do -> NVATTN_ERR_INVALID, message set
    rc = lib.nvattn_store_kvcache(None, 128, None, 128, None, None, None, 4, 128, 256, None, None)
    assert rc == _lib.ERR_INVALID
    assert b"NULL" in lib.nvattn_last_error()
    # nothing to do -> OK without touching the device
    assert lib.nvattn_store_kvcache(None, 0, None, 0, None, None, None, 0, 128, 0, None,
                                    None) == _lib.OK
    # unsupported head_dim / group sizes
    fake = ctypes.c_void_p(0x1000)
    rc = lib.nvattn_paged_decode(fake, 256, 64, fake, fake, fake, 256, 64, fake, fake, 4, 4,
                                 8, 256, 2, 4, 2, 64, ctypes.c_float(0.1), None, 0, None, None)
    assert rc == _lib.ERR_UNSUPPORTED and b"head_dim" in lib.nvattn_last_error()
    rc = lib.nvattn_paged_decode(fake, 256, 128, fake, fake, fake, 256, 128, fake, fake, 4, 4,
                                 8, 256, 2, 64, 2, 128, ctypes.c_float(0.1), None, 0, None, None)
    assert rc == _lib.ERR_UNSUPPORTED and b"16 query heads" in lib.nvattn_last_error()
    rc = lib.nvattn_paged_decode(fake, 256, 128, fake, fake, fake, 256, 128, fake, fake, 4, 4,
                                 8, 100, 2, 4, 2, 128, ctypes.c_float(0.1), None, 0, None, None)
    assert rc == _lib.ERR_UNSUPPORTED and b"block_size" in lib.nvattn_last_error()
    rc = lib.nvattn_tree_verify(fake, 256, 128, fake, fake, fake, 256, 128, fake, fake, fake,
                                fake, 4, 4, 8, 256, 1, 65, 65, 4, 1, 128, ctypes.c_float(0.1),
                                None, 0, None, None)
    assert rc == _lib.ERR_UNSUPPORTED and b"64 tree nodes" in lib.nvattn_last_error()
    rc = lib.nvattn_kv_move(None, None, None, None, None, 2, 4, 256, 100, None, None)
    assert rc == _lib.ERR_INVALID
    # fused q/k norm + rotary + scatter: head_dim, alignment, NULL pointers, empty batch
    rc = lib.nvattn_qk_norm_rope_store(fake, 2048, fake, 2048, fake, 2048, fake, fake, fake, 64,
                                       fake, None, fake, None, None, None, 0, 4, 16, 8, 64,
                                       ctypes.c_float(1e-6), None, None)
    assert rc == _lib.ERR_UNSUPPORTED and b"head_dim" in lib.nvattn_last_error()
    rc = lib.nvattn_qk_norm_rope_store(ctypes.c_void_p(0x1008), 4096, fake, 4096, fake, 4096, fake,
                                       fake, fake, 64, fake, None, fake, None, None, None, 0, 4,
                                       16, 8, 128, ctypes.c_float(1e-6), None, None)
    assert rc == _lib.ERR_UNSUPPORTED and b"16-byte" in lib.nvattn_last_error()
    rc = lib.nvattn_qk_norm_rope_store(fake, 4096, None, 4096, fake, 4096, fake, fake, fake, 64,
                                       fake, None, fake, None, None, None, 0, 4, 16, 8, 128,
                                       ctypes.c_float(1e-6), None, None)
    assert rc == _lib.ERR_INVALID and b"NULL" in lib.nvattn_last_error()
    rc = lib.nvattn_qk_norm_rope_store(fake, 4096, fake, 4096, fake, 4096, fake, fake, fake, 64,
                                       fake, fake, fake, None, None, None, 10, 4, 16, 8, 128,
                                       ctypes.c_float(1e-6), None, None)
    assert rc == _lib.ERR_INVALID and b"slot_mapping without caches" in lib.nvattn_last_error()
    assert lib.nvattn_qk_norm_rope_store(None, 4096, None, 4096, None, 4096, None, None, None, 64,
                                         None, None, None, None, None, None, 0, 0, 16, 8, 128,
                                         ctypes.c_float(1e-6), None, None) == _lib.OK
    # sampler: sizes, strides, NULL pointers, empty batch
    assert lib.nvattn_sample(fake, 100, 4, 0, None, 1, 0, fake, None) == _lib.ERR_INVALID
    assert lib.nvattn_sample(fake, 50, 4, 100, None, 1, 0, fake, None) == _lib.ERR_INVALID
    assert lib.nvattn_sample(None, 100, 4, 100, None, 1, 0, fake, None) == _lib.ERR_INVALID
    assert lib.nvattn_sample(None, 100, 0, 100, None, 1, 0, None, None) == _lib.OK
    # vocabulary-shard sampler and merge
    assert lib.nvattn_sample_shard(fake, 100, 4, 100, -4, None, 1, 0, fake, None) == _lib.ERR_INVALID
    assert lib.nvattn_sample_shard(fake, 100, 4, 100, 2 ** 32 - 50, None, 1, 0, fake,
                                   None) == _lib.ERR_INVALID
    assert b"columns" in lib.nvattn_last_error()
    assert lib.nvattn_sample_shard(fake, 50, 4, 100, 0, None, 1, 0, fake, None) == _lib.ERR_INVALID
    assert lib.nvattn_sample_shard(None, 100, 4, 100, 0, None, 1, 0, fake, None) == _lib.ERR_INVALID
    assert lib.nvattn_sample_shard(None, 100, 0, 100, 8, None, 1, 0, None, None) == _lib.OK
    assert lib.nvattn_sample_merge(fake, 0, 4, fake, None) == _lib.ERR_INVALID
    assert lib.nvattn_sample_merge(None, 2, 4, fake, None) == _lib.ERR_INVALID
    assert lib.nvattn_sample_merge(fake, 2, 4, fake, None) == _lib.ERR_INVALID
    assert b"in place" in lib.nvattn_last_error()
    assert lib.nvattn_sample_merge(None, 2, 0, None, None) == _lib.OK
    # one-shot all-reduce: argument checks before any launch
    import ctypes as C
    bufs = (C.c_uint64 * 2)(0x10000, 0x20000)
    # header + two halves + two LL receive areas of 8 slots (a 16-byte line per 4 elements)
    assert lib.nvattn_ar_buffer_bytes(1000) == 4096 + 2 * 2000 + 2 * 8 * 250 * 16
    x = C.c_void_p(0x40000)
    assert lib.nvattn_allreduce(C.addressof(bufs), 0, 0, 8, 8, x, fake, None, None) == _lib.ERR_INVALID
    assert lib.nvattn_allreduce(C.addressof(bufs), 2, 2, 8, 8, x, fake, None, None) == _lib.ERR_INVALID
    assert lib.nvattn_allreduce(C.addressof(bufs), 0, 9, 8, 8, x, fake, None, None) == _lib.ERR_INVALID
    assert lib.nvattn_allreduce(C.addressof(bufs), 0, 2, 9, 8, x, fake, None, None) == _lib.ERR_INVALID
    assert lib.nvattn_allreduce(C.addressof(bufs), 0, 2, 8, 8, None, fake, None,
                                None) == _lib.ERR_INVALID            # no input
    bad = (C.c_uint64 * 2)(0x10000, 0x20008)
    assert lib.nvattn_allreduce(C.addressof(bad), 0, 2, 8, 8, x, fake, None, None) == _lib.ERR_INVALID
    assert lib.nvattn_allreduce(C.addressof(bufs), 0, 2, 8, 8, x, C.c_void_p(0x10000 + 4096), None,
                                None) == _lib.ERR_INVALID            # out inside the shared buffer
    assert b"overlaps" in lib.nvattn_last_error()
    assert lib.nvattn_allreduce(C.addressof(bufs), 0, 2, 8, 8, C.c_void_p(0x10000 + 4096 + 16), fake,
                                None, None) == _lib.ERR_INVALID      # in inside the shared buffer
    assert lib.nvattn_allreduce(C.addressof(bufs), 0, 2, 8, 8, C.c_void_p(0x40008), fake, None,
                                None) == _lib.ERR_INVALID            # misaligned input
    prev = lib.nvattn_ar_set_wait_limit(1000)
    assert prev == 2_000_000_000 and lib.nvattn_ar_set_wait_limit(0) == 1000
    assert lib.nvattn_ar_set_wait_limit(0) == 2_000_000_000         # 0 restored the default
    # protocol choice: pushed words while (world - 1) * 4 * n <= 4 MiB and n <= 262144
    assert lib.nvattn_ar_protocol(2, 256 * 1024, 1 << 20) == 1
    assert lib.nvattn_ar_protocol(2, 256 * 1024 + 1, 1 << 20) == 0
    assert lib.nvattn_ar_protocol(4, 256 * 1024, 1 << 20) == 1
    assert lib.nvattn_ar_protocol(8, 149796, 1 << 20) == 1 and lib.nvattn_ar_protocol(8, 149797, 1 << 20) == 0
    assert lib.nvattn_ar_protocol(4, 1000, 999) == -1 and lib.nvattn_ar_protocol(9, 8, 8) == -1
    assert lib.nvattn_ar_alloc(10, None, None) == _lib.ERR_INVALID
    assert lib.nvattn_ar_open(None, None) == _lib.ERR_INVALID
    assert lib.nvattn_ar_close(None) == _lib.OK and lib.nvattn_ar_free(None) == _lib.OK
    # decode-step metadata
    assert lib.nvattn_decode_prepare_bytes(256, 16) == 256 * (16 + 64)
    assert lib.nvattn_decode_prepare_bytes(-1, 16) == 0
    assert lib.nvattn_decode_prepare(None, fake, 4, 2, 256, 3, None, None, None, None, None, 0,
                                     None, None) == _lib.ERR_INVALID       # pad_rows < seqs
    assert lib.nvattn_decode_prepare(None, fake, 4, 0, 256, 4, None, None, None, None, None, 0,
                                     None, None) == _lib.ERR_INVALID       # no block table
    assert lib.nvattn_decode_prepare(None, fake, 4, 2, 0, 4, None, None, None, None, None, 0,
                                     None, None) == _lib.ERR_INVALID       # block_size 0
    assert lib.nvattn_decode_prepare(None, fake, 4, 8, 256, 4, None, None, None, None, fake, 4,
                                     None, None) == _lib.ERR_INVALID       # table stride < width
    assert lib.nvattn_decode_prepare(None, None, 4, 2, 256, 4, None, None, None, None, None, 0,
                                     None, None) == _lib.ERR_INVALID       # no packed record
    assert lib.nvattn_decode_prepare(None, ctypes.c_void_p(0x1004), 4, 2, 256, 4, None, None, None,
                                     None, None, 0, None, None) == _lib.ERR_INVALID  # misaligned
    assert lib.nvattn_decode_prepare(None, None, 0, 0, 256, 0, None, None, None, None, None, 0,
                                     None, None) == _lib.OK


def test_noalloc_decode_checks_arguments_before_its_scratch_size():
    """A bad call gets the error nvattn_paged_decode would give, not the
    scratch-size error, even when the batch would also overflow the scratch."""
    lib = _lib.load()
    fake = ctypes.c_void_p(0x1000)

    def noalloc(num_heads, num_kv_heads, block_size, head_dim=128, batch=128, width=128):
        return lib.nvattn_paged_decode_noalloc(fake, 8192, 128, fake, fake, fake, 8192, 128, fake,
                                               fake, width, width, 4096, block_size, batch,
                                               num_heads, num_kv_heads, head_dim,
                                               ctypes.c_float(0.1), None, None)

    assert noalloc(64, 2, 256) == _lib.ERR_UNSUPPORTED  # 32 query heads per KV head
    assert b"16 query heads" in lib.nvattn_last_error()
    assert noalloc(60, 8, 256) == _lib.ERR_INVALID  # heads not a multiple of KV heads
    assert b"multiple of num_kv_heads" in lib.nvattn_last_error()
    assert noalloc(64, 8, 100) == _lib.ERR_UNSUPPORTED
    assert b"block_size" in lib.nvattn_last_error()
    assert noalloc(64, 8, 256, head_dim=64) == _lib.ERR_UNSUPPORTED
    assert b"head_dim" in lib.nvattn_last_error()
    assert noalloc(64, 8, 256, batch=-1) == _lib.ERR_INVALID
    assert lib.nvattn_paged_decode_noalloc(None, 0, 0, None, None, None, 0, 0, None, None, 0, 0,
                                           0, 256, 0, 64, 8, 128, ctypes.c_float(0.1), None,
                                           None) == _lib.OK  # empty batch: nothing to do


def test_python_wrapper_raises_through_error_path():
    with pytest.raises(_lib.NvattnError) as ei:
        _lib.call("nvattn_kv_move", None, None, None, None, None, 1, 2, 256, 10, None, None)
    assert ei.value.code == _lib.ERR_INVALID


def test_ops_refuse_cpu_tensors_no_fallback():
    k = torch.zeros(2, 1, 128, dtype=torch.bfloat16)
    kc = torch.zeros(1, 256, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.store_kvcache(k, k, kc, kc, torch.zeros(2, dtype=torch.int32))
    q = torch.zeros(2, 4, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.paged_decode(q, kc, kc, torch.ones(2, dtype=torch.int32),
                         torch.zeros(2, 1, dtype=torch.int32))
    w = torch.ones(128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        ops.qk_norm_rope_store(torch.zeros(2, dtype=torch.int64), q, k, k, w, w,
                               torch.zeros(8, 1, 128), 1e-6)
    with pytest.raises(ValueError, match="CUDA"):
        ops.sample(torch.zeros(2, 10, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="CUDA"):
        ops.sample_shard(torch.zeros(2, 10, dtype=torch.bfloat16), 0, seed=1, offset=0)
    with pytest.raises(ValueError, match="CUDA"):
        ops.sample_merge(torch.zeros(2, 4, dtype=torch.int64))


def test_store_kvcache_keeps_reference_assertions():
    # reference asserts (attention.py:36-39) fire before the device check
    k = torch.zeros(4, 2, 128, dtype=torch.bfloat16)
    kc = torch.zeros(1, 256, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        ops.store_kvcache(k, k, kc, kc, torch.zeros(3, dtype=torch.int32))
    with pytest.raises(AssertionError):
        ops.store_kvcache(k.transpose(0, 1).contiguous().transpose(0, 1), k, kc, kc,
                          torch.zeros(4, dtype=torch.int32))


def test_decode_workspace_size_is_deterministic():
    a = ops.decode_workspace_bytes(128, 64, 8, 128, 256)
    b = ops.decode_workspace_bytes(128, 64, 8, 128, 256)
    assert a == b and a > 0
    # one short sequence batch needs no split-K partials beyond one split
    assert ops.decode_workspace_bytes(1, 8, 8, 1, 256) >= 0


def test_draft_tree_shape_and_masks():
    parents, depths = tree.build_draft_tree((4, 3, 2, 1, 1, 1), 64)
    assert len(parents) == 64 and parents[0] == -1
    assert depths.max() == 6
    assert all(parents[j] < j for j in range(1, 64))
    # per-level fan-out never exceeds the branching factor
    for j in range(64):
        kids = int((parents == j).sum())
        assert kids <= (4, 3, 2, 1, 1, 1, 0)[depths[j]]
    m = tree.ancestor_masks(parents)
    for j in range(64):
        bits = [i for i in range(64) if (int(m[j]) >> i) & 1]
        chain, x = [], j
        while x >= 0:
            chain.append(x)
            x = int(parents[x])
        assert sorted(chain) == bits
    assert tree.chain_masks(3).tolist() == [1, 3, 7]


def test_greedy_accept_and_compaction_moves():
    parents, _ = tree.build_draft_tree((2, 2), 7)
    tokens = np.array([0, 10, 11, 20, 21, 22, 23])
    # root predicts 11 -> node 2; node 2 predicts 23 -> its child with token 23
    argmax = np.array([11, 0, 23, 0, 0, 0, 0])
    path = tree.greedy_accept(parents, tokens, argmax)
    assert path[0] == 0 and tokens[path[1]] == 11 and tokens[path[2]] == 23
    src, dst = tree.compaction_moves(300, path, [7, 3], 256)
    assert dst[0] == 3 * 256 + (301 - 256)
    assert len(src) == len(dst) == 2


def test_ngram_draft():
    toks = [5, 6, 7, 8, 1, 2, 5, 6, 7]
    assert tree.ngram_draft(toks, 3) == [8, 1, 2]
    assert tree.ngram_draft([1, 2, 3], 4) == []


def test_head_shard_matches_engine_split():
    assert parallel.head_shard(64, 8, 7, 8) == ((56, 64), (7, 8))
    assert parallel.head_shard(16, 8, 1, 2) == ((8, 16), (4, 8))
    with pytest.raises(ValueError):
        parallel.head_shard(16, 8, 0, 3)
    assert parallel.vocab_shard(151936, 1, 2) == (75968, 151936)
    assert parallel.vocab_shard(151936, 7, 8) == (132944, 151936)
    with pytest.raises(ValueError):
        parallel.vocab_shard(151937, 0, 2)


def test_package_surface():
    for name in ("Attention", "store_kvcache", "flash_attn_varlen_func",
                 "flash_attn_with_kvcache", "tree_attention", "kv_move", "qk_norm_rope_store",
                 "sample", "sample_shard", "sample_merge", "DecodeMetadata", "install"):
        assert hasattr(nvattn, name)
    a = nvattn.Attention(16, 128, 128 ** -0.5, 8)
    assert a.k_cache.numel() == 0 and hasattr(a, "v_cache")


def test_e2e_compare_finds_first_divergence_and_reference_margin(tmp_path):
    """nvattn.e2e.compare on two hand-made --out files."""
    from nvattn.e2e import compare
    ref = {"r0": np.array([5, 6, 7], np.int32), "r1": np.array([1, 2, 3, 4], np.int32),
           # top1, top2, id1, id2 per generated token (bf16 values)
           "m0": np.array([[2.0, 1.0, 5, 9], [3.0, 2.0, 6, 9], [1.0, 0.5, 7, 9]], np.float32),
           "m1": np.array([[4.0, 1.0, 1, 0], [4.0, 1.0, 2, 0], [2.0, 1.984375, 3, 8],
                           [4.0, 1.0, 4, 0]], np.float32)}
    ours = {"r0": ref["r0"].copy(), "r1": np.array([1, 2, 8, 0], np.int32)}
    np.savez(tmp_path / "a.npz", **ref)
    np.savez(tmp_path / "b.npz", **ours)
    res = compare(str(tmp_path / "a.npz"), str(tmp_path / "b.npz"), k_ulps=4)
    assert res["identical"] == 1 and res["diverged"] == 1
    row = res["rows"][1]
    assert row["first_divergence"] == 2 and row["ref_top2_ids"] == [3, 8]
    assert row["ours_token"] == 8
    # 2.0 - 1.984375 = 2^-6 = 1 ulp of 2.0 in bf16 (8 significant bits)
    assert row["ref_margin_ulps"] == 1.0
    assert res["diverged_within_k"] == 1


def test_split_policies_from_host_sizes():
    """The split choices of decode and tree verification depend only on host
    sizes (a captured graph keeps its grid); their workspace sizes expose them.
    Without a GPU the SM count reads as 148 (B200). A partial slot is 128 fp32
    of O plus a (max, sum) pair: 520 bytes."""
    lib = _lib.load()
    slot = 128 * 4 + 8

    def dec(B, H, KVH, W, BS=256):
        return lib.nvattn_decode_workspace_bytes(B, H, KVH, W, BS)

    # configs[3] at TP1: 128 x 8 pairs fill >= 8 CTAs per SM with 64-tile
    # (4096-key) splits of the 512-tile table: 8 splits
    assert dec(128, 64, 8, 128) == 128 * 64 * 8 * slot
    # one KV head per GPU (TP8): 128 pairs need 32-tile splits: 16 of them
    assert dec(128, 8, 1, 128) == 128 * 8 * 16 * slot
    # the e2e batch of 256 over a 16-block table: one split covers it, no merge
    assert dec(256, 16, 8, 16) == 0
    # batch 16: the smallest split (4 tiles), 8 per pair over an 8-block table
    assert dec(16, 16, 8, 8) == 16 * 16 * 8 * slot

    def tree(S, N, H, KVH, W, BS=256):
        return lib.nvattn_tree_workspace_bytes(S, N, S * N, H, KVH, W, BS)

    order = 256  # 32 int32 sequence indices, 256-byte aligned
    # 256 (sequence, KV head) items >= 148 SMs: no split, order only
    assert tree(32, 64, 32, 8, 33) == order
    # TP2 shard: 128 items -> 2 splits; TP8 shard: 32 items -> 5, doubled under a
    # quarter of the SMs, capped at 66 tiles / 8 = 8 splits
    assert tree(32, 64, 16, 4, 33) == order + 32 * 64 * 16 * 2 * slot
    assert tree(32, 64, 4, 1, 33) == order + 32 * 64 * 4 * 8 * slot


def test_row_parallel_forward_routing():
    """row_parallel_forward keeps the caller's NCCL path (returns None) before any
    GPU work when the message exceeds the buffer, or, with pushed_only, when
    it would not take the pushed-word protocol."""
    from nvattn.allreduce import row_parallel_forward

    class FakeAR:
        capacity = 4096

        def __init__(self, pushed):
            self.pushed = pushed
            self.calls = 0

        def pushes_words(self, numel):
            return self.pushed

        def all_reduce(self, y):
            self.calls += 1
            return y

    x = torch.randn(8, 64)
    w = torch.randn(1024, 64)             # 8 x 1024 = 8192 elements > capacity
    ar = FakeAR(True)
    assert row_parallel_forward(ar, x, w, None, 0) is None and ar.calls == 0
    x = torch.randn(2, 64)                # 2048 elements
    ar = FakeAR(False)
    assert row_parallel_forward(ar, x, w, None, 0, pushed_only=True) is None and ar.calls == 0
    y = row_parallel_forward(ar, x, w, None, 0)            # published halves are fine here
    assert ar.calls == 1 and torch.equal(y, torch.nn.functional.linear(x, w))
    ar = FakeAR(True)
    b = torch.randn(1024)
    y1 = row_parallel_forward(ar, x, w, b, 1, pushed_only=True)   # bias only on rank 0
    assert ar.calls == 1 and torch.equal(y1, torch.nn.functional.linear(x, w))
    y0 = row_parallel_forward(ar, x, w, b, 0, pushed_only=True)
    assert torch.equal(y0, torch.nn.functional.linear(x, w, b))


def test_e2e_allreduce_default():
    from nvattn.e2e import peer_memory_allreduce as pm
    assert pm("nvattn-fused", 2, None) and pm("nvattn-fused", 8, None)
    assert not pm("nvattn-fused", 2, False) and pm("nvattn-fused", 4, True)
    assert not pm("nvattn-fused", 1, None) and not pm("nvattn-fused", 1, True)
    assert not pm("nvattn", 2, None) and not pm("reference", 2, True)
