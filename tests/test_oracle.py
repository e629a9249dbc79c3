"""The CPU oracle pinned against the reference (golden fixtures), CPU only."""
from __future__ import annotations

import json

import numpy as np
import pytest
import torch

from conftest import GOLDEN, from_bits
from oracle import reference_math as R
from cases import CASES, make_case


def test_store_kvcache_matches_reference_triton_kernel():
    """Oracle scatter == the reference's Triton store_kvcache_kernel, bit for bit."""
    f = np.load(GOLDEN / "store_kvcache_triton.npz")
    N, H, KVH, d, nb, bs = (int(x) for x in f["shape"])
    qkv = f["qkv"]
    k = np.ascontiguousarray(qkv[:, H * d:(H + KVH) * d]).reshape(N, KVH, d)
    v = qkv[:, (H + KVH) * d:].reshape(N, KVH, d)  # strided view, as in the engine
    assert v.strides[0] == qkv.strides[0]
    kc = np.zeros((nb, bs, KVH, d), np.uint16)
    vc = np.zeros_like(kc)
    R.store_kvcache(k, v, kc, vc, f["slot_mapping"])
    assert np.array_equal(kc, f["k_cache"])
    assert np.array_equal(vc, f["v_cache"])
    assert (f["slot_mapping"] == -1).sum() == 2


def _states(step):
    return step["seqs"]


def test_prefill_metadata_matches_reference_model_runner():
    """Restated prepare_prefill == the reference's, on Scheduler/BlockManager states."""
    fix = json.loads((GOLDEN / "engine_metadata.json").read_text())
    bs = fix["block_size"]
    n = 0
    saw_prefix = saw_chunk = False
    for step in fix["steps"]:
        if not step["is_prefill"]:
            continue
        cu_q, cu_k, max_q, max_k, slots, tables = R.prepare_prefill_metadata(_states(step), bs)
        assert cu_q.tolist() == step["cu_seqlens_q"]
        assert cu_k.tolist() == step["cu_seqlens_k"]
        assert (max_q, max_k) == (step["max_seqlen_q"], step["max_seqlen_k"])
        assert slots.tolist() == step["slot_mapping"]
        assert (tables is None) == (step["block_tables"] is None)
        if tables is not None:
            assert tables.tolist() == step["block_tables"]
            saw_prefix = True
        saw_chunk |= any(s["start"] + s["num_scheduled"] < s["num_tokens"]
                         for s in step["seqs"])
        n += 1
    assert n >= 3 and saw_prefix and saw_chunk


def test_decode_metadata_matches_reference_model_runner():
    fix = json.loads((GOLDEN / "engine_metadata.json").read_text())
    bs = fix["block_size"]
    n = 0
    for step in fix["steps"]:
        if step["is_prefill"]:
            continue
        slots, lens, tables = R.prepare_decode_metadata(_states(step), bs)
        assert slots.tolist() == step["slot_mapping"]
        assert lens.tolist() == step["context_lens"]
        assert tables.tolist() == step["block_tables"]
        n += 1
    assert n >= 5


def _oracle_case(c):
    scale = 128 ** -0.5
    if c["kind"] == "varlen":
        bt = None if c["block_table"] is None else c["block_table"].numpy()
        return R.varlen_attention(c["q"], c["k"], c["v"], c["cu_q"].numpy(), c["cu_k"].numpy(),
                                  scale, True, bt)
    return R.decode_attention(c["q"], c["k_cache"], c["v_cache"], c["cache_seqlens"].numpy(),
                              c["block_table"].numpy(), scale)


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_flash_attn_golden(name):
    """Oracle == flash-attn (the reference's attention) run on a B200, within bf16 rounding."""
    path = GOLDEN / "flash_attn_golden.npz"
    if not path.exists():
        pytest.skip("flash-attn golden vectors not recorded")
    g = np.load(path)
    ref = from_bits(g[name]).float()
    ours = _oracle_case(make_case(name))
    assert ref.shape == ours.shape
    # flash-attn rounds its output to bf16 (and P to bf16 before P@V); the
    # fp32 oracle does neither: max-abs 1e-2 all the same.
    from helpers import assert_close
    assert_close(ref, ours, f"flash-attn golden {name} vs oracle")


def test_chain_tree_equals_paged_causal_prefill():
    """A chain-shaped tree mask is ordinary bottom-right causal prefill."""
    c = make_case("chain8")
    bt = c["block_table"].numpy()
    cu_q = c["cu_q"].numpy()
    cu_k = c["cu_k"].numpy()
    ctx = (np.diff(cu_k) - np.diff(cu_q)).astype(np.int32)
    masks = np.concatenate([np.array([(1 << (j + 1)) - 1 for j in range(int(n))], np.uint64)
                            for n in np.diff(cu_q)])
    a = R.tree_attention(c["q"], c["k"], c["v"], cu_q, ctx, masks, bt, 128 ** -0.5)
    b = R.varlen_attention(c["q"], c["k"], c["v"], cu_q, cu_k, 128 ** -0.5, True, bt)
    assert torch.allclose(a, b, atol=1e-6)


def test_decode_equals_single_query_prefill():
    c = make_case("decode")
    lens = c["cache_seqlens"].numpy()
    B = len(lens)
    cu_q = np.arange(B + 1, dtype=np.int32)
    cu_k = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    a = R.decode_attention(c["q"], c["k_cache"], c["v_cache"], lens, c["block_table"].numpy(),
                           128 ** -0.5)
    b = R.varlen_attention(c["q"], c["k_cache"], c["v_cache"], cu_q, cu_k, 128 ** -0.5, True,
                           c["block_table"].numpy())
    assert torch.allclose(a, b, atol=1e-6)


def test_causal_mask_is_bottom_right_aligned():
    m = R.causal_allowed(2, 5)
    assert m.tolist() == [[True, True, True, True, False], [True] * 5]
    # a row that sees no key produces zeros
    q = torch.randn(3, 2, 128).bfloat16()
    k = torch.randn(1, 1, 128).bfloat16()
    o = R.varlen_attention(q, k, k, [0, 3], [0, 1], 0.1, True)
    assert torch.all(o[:2] == 0) and torch.any(o[2] != 0)


def test_kv_move_reads_before_writes():
    kc = np.arange(8 * 4, dtype=np.uint16).reshape(1, 8, 1, 4)
    vc = kc + 1000
    R.kv_move(kc, vc, np.array([3, 5, 6]), np.array([2, 3, 4]), np.array([0, 3]))
    assert kc[0, 2, 0, 0] == 12 and kc[0, 3, 0, 0] == 20 and kc[0, 4, 0, 0] == 24
    assert vc[0, 3, 0, 0] == 1020


def test_qk_norm_rope_oracle_matches_reference_modules():
    """The fused q/k RMSNorm + rotary restatement against the reference's own
    RMSNorm and RotaryEmbedding modules (tests/golden/make_qk_norm_golden.py).

    The oracle fixes the order of the sum of squares (the CUDA kernel's
    butterfly); torch's CPU reduction uses another order, which may move the
    variance by one fp32 ulp and, rarely, a bf16 rounding: at most 1 ulp on
    at most 1 in 10^4 elements. The rotary cos/sin buffer is rebuilt exactly.
    """
    g = np.load(GOLDEN / "qk_norm_rope_ref.npz")
    N, H, KVH, D, max_pos = (int(x) for x in g["meta"])
    cache = R.rope_cache(D, max_pos, float(g["theta"])).numpy().reshape(-1, D)
    assert np.array_equal(cache[g["positions"]], g["cos_sin_rows"].reshape(-1, D))
    qkv = g["qkv"]
    q = qkv[:, :H * D].reshape(N, H, D)
    k = qkv[:, H * D:(H + KVH) * D].reshape(N, KVH, D)
    rows = g["cos_sin_rows"].reshape(N, 1, D)
    for x, w, ref in ((q, g["q_weight"], g["q_rot"]), (k, g["k_weight"], g["k_rot"])):
        out = R.qk_norm_rope(x, w, rows, float(g["eps"]))
        ulp = np.abs(out.astype(np.int32) - ref.astype(np.int32))
        assert ulp.max() <= 1
        assert (ulp > 0).mean() <= 1e-4


def test_qk_norm_rope_oracle_basic_properties():
    """Rotation preserves the pair norm; position 0 is the identity rotation."""
    rng = np.random.default_rng(0)
    x = R.f32_to_bf16_bits(rng.standard_normal((4, 3, 128)).astype(np.float32))
    w = R.f32_to_bf16_bits(np.ones(128, np.float32))
    cs = R.rope_cache(128, 16, 1e6).numpy().reshape(-1, 128)
    out0 = R.qk_norm_rope(x, w, cs[0][None, None, :], 1e-6)
    xf = R.bf16_bits_to_f32(x).reshape(-1, 128)
    rms = np.sqrt((xf.astype(np.float64) ** 2).mean(-1, keepdims=True))
    np.testing.assert_allclose(R.bf16_bits_to_f32(out0).reshape(-1, 128), xf / rms, rtol=1e-2)
    out5 = R.bf16_bits_to_f32(R.qk_norm_rope(x, w, cs[5][None, None, :], 1e-6)).reshape(-1, 128)
    a0 = R.bf16_bits_to_f32(out0).reshape(-1, 128)
    n0 = a0[:, :64] ** 2 + a0[:, 64:] ** 2
    n5 = out5[:, :64] ** 2 + out5[:, 64:] ** 2
    np.testing.assert_allclose(n5, n0, rtol=2e-2, atol=1e-3)


def test_philox_known_answers():
    """Philox4x32-10 against the known-answer vectors published with the
    algorithm (Random123 distribution): counter, key -> output."""
    kat = [((0, 0, 0, 0), (0, 0), (0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8)),
           ((0xffffffff,) * 4, (0xffffffff,) * 2, (0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd)),
           ((0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344), (0xa4093822, 0x299f31d0),
            (0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1))]
    for ctr, key, want in kat:
        got = R.philox4x32_10(np.array([ctr], dtype=np.uint32), key)[0]
        assert tuple(int(x) for x in got) == want


def test_sampler_law_is_the_exponential_race():
    """argmax(p / E), E ~ Exp(1) (sampler.py:11) picks i with probability p_i;
    the Gumbel form argmax(log p + G) used by the kernel is the same law."""
    g = torch.Generator().manual_seed(0)
    logits = torch.tensor([[2.0, 1.0, 0.5, -1.0, 0.0]])
    p = R.sample_probs(logits, 0.7)[0]
    n = 200000
    E = torch.empty(n, 5).exponential_(1, generator=g)
    race = (p[None, :] / E).argmax(-1)
    G = -torch.log(-torch.log(torch.rand(n, 5, generator=g).clamp_min(1e-12)))
    gum = (torch.log(p)[None, :] + G).argmax(-1)
    for picks in (race, gum):
        freq = torch.bincount(picks, minlength=5).double() / n
        assert (freq - p.double()).abs().max() < 5e-3


def test_vocab_shard_keys_merge_to_the_gathered_argmax():
    """Pick keys per vocabulary shard (embed_head.py:56-61) merged over the
    shards give the first-index argmax of the gathered row
    (embed_head.py:62-65, then argmax), with ties across shard borders, NaN,
    all -inf rows and -0 / +0."""
    g = torch.Generator().manual_seed(0)
    for trial in range(40):
        B, V = 9, int(torch.randint(1, 400, (1,), generator=g))
        x = (torch.randn(B, V, generator=g) * 2).round().bfloat16()  # many exact ties
        x[0] = float("-inf")
        x[1, ::3] = float("nan")
        if V > 2:
            x[2, :] = float("-inf")
            x[2, V // 2] = -0.0
            x[2, V - 1] = 0.0
        cuts = sorted(set([0, V] + torch.randint(0, V + 1, (3,), generator=g).tolist()))
        keys = np.stack([R.greedy_shard_keys(x[:, a:b], a) for a, b in zip(cuts[:-1], cuts[1:])])
        got = R.merge_pick_keys(keys)
        xf = x.float().clone()
        xf[torch.isnan(xf)] = float("-inf")
        want = xf.argmax(-1).numpy()
        want[(xf == float("-inf")).all(-1).numpy()] = 0
        assert np.array_equal(got, want), trial
    # key order: score first, then the lower column
    k = R.pick_keys(np.array([1.0, 1.0, 2.0, -0.0, 0.0, -np.inf, np.nan], np.float32),
                    np.array([5, 3, 9, 1, 2, 0, 0]))
    assert k[1] > k[0] and k[2] > k[1] and k[3] > k[4] and k[5] == 0 and k[6] == 0


def test_allreduce_oracle_is_the_rounded_fp32_sum():
    """Two ranks: one rounded bf16 add, as torch (and NCCL's bf16 sum) gives;
    more ranks: fp32 accumulation in rank order, rounded once."""
    g = torch.Generator().manual_seed(3)
    parts = (torch.randn(4, 5000, generator=g) * 10).bfloat16()
    parts[0, :4] = torch.tensor([-0.0, 0.0, float("inf"), 1.0])
    parts[1, :4] = torch.tensor([-0.0, -0.0, 1.0, float("nan")])
    bits = parts.view(torch.int16).numpy().view(np.uint16)
    two = R.allreduce_sum(bits[:2])
    want2 = (parts[0].float() + parts[1].float()).bfloat16().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(two[4:], want2[4:])
    assert two[0] == 0x8000 and two[1] == 0x0000 and two[2] == 0x7F80 and np.isnan(R.bf16_bits_to_f32(two[3:4]))[0]
    four = R.allreduce_sum(bits)
    acc = parts[0].float() + parts[1].float() + parts[2].float() + parts[3].float()
    assert np.array_equal(four[4:], acc.bfloat16().view(torch.int16).numpy().view(np.uint16)[4:])


def test_c_decode_restatement_matches_the_torch_oracle():
    """oracle/decode_ref.c (the timed CPU baseline) against decode_attention:
    GQA groups of 1, 2 and 8, empty sequences, permuted paged tables."""
    import sys
    sys.path.insert(0, str(GOLDEN.parents[1] / "oracle"))
    from build_oracle import build_c_oracle
    build_c_oracle()
    g = torch.Generator().manual_seed(9)
    for H, KVH, bs in ((8, 8, 16), (16, 8, 256), (64, 8, 64)):
        lens = np.array([0, 1, 37, 300, 513], np.int32)
        W = int((lens.max() + bs - 1) // bs) + 1
        nb = len(lens) * W
        perm = np.random.default_rng(H).permutation(nb).astype(np.int32)
        bt = perm.reshape(len(lens), W)
        kc = torch.randn(nb, bs, KVH, 128, generator=g).bfloat16()
        vc = torch.randn(nb, bs, KVH, 128, generator=g).bfloat16()
        q = torch.randn(len(lens), H, 128, generator=g).bfloat16()
        want = R.decode_attention(q, kc, vc, lens, bt, 128 ** -0.5)
        got = R.decode_attention_c(q, kc, vc, lens, bt, 128 ** -0.5)
        assert torch.allclose(got, want, atol=2e-5, rtol=1e-4), (H, (got - want).abs().max())
        assert got[0].abs().max() == 0
    with pytest.raises(ValueError):
        R.decode_attention_c(q, kc, vc, np.array([W * bs + 1] + [1] * 4, np.int32), bt, 1.0)
    # a block id outside the cache is refused before any read (the GPU kernel
    # flags the same table as NVATTN_STATUS_BAD_BLOCK)
    for bad in (-1, nb):
        bt_bad = bt.copy()
        bt_bad[3, 1] = bad  # used by sequence 3 (300 keys)
        with pytest.raises(ValueError):
            R.decode_attention_c(q, kc, vc, lens, bt_bad, 1.0)
    bt_unused = bt.copy()
    bt_unused[3, W - 1] = -1  # past sequence 3's keys: never read, so accepted
    R.decode_attention_c(q, kc, vc, lens, bt_unused, 128 ** -0.5)
