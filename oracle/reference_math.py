"""CPU oracle for the attention path — TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline arm may
import this module, and only as the checker (or as the timed CPU baseline).
The product path (nvattn) never calls it.

It restates, on the CPU, what the reference computes on the path that nvattn
replaces (nanovllm/layers/attention.py):

* ``store_kvcache``       — the Triton scatter store_kvcache_kernel
  (attention.py:10-30) and its wrapper's contract (attention.py:33-40);
  numpy index copy, bit-exact.
* ``varlen_attention``    — flash_attn_varlen_func as called at
  attention.py:67-70. flash-attn is a third-party dependency (unpinned in the
  reference's pyproject.toml:18; 2.8.3 in this image). Its published
  semantics are restated: softmax(scale * Q K^T + mask) V per sequence of
  the varlen batch, causal mask aligned to the bottom-right corner (query i
  of a sequence sees keys j <= seqlen_k - seqlen_q + i), GQA head map
  h -> h // (H / KVH), rows with no visible key output 0, and in paged mode
  (block_table given, attention.py:65-66) key j of sequence b is row
  j % block_size of block block_table[b, j // block_size].
* ``decode_attention``    — flash_attn_with_kvcache at attention.py:72-74:
  one query per sequence over cache_seqlens[b] cached keys (causal is moot
  for a single query); cache_seqlens == 0 gives 0. ``decode_attention_c`` is
  the same function restated in C with OpenMP (oracle/decode_ref.c), the
  timed CPU baseline.
* ``tree_attention``      — no reference code: the ancestor-mask definition
  (a node sees the whole committed context plus the tree nodes whose bits
  are set in its mask word).
* ``kv_move``             — grouped in-cache moves, read-all-then-write.
* ``qk_norm_rope``        — the producer side of the path, Qwen3Attention's
  q_norm/k_norm (RMSNorm, nanovllm/layers/layernorm.py:16-26) followed by
  rotary_emb (nanovllm/layers/rotary_embedding.py:6-14,37-48), in numpy
  float32 with every operation rounded and the reduction in the fixed order
  the CUDA kernel uses; ``rope_cache`` rebuilds the rotary module's fp32
  cos/sin buffer (rotary_embedding.py:25-33).
* ``sample_probs`` / ``greedy_tokens`` — the sampler (nanovllm/layers/
  sampler.py:5-12): its sampling law softmax(logits / T) (the exponential
  race picks token i with exactly that probability) and argmax for greedy
  decoding; ``philox4x32_10`` / ``sample_uniforms`` restate the counter-based
  generator the CUDA sampler draws its noise from (Salmon et al., SC 2011).
* ``pick_keys`` / ``greedy_shard_keys`` / ``merge_pick_keys`` — sampling over
  vocabulary shards (embed_head.py:17-23, 56-66): per-shard pick keys whose
  maximum over the shards is the pick on the gathered row.
* ``allreduce_sum`` — the sum of RowParallelLinear's partials over ranks
  (dist.all_reduce at linear.py:155) in a fixed order.
* ``prepare_decode_metadata`` / ``decode_graph_inputs`` — ModelRunner's
  decode metadata (model_runner.py:172-188) and what the decode graph's
  inputs hold after run_model's copies (model_runner.py:204-210).

All attention math is float32 on torch CPU tensors (inputs are bf16); the
result is float32 so tests can state their tolerance against it.
"""
from __future__ import annotations

import numpy as np
import torch


# ---------------------------------------------------------------- KV scatter

def store_kvcache(key: np.ndarray, value: np.ndarray, k_cache: np.ndarray,
                  v_cache: np.ndarray, slot_mapping: np.ndarray) -> None:
    """In place: k_cache.reshape(-1, D)[slot] = key.reshape(N, D)[i] for slot != -1.

    Follows store_kvcache_kernel (nanovllm/layers/attention.py:20-30): token i
    reads D contiguous elements at i*key_stride (numpy strides carry that) and
    writes them at slot*D; slot == -1 skips the token (attention.py:23).
    Arrays are raw 16-bit patterns (np.uint16) so the copy is bit-exact.
    """
    n = key.shape[0]
    D = int(np.prod(key.shape[1:]))
    kc = k_cache.reshape(-1, D)
    vc = v_cache.reshape(-1, D)
    slots = np.asarray(slot_mapping).astype(np.int64)
    assert slots.shape == (n,)
    keep = slots != -1
    kc[slots[keep]] = key.reshape(n, D)[keep]
    vc[slots[keep]] = value.reshape(n, D)[keep]


def kv_move(k_cache: np.ndarray, v_cache: np.ndarray, src: np.ndarray, dst: np.ndarray,
            cu_moves: np.ndarray) -> None:
    """Grouped moves: every source row of a group is read before any write."""
    D = k_cache.shape[-2] * k_cache.shape[-1]
    kc = k_cache.reshape(-1, D)
    vc = v_cache.reshape(-1, D)
    for g in range(len(cu_moves) - 1):
        a, b = int(cu_moves[g]), int(cu_moves[g + 1])
        s = np.asarray(src[a:b], dtype=np.int64)
        d = np.asarray(dst[a:b], dtype=np.int64)
        krows, vrows = kc[s].copy(), vc[s].copy()
        kc[d] = krows
        vc[d] = vrows


# ----------------------------------------------------------------- attention

def gather_paged(cache: torch.Tensor, block_row, n: int) -> torch.Tensor:
    """Keys 0..n-1 of one sequence from a (num_blocks, block_size, KVH, d) cache."""
    bs = cache.shape[1]
    nblk = (n + bs - 1) // bs
    blocks = torch.as_tensor(np.asarray(block_row[:nblk], dtype=np.int64))
    return cache[blocks].reshape(nblk * bs, *cache.shape[2:])[:n]


def _attend(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
            allowed: torch.Tensor | None) -> torch.Tensor:
    """q (Lq, H, d), k/v (Lk, KVH, d), allowed (Lq, Lk) bool or None -> (Lq, H, d) fp32."""
    Lq, H, d = q.shape
    Lk, KVH, _ = k.shape
    group = H // KVH
    qf = q.float().reshape(Lq, KVH, group, d).permute(1, 2, 0, 3)  # (KVH, g, Lq, d)
    kf = k.float().permute(1, 0, 2)                                # (KVH, Lk, d)
    vf = v.float().permute(1, 0, 2)
    s = torch.einsum("hgqd,hkd->hgqk", qf, kf) * scale
    if allowed is not None:
        s = s.masked_fill(~allowed.view(1, 1, Lq, Lk), float("-inf"))
    p = torch.softmax(s, dim=-1)
    p = torch.nan_to_num(p, nan=0.0)  # rows with no visible key -> 0
    o = torch.einsum("hgqk,hkd->hgqd", p, vf)                      # (KVH, g, Lq, d)
    return o.permute(2, 0, 1, 3).reshape(Lq, H, d)


def causal_allowed(Lq: int, Lk: int) -> torch.Tensor:
    """Bottom-right aligned causal mask: query i sees keys j <= Lk - Lq + i."""
    i = torch.arange(Lq).view(-1, 1)
    j = torch.arange(Lk).view(1, -1)
    return j <= (Lk - Lq) + i


def varlen_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                     cu_seqlens_q, cu_seqlens_k, scale: float, causal: bool = True,
                     block_table=None) -> torch.Tensor:
    """flash_attn_varlen_func semantics (attention.py:67-70); returns fp32 (total_q, H, d)."""
    cu_q = np.asarray(cu_seqlens_q, dtype=np.int64)
    cu_k = np.asarray(cu_seqlens_k, dtype=np.int64)
    out = torch.zeros(q.shape, dtype=torch.float32)
    for b in range(len(cu_q) - 1):
        qs, qe = int(cu_q[b]), int(cu_q[b + 1])
        Lq = qe - qs
        Lk = int(cu_k[b + 1] - cu_k[b])
        if Lq == 0:
            continue
        if block_table is not None:
            kb = gather_paged(k, block_table[b], Lk)
            vb = gather_paged(v, block_table[b], Lk)
        else:
            kb = k[int(cu_k[b]):int(cu_k[b + 1])]
            vb = v[int(cu_k[b]):int(cu_k[b + 1])]
        allowed = causal_allowed(Lq, Lk) if causal else None
        out[qs:qe] = _attend(q[qs:qe], kb, vb, scale, allowed)
    return out


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     cache_seqlens, block_table, scale: float) -> torch.Tensor:
    """flash_attn_with_kvcache for one query per sequence (attention.py:72-74).

    q (B, H, d) -> fp32 (B, H, d).
    """
    lens = np.asarray(cache_seqlens, dtype=np.int64)
    out = torch.zeros(q.shape, dtype=torch.float32)
    for b in range(q.shape[0]):
        n = int(lens[b])
        if n == 0:
            continue
        kb = gather_paged(k_cache, block_table[b], n)
        vb = gather_paged(v_cache, block_table[b], n)
        out[b:b + 1] = _attend(q[b:b + 1], kb, vb, scale, None)
    return out


_C_DECODE = None


def decode_attention_c(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                       cache_seqlens, block_table, scale: float,
                       threads: int | None = None) -> torch.Tensor:
    """decode_attention through the C restatement (oracle/decode_ref.c, OpenMP
    over (sequence, KV head) pairs): the same function, for the timed CPU
    baseline. Needs oracle/liboracle_decode.so (oracle/build_oracle.py)."""
    global _C_DECODE
    import ctypes
    import os
    from pathlib import Path
    if _C_DECODE is None:
        lib = ctypes.CDLL(str(Path(__file__).resolve().parent / "liboracle_decode.so"))
        f = lib.oracle_decode_attention
        f.restype = ctypes.c_int
        f.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 7 + [ctypes.c_float,
                                                                      ctypes.c_void_p, ctypes.c_int]
        _C_DECODE = f
    B, H, D = q.shape
    KVH, bs = k_cache.shape[2], k_cache.shape[1]
    qc = q.contiguous().view(torch.int16)
    kc = k_cache.contiguous().view(torch.int16)
    vc = v_cache.contiguous().view(torch.int16)
    lens = np.ascontiguousarray(cache_seqlens, dtype=np.int32)
    bt = np.ascontiguousarray(block_table, dtype=np.int32)
    out = torch.empty(B, H, D, dtype=torch.float32)
    rc = _C_DECODE(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), lens.ctypes.data, bt.ctypes.data,
                   B, H, KVH, D, bs, bt.shape[1], k_cache.shape[0], scale, out.data_ptr(),
                   threads or os.cpu_count() or 1)
    if rc != 0:
        raise ValueError("oracle_decode_attention: unsupported sizes, a length past its table "
                         "or a block id outside the cache")
    return out


def tree_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                   cu_seqlens_q, context_lens, tree_mask, block_table,
                   scale: float) -> torch.Tensor:
    """Ancestor-mask attention: node j of sequence b sees cache keys [0, ctx_b)
    and tree node i (cache position ctx_b + i) iff bit i of tree_mask[row j]."""
    cu_q = np.asarray(cu_seqlens_q, dtype=np.int64)
    ctx = np.asarray(context_lens, dtype=np.int64)
    masks = np.asarray(tree_mask).astype(np.uint64)
    out = torch.zeros(q.shape, dtype=torch.float32)
    for b in range(len(cu_q) - 1):
        qs, qe = int(cu_q[b]), int(cu_q[b + 1])
        n = qe - qs
        if n == 0:
            continue
        c = int(ctx[b])
        kb = gather_paged(k_cache, block_table[b], c + n)
        vb = gather_paged(v_cache, block_table[b], c + n)
        allowed = torch.ones(n, c + n, dtype=torch.bool)
        for j in range(n):
            w = int(masks[qs + j])
            allowed[j, c:] = torch.tensor([(w >> i) & 1 == 1 for i in range(n)])
        out[qs:qe] = _attend(q[qs:qe], kb, vb, scale, allowed)
    return out


# ------------------------------------------------------ engine-side metadata

def prepare_prefill_metadata(seqs, block_size: int):
    """Restates ModelRunner.prepare_prefill (model_runner.py:129-170).

    seqs: list of dicts with ``num_tokens`` (tokens scheduled end), ``start``
    (= num_cached_tokens), ``num_scheduled`` and ``block_table`` (list).
    Returns (cu_seqlens_q, cu_seqlens_k, max_q, max_k, slot_mapping,
    block_tables or None) as numpy int32 / ints.
    """
    cu_q, cu_k = [0], [0]
    max_q = max_k = 0
    slots = []
    for s in seqs:
        start = s["start"]
        seqlen_q = s["num_scheduled"]
        end = start + seqlen_q
        cu_q.append(cu_q[-1] + seqlen_q)
        cu_k.append(cu_k[-1] + end)
        max_q = max(max_q, seqlen_q)
        max_k = max(max_k, end)
        bt = s["block_table"]
        if not bt:
            continue
        for pos in range(start, end):
            slots.append(bt[pos // block_size] * block_size + pos % block_size)
    tables = None
    if cu_k[-1] > cu_q[-1]:  # prefix cache (model_runner.py:162-163)
        tables = padded_block_tables([s["block_table"] for s in seqs])
    return (np.array(cu_q, np.int32), np.array(cu_k, np.int32), max_q, max_k,
            np.array(slots, np.int32), tables)


def prepare_decode_metadata(seqs, block_size: int):
    """Restates ModelRunner.prepare_decode (model_runner.py:172-188).

    seqs: dicts with ``num_tokens`` (len(seq), the new token included) and
    ``block_table``. Returns (slot_mapping, context_lens, block_tables).
    """
    slots, lens = [], []
    for s in seqs:
        n = s["num_tokens"]
        last_block_tokens = n - (len(s["block_table"]) - 1) * block_size
        slots.append(s["block_table"][-1] * block_size + last_block_tokens - 1)
        lens.append(n)
    tables = padded_block_tables([s["block_table"] for s in seqs])
    return np.array(slots, np.int32), np.array(lens, np.int32), tables


def decode_graph_inputs(seqs, block_size: int, pad_rows: int, previous: dict) -> dict:
    """The decode graph's static inputs after one step: ModelRunner.prepare_decode
    (model_runner.py:172-188) followed by run_model's copies (:204-210), with
    pad_rows = the graph's batch rows (the fill_ and zero_ cover them all).

    seqs: dicts with ``last_token``, ``num_tokens`` and ``block_table``.
    previous: the buffers' contents before the step (``input_ids``,
    ``positions``, ``slot_mapping``, ``context_lens`` of >= pad_rows rows and
    a 2-D ``block_tables``); what the reference does not write keeps them.
    """
    out = {k: np.array(v, copy=True) for k, v in previous.items()}
    B = len(seqs)
    slots, lens, tables = prepare_decode_metadata(seqs, block_size)
    out["input_ids"][:B] = [s["last_token"] for s in seqs]          # :178, :204
    out["positions"][:B] = lens.astype(np.int64) - 1                 # :179, :205
    out["slot_mapping"][:pad_rows] = -1                              # :206
    out["slot_mapping"][:B] = slots                                  # :207
    out["context_lens"][:pad_rows] = 0                               # :208
    out["context_lens"][:B] = lens                                   # :209
    out["block_tables"][:B, :tables.shape[1]] = tables               # :210
    return out


def allreduce_sum(partials_bits: np.ndarray) -> np.ndarray:
    """Sum of bf16 partials over ranks, (world, n) uint16 bit patterns ->
    (n,) uint16: what dist.all_reduce(y) leaves in y (linear.py:155), restated
    with a fixed order: fp32 accumulation in rank order from rank 0's value,
    one round-to-nearest-even to bf16. With two ranks this is the single
    rounded bf16 add of NCCL's sum."""
    x = bf16_bits_to_f32(np.asarray(partials_bits, np.uint16))
    acc = x[0].astype(np.float32).copy()
    for p in range(1, x.shape[0]):
        acc = (acc + x[p]).astype(np.float32)
    return f32_to_bf16_bits(acc)


def padded_block_tables(tables):
    """model_runner.py:123-127: pad rows with -1 to the longest table."""
    width = max(len(t) for t in tables)
    return np.array([list(t) + [-1] * (width - len(t)) for t in tables], dtype=np.int32)


# ------------------------------------------------ q/k RMSNorm + rotary (fused)

def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bf16 bit patterns (NaN stays NaN)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    b = x.view(np.uint32)
    r = ((b + np.uint32(0x7FFF) + ((b >> 16) & np.uint32(1))) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        r[nan] = ((b[nan] >> 16) | np.uint32(0x40)).astype(np.uint16)
    return r


def _round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def rope_cache(head_dim: int, max_position: int, base: float) -> torch.Tensor:
    """The rotary module's buffer, (max_position, 1, head_dim) fp32 = [cos | sin].

    Same torch CPU operations as RotaryEmbedding.__init__
    (nanovllm/layers/rotary_embedding.py:25-33).
    """
    inv_freq = 1.0 / (base ** (torch.arange(0, head_dim, 2, dtype=torch.float) / head_dim))
    t = torch.arange(max_position, dtype=torch.float)
    freqs = torch.einsum("i,j -> ij", t, inv_freq)
    return torch.cat((freqs.cos(), freqs.sin()), dim=-1).unsqueeze_(1)


def qk_norm_rope(x_bits: np.ndarray, w_bits: np.ndarray, cos_sin_rows: np.ndarray,
                 eps: float) -> np.ndarray:
    """RMSNorm over the last dim (128) then rotary embedding, bf16 in and out.

    x_bits: (..., 128) uint16 rows; w_bits: (128,) uint16 weight;
    cos_sin_rows: (..., 128) float32 [cos(64) | sin(64)] of each row's
    position (broadcast over heads by the caller). Order of operations:
      lane sums (((((((x0^2 + x1^2) + x2^2) + x3^2) + x4^2) + x5^2) + x6^2) + x7^2
      over dims 8i..8i+7 (16 lanes per row), then a butterfly over lane
      distances 8, 4, 2, 1; var = sum / 128;
      r = 1 / sqrt(var + eps); n = bf16(bf16(x * r) * w)   (layernorm.py:20-24)
      out[:64] = n1*cos - n2*sin; out[64:] = n2*cos + n1*sin (rotary_embedding.py:11-13)
    """
    x = bf16_bits_to_f32(x_bits)
    shape = x.shape
    assert shape[-1] == 128
    x = x.reshape(-1, 128)
    cs = np.broadcast_to(np.asarray(cos_sin_rows, dtype=np.float32), shape).reshape(-1, 128)
    f32 = np.float32
    sq = (x * x).reshape(-1, 16, 8)
    lanes = sq[:, :, 0]
    for e in range(1, 8):
        lanes = lanes + sq[:, :, e]
    idx = np.arange(16)
    for off in (8, 4, 2, 1):
        lanes = lanes + lanes[:, idx ^ off]
    total = lanes[:, 0]
    var = total * f32(1.0 / 128.0)
    r = f32(1.0) / np.sqrt(var + f32(eps))
    w = bf16_bits_to_f32(w_bits)
    n = _round_bf16(_round_bf16(x * r[:, None]) * w[None, :])
    n1, n2 = n[:, :64], n[:, 64:]
    cos, sin = cs[:, :64], cs[:, 64:]
    out = np.concatenate(((n1 * cos) - (n2 * sin), (n2 * cos) + (n1 * sin)), axis=1)
    return f32_to_bf16_bits(out).reshape(shape)


def qk_norm_rope_store(positions: np.ndarray, q_bits: np.ndarray, k_bits: np.ndarray,
                       v_bits: np.ndarray, qw_bits: np.ndarray, kw_bits: np.ndarray,
                       cos_sin: np.ndarray, eps: float, k_cache=None, v_cache=None,
                       slot_mapping=None):
    """q (N,H,128), k/v (N,KVH,128) as uint16; cos_sin (max_pos, 1, 128) fp32.

    Returns (q_rot, k_rot) bit patterns; with caches and slot_mapping also
    scatters k_rot and v (store_kvcache semantics, slot -1 skipped).
    """
    pos = np.asarray(positions, dtype=np.int64)
    rows = np.asarray(cos_sin, dtype=np.float32).reshape(-1, 128)[pos][:, None, :]
    q_rot = qk_norm_rope(q_bits, qw_bits, rows, eps)
    k_rot = qk_norm_rope(k_bits, kw_bits, rows, eps)
    if slot_mapping is not None and k_cache is not None:
        store_kvcache(k_rot, np.ascontiguousarray(v_bits), k_cache, v_cache, slot_mapping)
    return q_rot, k_rot


# ------------------------------------------------------------------- sampling

_PHILOX_M = (np.uint64(0xD2511F53), np.uint64(0xCD9E8D57))
_PHILOX_W = (0x9E3779B9, 0xBB67AE85)


def philox4x32_10(ctr: np.ndarray, key) -> np.ndarray:
    """Philox4x32 with 10 rounds (Salmon, Moraes, Dror, Shaw, SC 2011).

    ctr: (..., 4) uint32 counters; key: two uint32 words. Returns (..., 4) uint32.
    """
    c = [np.asarray(ctr, dtype=np.uint64)[..., i] for i in range(4)]
    k0, k1 = int(key[0]) & 0xFFFFFFFF, int(key[1]) & 0xFFFFFFFF
    mask = np.uint64(0xFFFFFFFF)
    for r in range(10):
        if r:
            k0 = (k0 + _PHILOX_W[0]) & 0xFFFFFFFF
            k1 = (k1 + _PHILOX_W[1]) & 0xFFFFFFFF
        p0 = _PHILOX_M[0] * c[0]
        p1 = _PHILOX_M[1] * c[2]
        hi0, lo0 = p0 >> np.uint64(32), p0 & mask
        hi1, lo1 = p1 >> np.uint64(32), p1 & mask
        c = [hi1 ^ c[1] ^ np.uint64(k0), lo1, hi0 ^ c[3] ^ np.uint64(k1), lo0]
    return np.stack(c, axis=-1).astype(np.uint32)


def sample_uniforms(row: int, vocab: int, seed: int, offset: int) -> np.ndarray:
    """The 32-bit noise words of one row: column i takes word i % 4 of
    Philox4x32-10 at counter (i // 4, row, offset_lo, offset_hi), key (seed_lo, seed_hi)."""
    n = (vocab + 3) // 4
    ctr = np.zeros((n, 4), np.uint64)
    ctr[:, 0] = np.arange(n)
    ctr[:, 1] = row
    ctr[:, 2] = offset & 0xFFFFFFFF
    ctr[:, 3] = (offset >> 32) & 0xFFFFFFFF
    words = philox4x32_10(ctr, (seed & 0xFFFFFFFF, (seed >> 32) & 0xFFFFFFFF))
    return words.reshape(-1)[:vocab]


def sample_probs(logits: torch.Tensor, temperature: float) -> torch.Tensor:
    """The reference sampler's law: logits.float() / T, softmax (sampler.py:9-10)."""
    return torch.softmax(logits.float() / temperature, dim=-1)


def greedy_tokens(logits: torch.Tensor) -> torch.Tensor:
    """argmax over the last dim, first index on ties (torch.argmax)."""
    return logits.float().argmax(dim=-1)


def pick_keys(scores: np.ndarray, cols: np.ndarray) -> np.ndarray:
    """64-bit pick keys of float32 scores at global columns: monotone score
    bits (-0 folded into +0) in the high word, 0xFFFFFFFF - column in the low
    word; NaN and -inf give 0 (never picked). Unsigned order = pick order:
    larger score first, then the lower column."""
    s = np.asarray(scores, np.float32).copy()
    s[s == 0] = 0.0
    b = s.view(np.uint32).astype(np.uint64)
    neg = (b & np.uint64(0x80000000)) != 0
    hi = np.where(neg, (~b) & np.uint64(0xFFFFFFFF), b | np.uint64(0x80000000))
    key = (hi << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - np.asarray(cols, np.uint64))
    return np.where(s > -np.inf, key, np.uint64(0))


def greedy_shard_keys(logits: torch.Tensor, vocab_offset: int) -> np.ndarray:
    """Greedy pick key per row of one vocabulary shard of the LM head's
    logits (embed_head.py:56-61 gives rank r the columns
    [vocab_offset, vocab_offset + V/tp)): the key of its first maximal column."""
    x = logits.float().numpy()
    B, V = x.shape
    keys = pick_keys(x, np.broadcast_to(np.arange(V, dtype=np.uint64) + np.uint64(vocab_offset),
                                        (B, V)))
    return keys.max(axis=1) if V else np.zeros(B, np.uint64)


def merge_pick_keys(keys: np.ndarray) -> np.ndarray:
    """(S, B) uint64 keys -> (B,) int64 tokens: the column of the largest key
    per row, 0 where every key is 0. Equals sampling the gathered row
    (embed_head.py:62-65 followed by sampler.py:5-12)."""
    k = np.asarray(keys, np.uint64).max(axis=0)
    col = (np.uint64(0xFFFFFFFF) - (k & np.uint64(0xFFFFFFFF))).astype(np.int64)
    return np.where(k != 0, col, 0)
