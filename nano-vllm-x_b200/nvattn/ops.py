"""Torch-facing operators over the libnvattn C ABI.

Each function mirrors one call the reference makes from
``nanovllm/layers/attention.py`` — same argument names and meaning, same
assertions — and forwards raw device pointers, element strides and the
current CUDA stream to the C entry point. Nothing here computes attention:
on a machine without the CUDA library these functions raise.

    store_kvcache            attention.py:33-40 (+ Triton kernel :10-30)
    flash_attn_varlen_func   flash-attn call at attention.py:67-70
    flash_attn_with_kvcache  flash-attn call at attention.py:72-74
    tree_attention           new: EAGLE-style draft-tree verification
    kv_move                  new: in-cache compaction of accepted slots
    qk_norm_rope_store       q/k RMSNorm + rotary + scatter, the steps of
                             Qwen3Attention.forward at qwen3.py:82-86
    sample                   Sampler.forward (sampler.py:5-12) / greedy argmax
    sample_shard,            the same pick per vocabulary shard and the merge
    sample_merge             of the shards' keys, in place of ParallelLMHead's
                             logits gather at TP > 1 (embed_head.py:56-66)

Every launch is asynchronous on ``torch.cuda.current_stream()``, performs
no host synchronisation and allocates only through torch's caching
allocator, so the decode path can be captured in a CUDA graph the way
``ModelRunner.capture_cudagraph`` (model_runner.py:222-257) does.
"""
from __future__ import annotations

import torch

from . import _lib

__all__ = [
    "store_kvcache",
    "flash_attn_varlen_func",
    "flash_attn_with_kvcache",
    "varlen_prefill",
    "paged_decode",
    "tree_attention",
    "kv_move",
    "qk_norm_rope_store",
    "sample",
    "sample_shard",
    "sample_merge",
    "decode_workspace_bytes",
    "tree_workspace_bytes",
    "status_tensor",
    "read_status",
]

_status: dict[int, torch.Tensor] = {}


def _require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = None
    for t in tensors:
        if t is None:
            continue
        if not t.is_cuda:
            raise ValueError("nvattn operates on CUDA tensors only (no CPU fallback); "
                             f"got a tensor on {t.device}")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"tensors on different devices: {dev} and {t.device}")
    return dev


def _dev_index(device) -> int:
    if device is None:
        return torch.cuda.current_device()
    if isinstance(device, int):
        return device
    device = torch.device(device)
    return device.index if device.index is not None else torch.cuda.current_device()


def status_tensor(device: torch.device | int | None = None) -> torch.Tensor | None:
    """Per-device int32 status word that kernels OR error bits into.

    Created on first use outside stream capture; while a capture is running
    and the word does not exist yet, None (no status reporting) is used.
    """
    idx = _dev_index(device)
    t = _status.get(idx)
    if t is None:
        if torch.cuda.is_current_stream_capturing():
            return None
        # a normal tensor even when first used under torch.inference_mode(),
        # so read_status() can clear it anywhere
        with torch.inference_mode(False):
            t = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status[idx] = t
    return t


def read_status(device: torch.device | int | None = None, clear: bool = True) -> int:
    """Return (and by default clear) the device status bits (synchronises)."""
    t = status_tensor(device)
    if t is None:
        return 0
    v = int(t.item())
    if clear:
        t.zero_()
    return v


def _status_ptr(device: torch.device) -> int | None:
    t = status_tensor(device)
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check_bf16(*tensors: torch.Tensor) -> None:
    for t in tensors:
        if t is not None and t.dtype != torch.bfloat16:
            raise TypeError(f"nvattn kernels take bfloat16 tensors, got {t.dtype}")


def _check_i32(name: str, t: torch.Tensor) -> None:
    if t.dtype != torch.int32:
        raise TypeError(f"{name} must be int32, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


# --------------------------------------------------------------------- scatter

def store_kvcache(key: torch.Tensor, value: torch.Tensor, k_cache: torch.Tensor,
                  v_cache: torch.Tensor, slot_mapping: torch.Tensor) -> None:
    """k_cache.view(-1, D)[slot] = key.view(N, D) for every slot != -1; same for V.

    Same contract and assertions as store_kvcache in
    nanovllm/layers/attention.py:33-40.
    """
    N, num_heads, head_dim = key.shape
    D = num_heads * head_dim
    assert key.stride(-1) == 1 and value.stride(-1) == 1
    assert key.stride(1) == head_dim and value.stride(1) == head_dim
    assert k_cache.stride(1) == D and v_cache.stride(1) == D
    assert slot_mapping.numel() == N
    dev = _require_cuda(key, value, k_cache, v_cache, slot_mapping)
    _check_bf16(key, value, k_cache, v_cache)
    _check_i32("slot_mapping", slot_mapping)
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("k_cache/v_cache must be contiguous [num_blocks, block_size, kv_heads, d]")
    if k_cache.shape != v_cache.shape:
        raise ValueError("k_cache and v_cache shapes differ")
    num_slots = k_cache.numel() // D
    _lib.call("nvattn_store_kvcache", key.data_ptr(), key.stride(0), value.data_ptr(),
              value.stride(0), k_cache.data_ptr(), v_cache.data_ptr(), slot_mapping.data_ptr(),
              N, D, num_slots, _status_ptr(dev), _stream(dev))


# --------------------------------------------------------------------- prefill

def varlen_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   cu_seqlens_q: torch.Tensor, cu_seqlens_k: torch.Tensor,
                   max_seqlen_q: int, max_seqlen_k: int, softmax_scale: float | None = None,
                   causal: bool = False, block_table: torch.Tensor | None = None,
                   out: torch.Tensor | None = None) -> torch.Tensor:
    """Varlen attention with flash_attn_varlen_func's contract (attention.py:67-70).

    q: (total_q, H, d). Dense: k, v (total_k, KVH, d). Paged (block_table
    given): k, v are the caches (num_blocks, block_size, KVH, d) and
    block_table (batch, max_blocks) int32. Causal masks are bottom-right
    aligned. Returns (total_q, H, d) bf16.
    """
    dev = _require_cuda(q, k, v, cu_seqlens_q, cu_seqlens_k, block_table, out)
    _check_bf16(q, k, v, out)
    _check_i32("cu_seqlens_q", cu_seqlens_q)
    _check_i32("cu_seqlens_k", cu_seqlens_k)
    if q.dim() != 3:
        raise ValueError("q must be (total_q, num_heads, head_dim)")
    total_q, num_heads, head_dim = q.shape
    if q.stride(-1) != 1 or k.stride(-1) != 1 or v.stride(-1) != 1:
        raise ValueError("q/k/v must have a contiguous last dimension")
    num_seqs = cu_seqlens_q.numel() - 1
    if cu_seqlens_k.numel() != num_seqs + 1:
        raise ValueError("cu_seqlens_q and cu_seqlens_k lengths differ")
    if softmax_scale is None:
        softmax_scale = head_dim ** -0.5
    if out is None:
        out = torch.empty((total_q, num_heads, head_dim), dtype=q.dtype, device=q.device)
    if block_table is not None:
        _check_i32("block_table", block_table)
        if k.dim() != 4 or k.shape != v.shape:
            raise ValueError("paged k/v must be caches (num_blocks, block_size, kv_heads, d)")
        if not (k.is_contiguous() and v.is_contiguous()):
            raise ValueError("paged caches must be contiguous")
        num_blocks, block_size, num_kv_heads, hd = k.shape
        if block_table.shape[0] != num_seqs:
            raise ValueError("block_table rows != number of sequences")
        args_kv = (k.data_ptr(), 0, 0, v.data_ptr(), 0, 0)
        total_k = 0
        bt_ptr, bt_stride, bt_width = (block_table.data_ptr(), block_table.stride(0),
                                       block_table.shape[1])
    else:
        if k.dim() != 3 or k.shape != v.shape:
            raise ValueError("dense k/v must be (total_k, kv_heads, d)")
        total_k, num_kv_heads, hd = k.shape
        num_blocks = block_size = 0
        args_kv = (k.data_ptr(), k.stride(0), k.stride(1), v.data_ptr(), v.stride(0), v.stride(1))
        bt_ptr, bt_stride, bt_width = None, 0, 0
    if hd != head_dim:
        raise ValueError("q and k/v head_dim differ")
    if num_heads % num_kv_heads:
        raise ValueError("num_heads must be a multiple of num_kv_heads")
    _lib.call("nvattn_varlen_prefill", q.data_ptr(), q.stride(0), q.stride(1), *args_kv,
              out.data_ptr(), out.stride(0), out.stride(1), cu_seqlens_q.data_ptr(),
              cu_seqlens_k.data_ptr(), num_seqs, int(max_seqlen_q), int(max_seqlen_k), total_q,
              total_k, bt_ptr, bt_stride, bt_width, num_blocks, block_size, num_heads, num_kv_heads,
              head_dim, float(softmax_scale), 1 if causal else 0, _status_ptr(dev), _stream(dev))
    return out


def flash_attn_varlen_func(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                           dropout_p: float = 0.0, softmax_scale=None, causal: bool = False,
                           block_table=None, **unsupported):
    """Keyword-compatible stand-in for the flash-attn call at attention.py:67-70."""
    if dropout_p:
        raise NotImplementedError("dropout is not supported (inference path)")
    for key, val in unsupported.items():
        if val not in (None, False, 0, 0.0, (-1, -1)):
            raise NotImplementedError(f"flash_attn_varlen_func option {key}={val!r}")
    return varlen_prefill(q, k, v, cu_seqlens_q, cu_seqlens_k, max_seqlen_q, max_seqlen_k,
                          softmax_scale=softmax_scale, causal=causal, block_table=block_table)


# ---------------------------------------------------------------------- decode

def decode_workspace_bytes(batch: int, num_heads: int, num_kv_heads: int, max_blocks: int,
                           block_size: int) -> int:
    return int(_lib.load().nvattn_decode_workspace_bytes(batch, num_heads, num_kv_heads,
                                                         max_blocks, block_size))


def paged_decode(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 cache_seqlens: torch.Tensor, block_table: torch.Tensor,
                 softmax_scale: float | None = None, out: torch.Tensor | None = None,
                 workspace: torch.Tensor | None = None) -> torch.Tensor:
    """One query token per sequence over the paged cache; q, out: (B, H, d)."""
    dev = _require_cuda(q, k_cache, v_cache, cache_seqlens, block_table, out, workspace)
    _check_bf16(q, k_cache, v_cache, out)
    _check_i32("cache_seqlens", cache_seqlens)
    _check_i32("block_table", block_table)
    if q.dim() != 3:
        raise ValueError("q must be (batch, num_heads, head_dim)")
    batch, num_heads, head_dim = q.shape
    if q.stride(-1) != 1:
        raise ValueError("q must have a contiguous last dimension")
    if k_cache.dim() != 4 or k_cache.shape != v_cache.shape:
        raise ValueError("caches must be (num_blocks, block_size, kv_heads, d)")
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("caches must be contiguous")
    num_blocks, block_size, num_kv_heads, hd = k_cache.shape
    if hd != head_dim:
        raise ValueError("q and cache head_dim differ")
    if num_heads % num_kv_heads:
        raise ValueError("num_heads must be a multiple of num_kv_heads")
    if cache_seqlens.numel() != batch or block_table.shape[0] != batch:
        raise ValueError("cache_seqlens/block_table rows must equal the batch size")
    max_blocks = block_table.shape[1]
    if softmax_scale is None:
        softmax_scale = head_dim ** -0.5
    if out is None:
        out = torch.empty((batch, num_heads, head_dim), dtype=q.dtype, device=q.device)
    ws_bytes = decode_workspace_bytes(batch, num_heads, num_kv_heads, max_blocks, block_size)
    if ws_bytes and (workspace is None or workspace.numel() * workspace.element_size() < ws_bytes):
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    ws_ptr = workspace.data_ptr() if (ws_bytes and workspace is not None) else None
    _lib.call("nvattn_paged_decode", q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(),
              v_cache.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
              cache_seqlens.data_ptr(), block_table.data_ptr(), block_table.stride(0),
              max_blocks, num_blocks, block_size, batch, num_heads, num_kv_heads, head_dim,
              float(softmax_scale), ws_ptr, ws_bytes, _status_ptr(dev), _stream(dev))
    return out


def flash_attn_with_kvcache(q, k_cache, v_cache, cache_seqlens=None, block_table=None,
                            softmax_scale=None, causal: bool = False, **unsupported):
    """Keyword-compatible stand-in for the flash-attn call at attention.py:72-74.

    q: (batch, seqlen_q, H, d) -> returns (batch, seqlen_q, H, d). seqlen_q == 1
    is the decode kernel; longer queries run the paged varlen kernel with
    bottom-right causal alignment (flash-attn's semantics).
    """
    for key, val in unsupported.items():
        if val is not None and val is not False:
            raise NotImplementedError(f"flash_attn_with_kvcache option {key}={val!r}")
    if cache_seqlens is None or block_table is None:
        raise NotImplementedError("only the paged form (cache_seqlens + block_table) is built")
    if isinstance(cache_seqlens, int):
        cache_seqlens = torch.full((q.shape[0],), cache_seqlens, dtype=torch.int32,
                                   device=q.device)
    batch, seqlen_q, num_heads, head_dim = q.shape
    if seqlen_q == 1:
        o = paged_decode(q[:, 0], k_cache, v_cache, cache_seqlens, block_table, softmax_scale)
        return o.unsqueeze(1)
    cu_q = torch.arange(0, (batch + 1) * seqlen_q, seqlen_q, dtype=torch.int32, device=q.device)
    cu_k = torch.zeros(batch + 1, dtype=torch.int32, device=q.device)
    torch.cumsum(cache_seqlens, 0, out=cu_k[1:])
    max_k = block_table.shape[1] * k_cache.shape[1]
    o = varlen_prefill(q.reshape(batch * seqlen_q, num_heads, head_dim), k_cache, v_cache, cu_q,
                       cu_k, seqlen_q, max_k, softmax_scale=softmax_scale, causal=causal,
                       block_table=block_table)
    return o.view(batch, seqlen_q, num_heads, head_dim)


# ------------------------------------------------------------------------ tree

def tree_workspace_bytes(num_seqs: int, max_nodes: int, total_q: int, num_heads: int,
                         num_kv_heads: int, max_blocks: int, block_size: int) -> int:
    return int(_lib.load().nvattn_tree_workspace_bytes(num_seqs, max_nodes, total_q, num_heads,
                                                       num_kv_heads, max_blocks, block_size))


def tree_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                   cu_seqlens_q: torch.Tensor, context_lens: torch.Tensor,
                   tree_mask: torch.Tensor, block_table: torch.Tensor, max_nodes: int,
                   softmax_scale: float | None = None, out: torch.Tensor | None = None,
                   workspace: torch.Tensor | None = None) -> torch.Tensor:
    """Draft-tree verification attention.

    q: (total_nodes, H, d); sequence b's nodes are rows cu_seqlens_q[b]..;
    their K/V sit in the cache at positions context_lens[b] + node index.
    tree_mask: (total_nodes,) int64 (bit pattern of a uint64): bit i set =>
    the row attends tree node i. Every committed token is visible.
    """
    dev = _require_cuda(q, k_cache, v_cache, cu_seqlens_q, context_lens, tree_mask, block_table,
                        out)
    _check_bf16(q, k_cache, v_cache, out)
    _check_i32("cu_seqlens_q", cu_seqlens_q)
    _check_i32("context_lens", context_lens)
    _check_i32("block_table", block_table)
    if tree_mask.dtype not in (torch.int64, torch.uint64) or not tree_mask.is_contiguous():
        raise TypeError("tree_mask must be a contiguous int64/uint64 tensor")
    total_q, num_heads, head_dim = q.shape
    if tree_mask.numel() != total_q:
        raise ValueError("tree_mask needs one word per query row")
    if k_cache.dim() != 4 or k_cache.shape != v_cache.shape:
        raise ValueError("caches must be (num_blocks, block_size, kv_heads, d)")
    num_blocks, block_size, num_kv_heads, _ = k_cache.shape
    num_seqs = cu_seqlens_q.numel() - 1
    if max_nodes > 64:
        raise ValueError("at most 64 tree nodes per sequence")
    if softmax_scale is None:
        softmax_scale = head_dim ** -0.5
    if out is None:
        out = torch.empty((total_q, num_heads, head_dim), dtype=q.dtype, device=q.device)
    ws_bytes = tree_workspace_bytes(num_seqs, int(max_nodes), total_q, num_heads, num_kv_heads,
                                    block_table.shape[1], block_size)
    if ws_bytes and (workspace is None or workspace.numel() * workspace.element_size() < ws_bytes):
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device)
    ws_ptr = workspace.data_ptr() if (ws_bytes and workspace is not None) else None
    _lib.call("nvattn_tree_verify", q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(),
              v_cache.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
              cu_seqlens_q.data_ptr(), context_lens.data_ptr(), tree_mask.data_ptr(),
              block_table.data_ptr(), block_table.stride(0), block_table.shape[1], num_blocks,
              block_size, num_seqs, int(max_nodes), total_q, num_heads, num_kv_heads, head_dim,
              float(softmax_scale), ws_ptr, ws_bytes, _status_ptr(dev), _stream(dev))
    return out


def kv_move(k_cache: torch.Tensor, v_cache: torch.Tensor, src_slots: torch.Tensor,
            dst_slots: torch.Tensor, cu_moves: torch.Tensor) -> None:
    """Grouped in-cache row moves (accepted-path compaction after verification)."""
    dev = _require_cuda(k_cache, v_cache, src_slots, dst_slots, cu_moves)
    _check_bf16(k_cache, v_cache)
    for n, t in (("src_slots", src_slots), ("dst_slots", dst_slots), ("cu_moves", cu_moves)):
        _check_i32(n, t)
    if not (k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("caches must be contiguous")
    if src_slots.numel() != dst_slots.numel():
        raise ValueError("src_slots and dst_slots lengths differ")
    D = k_cache.shape[-2] * k_cache.shape[-1]
    num_slots = k_cache.numel() // D
    _lib.call("nvattn_kv_move", k_cache.data_ptr(), v_cache.data_ptr(), src_slots.data_ptr(),
              dst_slots.data_ptr(), cu_moves.data_ptr(), cu_moves.numel() - 1, src_slots.numel(),
              D, num_slots,
              _status_ptr(dev), _stream(dev))


# ------------------------------------------------------- fused q/k producer side

def qk_norm_rope_store(positions: torch.Tensor, q: torch.Tensor, k: torch.Tensor,
                       v: torch.Tensor, q_weight: torch.Tensor, k_weight: torch.Tensor,
                       cos_sin_cache: torch.Tensor, eps: float,
                       k_cache: torch.Tensor | None = None, v_cache: torch.Tensor | None = None,
                       slot_mapping: torch.Tensor | None = None, need_k: bool = True,
                       q_out: torch.Tensor | None = None, k_out: torch.Tensor | None = None
                       ) -> tuple[torch.Tensor, torch.Tensor | None]:
    """One launch for ``q = q_norm(q); k = k_norm(k); q, k = rotary_emb(positions, q, k)``
    (qwen3.py:82-86) plus, when caches and slot_mapping are given, the K/V
    scatter of ``store_kvcache`` (attention.py:33-40, slot -1 skipped).

    q: (N, H, 128), k/v: (N, KVH, 128) bf16 views with unit element and head
    strides (the split of the fused QKV projection); q_weight/k_weight: the
    RMSNorm weights (128,) bf16; cos_sin_cache: the rotary module's fp32
    buffer (max_position, 1, 128) = [cos | sin]; positions: (N,) int64.
    Returns (q_rot (N, H, 128), k_rot (N, KVH, 128) or None if not need_k).
    """
    dev = _require_cuda(positions, q, k, v, q_weight, k_weight, cos_sin_cache, k_cache, v_cache,
                        slot_mapping, q_out, k_out)
    _check_bf16(q, k, v, q_weight, k_weight, k_cache, v_cache, q_out, k_out)
    N, H, d = q.shape
    KVH = k.shape[1]
    if k.shape != (N, KVH, d) or v.shape != (N, KVH, d):
        raise ValueError("q, k, v token counts or head sizes differ")
    for n, t in (("q", q), ("k", k), ("v", v)):
        if t.stride(-1) != 1 or t.stride(1) != d:
            raise ValueError(f"{n} must have unit element stride and head stride head_dim")
    if positions.dtype != torch.int64 or positions.numel() != N or not positions.is_contiguous():
        raise ValueError("positions must be int64 with one entry per token")
    if cos_sin_cache.dtype != torch.float32 or not cos_sin_cache.is_contiguous() \
            or cos_sin_cache.shape[-1] != d:
        raise ValueError("cos_sin_cache must be a contiguous fp32 (max_position, 1, head_dim) tensor")
    for n, t in (("q_weight", q_weight), ("k_weight", k_weight)):
        if t.numel() != d or not t.is_contiguous():
            raise ValueError(f"{n} must be a contiguous ({d},) tensor")
    max_position = cos_sin_cache.numel() // d
    if q_out is None:
        q_out = torch.empty((N, H, d), dtype=torch.bfloat16, device=dev)
    if k_out is None and need_k:
        k_out = torch.empty((N, KVH, d), dtype=torch.bfloat16, device=dev)
    for n, t, shape in (("q_out", q_out, (N, H, d)), ("k_out", k_out, (N, KVH, d))):
        if t is not None and (tuple(t.shape) != shape or not t.is_contiguous()):
            raise ValueError(f"{n} must be contiguous {shape}")
    store = slot_mapping is not None and k_cache is not None and k_cache.numel() > 0
    num_slots = 0
    if store:
        _check_i32("slot_mapping", slot_mapping)
        if slot_mapping.numel() != N:
            raise ValueError("slot_mapping must have one entry per token")
        if not (k_cache.is_contiguous() and v_cache.is_contiguous()) or k_cache.shape != v_cache.shape:
            raise ValueError("k_cache/v_cache must be contiguous and of equal shape")
        if k_cache.shape[-2] * k_cache.shape[-1] != KVH * d:
            raise ValueError("cache rows do not match num_kv_heads * head_dim")
        num_slots = k_cache.numel() // (KVH * d)
    _lib.call("nvattn_qk_norm_rope_store", q.data_ptr(), q.stride(0), k.data_ptr(), k.stride(0),
              v.data_ptr(), v.stride(0), q_weight.data_ptr(), k_weight.data_ptr(),
              cos_sin_cache.data_ptr(), max_position, positions.data_ptr(),
              slot_mapping.data_ptr() if store else None, q_out.data_ptr(),
              k_out.data_ptr() if k_out is not None else None,
              k_cache.data_ptr() if store else None, v_cache.data_ptr() if store else None,
              num_slots, N, H, KVH, d, float(eps), _status_ptr(dev), _stream(dev))
    return q_out, k_out


# -------------------------------------------------------------------- sampling

_sample_calls = 0


def sample(logits: torch.Tensor, temperatures: torch.Tensor | None = None,
           seed: int | None = None, offset: int | None = None,
           out: torch.Tensor | None = None) -> torch.Tensor:
    """One token per row of (B, V) bf16 logits, one kernel.

    temperatures (B,) fp32: rows with T > 0 are sampled from softmax(logits/T)
    (the law of Sampler.forward, sampler.py:5-12); rows with T <= 0, or all
    rows when temperatures is None, take the greedy argmax (first index on
    ties, as torch.argmax). The noise is Philox4x32-10 keyed by ``seed``
    (default: drawn from torch's CPU generator) at counter ``offset``
    (default: a per-process call count, so repeated calls differ).
    Returns (B,) int64.
    """
    global _sample_calls
    dev = _require_cuda(logits, temperatures, out)
    _check_bf16(logits)
    if logits.dim() != 2 or logits.stride(-1) != 1:
        raise ValueError("logits must be a (B, V) tensor with unit column stride")
    B, V = logits.shape
    if temperatures is not None:
        if temperatures.dtype != torch.float32 or temperatures.numel() != B \
                or not temperatures.is_contiguous():
            raise ValueError("temperatures must be a contiguous float32 (B,) tensor")
    if seed is None:
        seed = int(torch.randint(0, 2 ** 62, (1,)).item())
    if offset is None:
        offset = _sample_calls
    _sample_calls += 1
    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=dev)
    elif out.dtype != torch.int64 or out.numel() != B or not out.is_contiguous():
        raise ValueError("out must be a contiguous int64 (B,) tensor")
    _lib.call("nvattn_sample", logits.data_ptr(), logits.stride(0), B, V,
              temperatures.data_ptr() if temperatures is not None else None,
              int(seed) & (2 ** 64 - 1), int(offset) & (2 ** 64 - 1), out.data_ptr(), _stream(dev))
    return out


def _check_sample_rows(logits: torch.Tensor, temperatures: torch.Tensor | None):
    _check_bf16(logits)
    if logits.dim() != 2 or logits.stride(-1) != 1:
        raise ValueError("logits must be a (B, V) tensor with unit column stride")
    B = logits.shape[0]
    if temperatures is not None:
        if temperatures.dtype != torch.float32 or temperatures.numel() != B \
                or not temperatures.is_contiguous():
            raise ValueError("temperatures must be a contiguous float32 (B,) tensor")


def sample_shard(logits: torch.Tensor, vocab_offset: int, temperatures: torch.Tensor | None = None,
                 *, seed: int, offset: int, out: torch.Tensor | None = None) -> torch.Tensor:
    """Pick keys of one vocabulary shard: (B, V_shard) bf16 logits holding
    global columns [vocab_offset, vocab_offset + V_shard).

    Returns (B,) int64 holding each row's 64-bit key (the bits of a uint64;
    unsigned order = pick order). ``seed`` and ``offset`` are required: every
    shard of a row must draw the same noise. The largest key over all shards
    (``sample_merge``) gives the token ``sample`` gives on the whole row.
    """
    dev = _require_cuda(logits, temperatures, out)
    _check_sample_rows(logits, temperatures)
    B, V = logits.shape
    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=dev)
    elif out.dtype != torch.int64 or out.numel() != B or not out.is_contiguous():
        raise ValueError("out must be a contiguous int64 (B,) tensor")
    _lib.call("nvattn_sample_shard", logits.data_ptr(), logits.stride(0), B, V, int(vocab_offset),
              temperatures.data_ptr() if temperatures is not None else None,
              int(seed) & (2 ** 64 - 1), int(offset) & (2 ** 64 - 1), out.data_ptr(), _stream(dev))
    return out


def sample_merge(keys: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """Tokens from (S, B) int64 keys of S shards (or (B,) for one): the
    column of each row's largest key, 0 where no shard had a candidate."""
    dev = _require_cuda(keys, out)
    if keys.dtype != torch.int64 or not keys.is_contiguous() or keys.dim() not in (1, 2):
        raise ValueError("keys must be a contiguous int64 (S, B) or (B,) tensor")
    S, B = (1, keys.shape[0]) if keys.dim() == 1 else keys.shape
    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=dev)
    elif out.dtype != torch.int64 or out.numel() != B or not out.is_contiguous():
        raise ValueError("out must be a contiguous int64 (B,) tensor")
    if S == 0:
        raise ValueError("keys must hold at least one shard")
    _lib.call("nvattn_sample_merge", keys.data_ptr(), S, B, out.data_ptr(), _stream(dev))
    return out
