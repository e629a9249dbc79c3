"""KV-cache scatter on the GPU: bit-exact against the oracle and the
reference's Triton kernel (golden fixture)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import GOLDEN, bf16_bits, from_bits
from oracle import reference_math as R

import nvattn
from nvattn import ops

pytestmark = pytest.mark.gpu
dev = torch.device("cuda")


def test_matches_reference_triton_golden():
    f = np.load(GOLDEN / "store_kvcache_triton.npz")
    N, H, KVH, d, nb, bs = (int(x) for x in f["shape"])
    qkv = from_bits(f["qkv"]).to(dev)
    _, k, v = qkv.split([H * d, KVH * d, KVH * d], dim=-1)
    k = k.contiguous().view(N, KVH, d)
    v = v.view(N, KVH, d)  # strided view: stride(0) = (H + 2KVH) d
    kc = torch.zeros(nb, bs, KVH, d, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    ops.store_kvcache(k, v, kc, vc, torch.from_numpy(f["slot_mapping"]).to(dev))
    torch.cuda.synchronize()
    assert np.array_equal(bf16_bits(kc), f["k_cache"])
    assert np.array_equal(bf16_bits(vc), f["v_cache"])
    assert ops.read_status() == 0


@pytest.mark.parametrize("N,KVH,H,frac_skip", [(1, 8, 16, 0.0), (7, 8, 16, 0.3),
                                               (1000, 8, 16, 0.1), (16384, 8, 16, 0.0),
                                               (333, 3, 6, 0.2), (64, 1, 8, 0.5),
                                               # rows of exactly 256 and of 512 16-byte vectors
                                               (40, 16, 32, 0.1), (20, 32, 64, 0.0)])
def test_random_slots_bit_exact(N, KVH, H, frac_skip):
    g = torch.Generator().manual_seed(N * 31 + KVH)
    nb, bs = (N + 255) // 256 + 3, 256
    qkv = torch.randn(N, (H + 2 * KVH) * 128, generator=g).to(torch.bfloat16)
    k = qkv[:, H * 128:(H + KVH) * 128].contiguous().view(N, KVH, 128)
    v = qkv[:, (H + KVH) * 128:].view(N, KVH, 128)
    slots = torch.randperm(nb * bs, generator=g)[:N].to(torch.int32)
    skip = torch.rand(N, generator=g) < frac_skip
    slots[skip] = -1
    kc0 = torch.randn(nb, bs, KVH, 128, generator=g).to(torch.bfloat16)
    vc0 = torch.randn(nb, bs, KVH, 128, generator=g).to(torch.bfloat16)
    kc, vc = kc0.to(dev), vc0.to(dev)
    qkv_d = qkv.to(dev)
    kd = qkv_d[:, H * 128:(H + KVH) * 128].contiguous().view(N, KVH, 128)
    vd = qkv_d[:, (H + KVH) * 128:].view(N, KVH, 128)
    ops.store_kvcache(kd, vd, kc, vc, slots.to(dev))
    torch.cuda.synchronize()
    ek, ev = bf16_bits(kc0), bf16_bits(vc0)
    R.store_kvcache(bf16_bits(k), np.ascontiguousarray(bf16_bits(v)), ek, ev, slots.numpy())
    assert np.array_equal(bf16_bits(kc), ek)
    assert np.array_equal(bf16_bits(vc), ev)
    assert ops.read_status() == 0


@pytest.mark.parametrize("N", [50, 3000])  # both layouts: vector per thread, warp per token
def test_unaligned_stride_takes_narrow_vectors(N):
    # value row stride of D+1 elements: 2-byte aligned only
    KVH = 2
    D = KVH * 128
    buf = torch.randn(N * (D + 1) + 1, device=dev).to(torch.bfloat16)
    v = buf[1:1 + N * (D + 1)].view(N, D + 1)[:, :D].view(N, KVH, 128)
    assert v.stride(0) == D + 1 and v.stride(1) == 128
    k = torch.randn(N, KVH, 128, device=dev).to(torch.bfloat16)
    nb = (N + 255) // 256
    kc = torch.zeros(nb, 256, KVH, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    slots = (torch.arange(N, dtype=torch.int64, device=dev) * 7 % (nb * 256)).to(torch.int32)
    assert len(set(slots.tolist())) == N
    ops.store_kvcache(k, v, kc, vc, slots)
    torch.cuda.synchronize()
    ek = np.zeros((nb, 256, KVH, 128), np.uint16)
    ev = np.zeros_like(ek)
    R.store_kvcache(bf16_bits(k), np.ascontiguousarray(bf16_bits(v)), ek, ev, slots.cpu().numpy())
    assert np.array_equal(bf16_bits(kc), ek) and np.array_equal(bf16_bits(vc), ev)


def test_out_of_range_slot_is_skipped_and_flagged():
    k = torch.randn(4, 1, 128, device=dev).to(torch.bfloat16)
    kc = torch.zeros(1, 256, 1, 128, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    ops.read_status()
    ops.store_kvcache(k, k, kc, vc, torch.tensor([0, 256, -5, 3], dtype=torch.int32, device=dev))
    st = ops.read_status()
    assert st & nvattn._lib.STATUS_BAD_SLOT
    assert torch.equal(kc[0, 0], k[0]) and torch.equal(kc[0, 3], k[3])
    assert int((kc != 0).any(dim=-1).sum()) == 2


def test_empty_batch_is_a_no_op():
    k = torch.empty(0, 8, 128, dtype=torch.bfloat16, device=dev)
    kc = torch.zeros(1, 256, 8, 128, dtype=torch.bfloat16, device=dev)
    ops.store_kvcache(k, k, kc, kc, torch.empty(0, dtype=torch.int32, device=dev))
    torch.cuda.synchronize()
    assert int(kc.abs().sum()) == 0


def test_kv_move_groups_bit_exact():
    g = torch.Generator().manual_seed(5)
    nb, KVH = 4, 8
    kc0 = torch.randn(nb, 256, KVH, 128, generator=g).to(torch.bfloat16)
    vc0 = torch.randn(nb, 256, KVH, 128, generator=g).to(torch.bfloat16)
    # group 0 shifts a path left onto its own sources; group 1 elsewhere
    src = np.array([303, 305, 310, 600, 601], np.int32)
    dst = np.array([301, 302, 303, 40, 41], np.int32)
    cu = np.array([0, 3, 5], np.int32)
    kc, vc = kc0.to(dev), vc0.to(dev)
    ops.kv_move(kc, vc, torch.from_numpy(src).to(dev), torch.from_numpy(dst).to(dev),
                torch.from_numpy(cu).to(dev))
    torch.cuda.synchronize()
    ek, ev = bf16_bits(kc0), bf16_bits(vc0)
    R.kv_move(ek, ev, src, dst, cu)
    assert np.array_equal(bf16_bits(kc), ek) and np.array_equal(bf16_bits(vc), ev)
    assert ops.read_status() == 0
