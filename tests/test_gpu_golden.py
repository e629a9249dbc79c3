"""nvattn kernels against flash-attn outputs recorded on a B200 (the
reference's own attention calls, attention.py:67-74, on the seeded cases)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from cases import CASES, make_case
from conftest import GOLDEN, from_bits
from helpers import assert_close

from nvattn import ops

pytestmark = pytest.mark.gpu
dev = torch.device("cuda")


@pytest.mark.parametrize("name", CASES)
def test_matches_flash_attn_golden(name):
    path = GOLDEN / "flash_attn_golden.npz"
    if not path.exists():
        pytest.skip("flash-attn golden vectors not recorded")
    ref = from_bits(np.load(path)[name])
    c = make_case(name)
    if c["kind"] == "varlen":
        bt = None if c["block_table"] is None else c["block_table"].to(dev)
        if "qkv" in c:
            H, KVH = c["H"], c["KVH"]
            _, k, v = c["qkv"].to(dev).split([H * 128, KVH * 128, KVH * 128], dim=-1)
            k, v = k.contiguous().view(-1, KVH, 128), v.view(-1, KVH, 128)
        else:
            k, v = c["k"].to(dev), c["v"].to(dev)
        out = ops.flash_attn_varlen_func(c["q"].to(dev), k, v, max_seqlen_q=c["max_q"],
                                         cu_seqlens_q=c["cu_q"].to(dev),
                                         max_seqlen_k=c["max_k"],
                                         cu_seqlens_k=c["cu_k"].to(dev),
                                         softmax_scale=128 ** -0.5, causal=True, block_table=bt)
    else:
        out = ops.flash_attn_with_kvcache(c["q"].to(dev).unsqueeze(1), c["k_cache"].to(dev),
                                          c["v_cache"].to(dev),
                                          cache_seqlens=c["cache_seqlens"].to(dev),
                                          block_table=c["block_table"].to(dev),
                                          softmax_scale=128 ** -0.5, causal=True)[:, 0]
    torch.cuda.synchronize()
    # both sides are bf16 outputs of fp32-accumulated attention
    assert_close(out, ref)
