"""Golden vectors for the fused q/k RMSNorm + rotary op, from the reference's own modules.

Runs nanovllm.layers.layernorm.RMSNorm and nanovllm.layers.rotary_embedding
(get_rope) eagerly on CPU (torch.compile disabled: the decorated methods run
as written) on seeded bf16 inputs at the Qwen3-0.6B attention shape (16 Q /
8 KV heads, head_dim 128, rope theta 1e6, max_position 40960, eps 1e-6), the
same sequence of calls as Qwen3Attention.forward (qwen3.py:82-85). Needs the
reference source on sys.path:

    PYTHONPATH=<reference checkout> python tests/golden/make_qk_norm_golden.py

Writes tests/golden/qk_norm_rope_ref.npz (bf16 arrays as uint16 bit patterns).
"""
from pathlib import Path

import numpy as np
import torch
import torch._dynamo

torch._dynamo.config.disable = True

from nanovllm.layers.layernorm import RMSNorm  # noqa: E402
from nanovllm.layers.rotary_embedding import get_rope  # noqa: E402

N, H, KVH, D = 32, 16, 8, 128
MAX_POS, THETA, EPS = 40960, 1e6, 1e-6


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    g = torch.Generator().manual_seed(7)
    qkv = (torch.randn(N, (H + 2 * KVH) * D, generator=g) * 2.0).to(torch.bfloat16)
    qkv[3, :D] *= 40  # a row with a large norm
    qkv[5, H * D:(H + 1) * D] *= 1e-3  # a row with a tiny norm
    q, k, v = qkv.split([H * D, KVH * D, KVH * D], dim=-1)
    q = q.view(N, H, D)
    k = k.view(N, KVH, D)
    positions = torch.randint(0, MAX_POS, (N,), generator=g, dtype=torch.int64)
    positions[:4] = torch.tensor([0, 1, MAX_POS - 1, 4095])
    q_norm = RMSNorm(D, eps=EPS)
    k_norm = RMSNorm(D, eps=EPS)
    q_norm.weight.data = (1.0 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    k_norm.weight.data = (1.0 + 0.1 * torch.randn(D, generator=g)).to(torch.bfloat16)
    rope = get_rope(D, rotary_dim=D, max_position=MAX_POS, base=THETA)
    with torch.no_grad():
        qn = q_norm(q)
        kn = k_norm(k)
        qr, kr = rope(positions, qn, kn)
    out = Path(__file__).resolve().parent / "qk_norm_rope_ref.npz"
    np.savez_compressed(
        out, qkv=bits(qkv), positions=positions.numpy(), q_weight=bits(q_norm.weight.data),
        k_weight=bits(k_norm.weight.data), cos_sin_rows=rope.cos_sin_cache[positions].numpy(),
        q_norm=bits(qn), k_norm=bits(kn), q_rot=bits(qr), k_rot=bits(kr),
        meta=np.array([N, H, KVH, D, MAX_POS], dtype=np.int64), theta=np.float64(THETA),
        eps=np.float64(EPS))
    print("wrote", out, out.stat().st_size, "bytes")


if __name__ == "__main__":
    main()
