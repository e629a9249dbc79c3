"""Golden outputs of the reference's attention calls, produced on a B200.

The reference's attention math is flash-attn's CUDA code (called at
nanovllm/layers/attention.py:67-74); it has no CPU path, so its outputs are
recorded on the GPU box by calling flash-attn exactly as the reference does,
on the seeded cases of ``cases.py``:

    python tests/golden/make_flash_attn_golden.py --out flash_attn_golden.npz

The resulting npz (bf16 outputs as uint16 bit patterns, plus the flash-attn
version) is committed as tests/golden/flash_attn_golden.npz. If flash-attn
cannot run, the script writes the error instead and exits 0.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np
import torch

sys.path.insert(0, str(Path(__file__).resolve().parent))
from cases import CASES, make_case  # noqa: E402


def run_case(c: dict) -> torch.Tensor:
    from flash_attn import flash_attn_varlen_func, flash_attn_with_kvcache
    dev = torch.device("cuda")
    scale = 128 ** -0.5
    if c["kind"] == "varlen":
        bt = None if c["block_table"] is None else c["block_table"].to(dev)
        if c["block_table"] is None and "qkv" in c:
            # rebuild the strided v view on the device, as the engine passes it
            H, KVH = c["H"], c["KVH"]
            qkv = c["qkv"].to(dev)
            _, k, v = qkv.split([H * 128, KVH * 128, KVH * 128], dim=-1)
            k = k.contiguous().view(-1, KVH, 128)
            v = v.view(-1, KVH, 128)
        else:
            k, v = c["k"].to(dev), c["v"].to(dev)
        o = flash_attn_varlen_func(c["q"].to(dev), k, v,
                                   max_seqlen_q=c["max_q"], cu_seqlens_q=c["cu_q"].to(dev),
                                   max_seqlen_k=c["max_k"], cu_seqlens_k=c["cu_k"].to(dev),
                                   softmax_scale=scale, causal=True, block_table=bt)
    else:
        o = flash_attn_with_kvcache(c["q"].to(dev).unsqueeze(1), c["k_cache"].to(dev),
                                    c["v_cache"].to(dev),
                                    cache_seqlens=c["cache_seqlens"].to(dev),
                                    block_table=c["block_table"].to(dev),
                                    softmax_scale=scale, causal=True)
        o = o.squeeze(1)
    torch.cuda.synchronize()
    return o.cpu()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", required=True)
    args = ap.parse_args()
    out = Path(args.out)
    out.parent.mkdir(parents=True, exist_ok=True)
    try:
        import flash_attn
        res = {"flash_attn_version": np.array(flash_attn.__version__),
               "device": np.array(torch.cuda.get_device_name())}
        for name in CASES:
            o = run_case(make_case(name))
            res[name] = o.view(torch.int16).numpy().view(np.uint16)
        np.savez_compressed(out, **res)
        print("flash-attn", flash_attn.__version__, "ran on", torch.cuda.get_device_name())
    except Exception as e:  # record why the reference's GPU path did not run
        out.with_suffix(".json").write_text(json.dumps({"error": repr(e)}))
        print("flash-attn did not run:", repr(e))


if __name__ == "__main__":
    main()
