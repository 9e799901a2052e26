"""Causal attention prefill timing (CUDA events, after warm-up): the tcgen05/TMEM kernel,
the mma.sync kernel and PyTorch SDPA (library flash attention) on the same inputs.

  python -m helexa_b200.bench.attn_prefill_bench --tokens 8192 --hq 16 --hkv 2 --dim 256

FLOPs count the causal half: 2 matmuls x 2 FLOP x T(T+1)/2 x D per query head.
"""
from __future__ import annotations

import argparse
import json

import torch


def main():
    from .. import ops
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--hq", type=int, default=16)
    ap.add_argument("--hkv", type=int, default=2)
    ap.add_argument("--dim", type=int, default=256)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--only", default="", help="comma list of tc,mma,sdpa (default all)")
    args = ap.parse_args()
    C = ops.C
    T, Hq, Hkv, D = args.tokens, args.hq, args.hkv, args.dim
    torch.manual_seed(0)
    q = torch.randn(T, Hq * D, device="cuda").bfloat16()
    kc = torch.randn(Hkv, T, D, device="cuda").bfloat16()
    vc = torch.randn(Hkv, T, D, device="cuda").bfloat16()
    out = torch.empty(T, Hq * D, device="cuda").bfloat16()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    qs = q.view(T, Hq, D).transpose(0, 1)[None]
    runs = {
        "tc": lambda: C.attn_prefill_tc(q, kc, vc, out, Hq, 0, D ** -0.5, None, 0, err),
        "mma": lambda: C.attn_prefill(q, kc, vc, out, Hq, 0, D ** -0.5),
        "sdpa": lambda: torch.nn.functional.scaled_dot_product_attention(qs, kc[None], vc[None], is_causal=True,
                                                                         enable_gqa=True),
    }
    only = [x for x in args.only.split(",") if x] or list(runs)
    flops = 4.0 * T * (T + 1) / 2 * D * Hq
    res = {}
    for name in only:
        fn = runs[name]
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.iters):
            fn()
        e1.record()
        e1.synchronize()
        ms = e0.elapsed_time(e1) / args.iters
        res[name] = {"ms": round(ms, 4), "tflops": round(flops / ms / 1e9, 1)}
    res["device_error"] = int(err.item())
    print(json.dumps({"tokens": T, "hq": Hq, "hkv": Hkv, "dim": D, **res}))


if __name__ == "__main__":
    main()
