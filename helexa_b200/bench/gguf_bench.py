"""Fused-dequant k-quant decode GEMV bandwidth (CUDA events, warm clocks), cycling
through weight copies larger than the 126 MB L2 so every call streams blocks from HBM.

Default shapes are Qwen3-32B's decode projections (N x K): fused q/k/v, o_proj,
gate+up (SiLU-pair epilogue), down_proj; each in Q4_K and Q6_K (padded 224-byte rows).

  python -m helexa_b200.bench.gguf_bench [--shapes 10240x5120,...] [--batch 1]
"""
from __future__ import annotations

import argparse
import json

import torch

DEFAULT = "10240x5120,5120x8192,51200x5120,5120x25600"
Q4_K, Q6_K, Q6_K_PADDED = 12, 14, 114
BLOCK = {Q4_K: (144, 256), Q6_K_PADDED: (224, 256)}


def main():
    from .. import ops
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default=DEFAULT)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--iters", type=int, default=50)
    args = ap.parse_args()
    C = ops.C
    for s in args.shapes.split(","):
        N, K = (int(v) for v in s.split("x"))
        w = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
        x = torch.randn(args.batch, K, device="cuda", dtype=torch.bfloat16)
        for gt in (Q4_K, Q6_K):
            raw = C.gguf_quant(w, gt)
            t = gt
            if gt == Q6_K:
                raw, t = C.gguf_pad_q6k(raw), Q6_K_PADDED
            nbytes = raw.numel()
            copies = max(2, (512 << 20) // nbytes + 1)
            Ws = [raw.clone() for _ in range(copies)]
            for mode, name in ((ops.STORE_BF16, "store"),) + (((ops.SILU_PAIR, "silu_pair"),) if N > 4 * K else ()):
                y = torch.empty(args.batch, N // 2 if mode == ops.SILU_PAIR else N, device="cuda",
                                dtype=torch.bfloat16)
                for i in range(5):
                    C.gguf_gemv(Ws[i % copies], t, K, x, y, mode, None, None, 0.0)
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for i in range(args.iters):
                    C.gguf_gemv(Ws[i % copies], t, K, x, y, mode, None, None, 0.0)
                e1.record()
                e1.synchronize()
                us = e0.elapsed_time(e1) / args.iters * 1e3
                print(json.dumps({"N": N, "K": K, "type": "Q4_K" if gt == Q4_K else "Q6_K(224)", "epilogue": name,
                                  "batch": args.batch, "MB": round(nbytes / 1e6, 1), "us": round(us, 2),
                                  "GBps": round(nbytes / us / 1e3, 1)}))
            del Ws
            torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
