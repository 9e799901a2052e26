"""Decode GEMV bandwidth (CUDA events, warm clocks) against cuBLAS, cycling through a
pool of weight copies larger than the 126 MB L2 so every call streams from HBM.

  python -m helexa_b200.bench.gemv_bench [--shapes 12352x2048,2048x4096,151936x2048]
"""
from __future__ import annotations

import argparse
import json

import torch

DEFAULT = "12352x2048,2048x4096,513x2048,1024x2048,151936x2048,9216x2048"


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
        nbytes = N * K * 2
        copies = max(2, (512 << 20) // nbytes + 1)
        Ws = [torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05 for _ in range(copies)]
        x = torch.randn(args.batch, K, device="cuda", dtype=torch.bfloat16)
        y = torch.empty(args.batch, N, device="cuda", dtype=torch.bfloat16)

        def run(fn):
            for i in range(5):
                fn(Ws[i % copies])
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(args.iters):
                fn(Ws[i % copies])
            e1.record()
            e1.synchronize()
            return e0.elapsed_time(e1) / args.iters * 1e3  # us

        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        us = run(lambda W: C.gemv(W, x, y, ops.STORE_BF16, None, None, 0.0))
        us_tma = run(lambda W: C.gemv_tma(W, x, y, ops.STORE_BF16, None, None, 0.0, err)) \
            if C.gemv_tma_ok(N, K, args.batch, 1) else float("nan")
        us_ref = run(lambda W: torch.matmul(x, W.t()))
        print(json.dumps({"N": N, "K": K, "batch": args.batch, "MB": round(nbytes / 1e6, 1), "ld_us": round(us, 2),
                          "ld_GBps": round(nbytes / us / 1e3, 1), "tma_us": round(us_tma, 2),
                          "tma_GBps": round(nbytes / us_tma / 1e3, 1), "cublas_us": round(us_ref, 2),
                          "cublas_GBps": round(nbytes / us_ref / 1e3, 1), "err": int(err.item())}))
        del Ws
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
