"""Standalone decode-attention timing (CUDA events) on one sequence of a given context
length, small enough for an ncu capture (a few tens of MB on the device).

  python -m helexa_b200.bench.attn_bench --context 8192 --hq 16 --hkv 2 --dim 256 --splits 32
"""
from __future__ import annotations

import argparse
import json

import torch


def main():
    from .. import ops
    ap = argparse.ArgumentParser()
    ap.add_argument("--context", type=int, default=8192)
    ap.add_argument("--hq", type=int, default=16)
    ap.add_argument("--hkv", type=int, default=2)
    ap.add_argument("--dim", type=int, default=256)
    ap.add_argument("--splits", type=int, default=32)
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--graph", action="store_true", help="time replays of a CUDA graph of the launches")
    ap.add_argument("--cold", action="store_true",
                    help="write a 256 MB buffer (2x L2) before every launch and subtract the time of the writes alone")
    args = ap.parse_args()
    C = ops.C
    D, Hq, Hkv = args.dim, args.hq, args.hkv
    gated = True
    qw = 2 * D
    L = args.context + 16
    kc = torch.randn(1, Hkv, L, D, device="cuda").bfloat16()
    vc = torch.randn(1, Hkv, L, D, device="cuda").bfloat16()
    proj = torch.randn(1, Hq * qw + 2 * Hkv * D, device="cuda").bfloat16()
    qn = torch.ones(D, device="cuda")
    inv = (1.0 / (1e7 ** (torch.arange(0, D // 4, 2).float() / (D // 4)))).cuda()
    part_o = torch.empty(1, Hq, args.splits, D, device="cuda")
    part_ml = torch.empty(1, Hq, args.splits, 2, device="cuda")
    cnt = torch.zeros(1, Hkv, dtype=torch.int32, device="cuda")
    out = torch.empty(1, Hq * D, device="cuda", dtype=torch.bfloat16)
    slots = torch.zeros(1, dtype=torch.int32, device="cuda")
    pos = torch.full((1,), args.context, dtype=torch.int32, device="cuda")

    def run():
        C.attn_decode(proj, qn, qn, inv, kc, vc, slots, pos, part_o, part_ml, cnt, out, Hq, Hkv, D, D // 4, gated,
                      1e-6)

    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def timed(fn) -> float:
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        body = fn
        if args.graph:
            g = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                with torch.cuda.graph(g, stream=s):
                    for _ in range(args.iters):
                        fn()
            torch.cuda.current_stream().wait_stream(s)
            g.replay()
            torch.cuda.synchronize()
            body = None
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        if body is None:
            g.replay()
        else:
            for _ in range(args.iters):
                body()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1)

    if args.cold:
        ms = timed(lambda: (flush.fill_(1), run())) - timed(lambda: flush.fill_(1))
    else:
        ms = timed(run)
    us = ms / args.iters * 1e3
    kv_bytes = 2 * Hkv * (args.context + 1) * D * 2
    print(json.dumps({"context": args.context, "hq": Hq, "hkv": Hkv, "dim": D, "splits": args.splits, "graph": args.graph, "cold": args.cold,
                      "us": round(us, 2), "kv_MB": round(kv_bytes / 1e6, 2),
                      "GBps": round(kv_bytes / us / 1e3, 1)}))


if __name__ == "__main__":
    main()
