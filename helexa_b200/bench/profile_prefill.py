"""Prefill timing by phase (GDN mixer / attention mixer / MoE / dense MLP / head) with
CUDA events, on a random-init model (optionally truncated to --layers).

  python -m helexa_b200.bench.profile_prefill --model qwen3-next-80b-a3b --tokens 8192
"""
from __future__ import annotations

import argparse
import dataclasses
import json

import torch

from ..config import get_preset
from ..models.fast import FastModel, PhaseTimer


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-next-80b-a3b")
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--reps", type=int, default=2)
    args = ap.parse_args()
    cfg = get_preset(args.model)
    if args.layers:
        cfg = dataclasses.replace(cfg, num_hidden_layers=args.layers, layer_types=cfg.layer_types[:args.layers])
    dev = torch.device("cuda", 0)
    fm = FastModel.random(cfg, dev, max_slots=1, max_len=args.tokens + 64)
    toks = torch.randint(0, cfg.vocab_size, (args.tokens,), device=dev, dtype=torch.int32)
    fm.prefill(0, toks, 0)  # warm-up
    torch.cuda.synchronize()
    for _ in range(args.reps):
        fm.prefill_timer = PhaseTimer()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fm.prefill(0, toks, 0)
        e1.record()
        e1.synchronize()
        phases = fm.prefill_timer.totals()
        fm.prefill_timer = None
        print(json.dumps({"model": cfg.name, "layers": cfg.num_hidden_layers, "tokens": args.tokens,
                          "prefill_ms": round(e0.elapsed_time(e1), 2), "phases_ms": phases}))


if __name__ == "__main__":
    main()
