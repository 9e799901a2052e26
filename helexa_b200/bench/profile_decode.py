"""Decode-step driver for kernel profiling and per-step timing.

Builds a random-init model (optionally truncated to --layers to keep an ncu capture
small), places the sequence at --context tokens (the KV / GDN state contents do not
change the work a decode step does, so no prefill is run), then times --steps
decode steps with CUDA events, eagerly or as one replayed CUDA graph.

  python -m helexa_b200.bench.profile_decode --model qwen3-next-80b-a3b --layers 8 \
      --context 8192 --steps 20 [--eager]
"""
from __future__ import annotations

import argparse
import dataclasses
import json

import torch

from ..config import get_preset
from ..models.fast import FastModel


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-next-80b-a3b")
    ap.add_argument("--layers", type=int, default=0, help="truncate to the first N layers (0 = all)")
    ap.add_argument("--context", type=int, default=8192)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--eager", action="store_true")
    ap.add_argument("--quant", default=None, help="in-situ quantization (Q8_0, Q6_K, Q4_K, Q4_K_M)")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    ap.add_argument("--skip", default="", help="profiling only: comma list of gdn,attn,gdn_core,attn_core,ffn,experts")
    args = ap.parse_args()
    if args.no_pdl:
        from .. import ops
        ops.C.set_pdl(False)
    cfg = get_preset(args.model)
    if args.layers:
        cfg = dataclasses.replace(cfg, num_hidden_layers=args.layers, layer_types=cfg.layer_types[:args.layers])
    dev = torch.device("cuda", 0)
    fm = FastModel.random(cfg, dev, max_slots=args.batch, max_len=args.context + args.steps * 4 + 64)
    B = args.batch
    if args.quant:
        fm.quantize_(args.quant.upper())
    fm.profile_skip = set(x for x in args.skip.split(",") if x)
    if args.eager:
        nb = fm.buffers(B)
    else:
        nb = fm.capture(B, steps=args.steps)
    nb.slots.copy_(torch.arange(B, dtype=torch.int32, device=dev))

    def run():
        fm.pos.fill_(args.context)
        if args.eager:
            for _ in range(args.steps):
                fm.decode_step_launch(nb)
        else:
            fm.replay(nb)

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    gb = fm.decode_bytes_per_token() / 1e9
    print(json.dumps({"model": cfg.name, "layers": cfg.num_hidden_layers, "context": args.context, "batch": B,
                      "graph": not args.eager, "pdl": not args.no_pdl, "skip": args.skip, "ms_per_step": round(ms, 4),
                      "weight_gb_per_step": round(gb, 3), "achieved_gbs": round(gb / (ms / 1e3), 1),
                      "launches_per_step": fm.launches_per_step()}))


if __name__ == "__main__":
    main()
