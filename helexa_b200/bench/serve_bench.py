"""Serving-shape benchmarks through FastRunner (the runner the engine drives), one rank
per GPU under torchrun for tensor parallelism. Device-timed with CUDA events; every
figure is the max over ranks.

Two serving workloads that a single-request bench does not cover:

* ``--mode prefix``: a cold request of ``--prompt`` tokens, a snapshot of the first
  ``--share`` tokens (attention K/V plus a deep copy of the GDN conv ring and recurrent
  state), then a second request with the same first ``--share`` tokens and a different
  suffix: restore + suffix prefill + first token is the warm TTFT. The warm request's
  first token is checked against a cold prefill of the same prompt (prefix snapshots
  must not change the output).
* ``--mode concurrent``: ``--requests`` requests of ``--prompt`` tokens are prefilled
  one after another into their own slots and then decoded together as one batch of
  ``--decode`` greedy steps (captured graphs of ``--graph-steps`` steps). Reports the
  aggregate decode tok/s and the p50 TTFT (the queue of prefills included).

  python -m helexa_b200.bench.serve_bench --mode prefix --prompt 8192 --share 7680
  torchrun --nproc-per-node 8 -m helexa_b200.bench.serve_bench --model qwen3-235b-a22b \
      --mode concurrent --requests 4 --prompt 4096 --decode 256 --ep
"""
from __future__ import annotations

import argparse
import json
import os
import statistics

import torch
import torch.distributed as dist

from ..config import get_preset
from ..models.fast import FastModel
from ..runtime.runner import FastRunner


def _max_over_ranks(vals: list[float], dev) -> list[float]:
    t = torch.tensor(vals, dtype=torch.float64, device=dev)
    if dist.is_initialized():
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


class _Timer:
    def __init__(self):
        self.a = torch.cuda.Event(enable_timing=True)
        self.b = torch.cuda.Event(enable_timing=True)

    def __enter__(self):
        torch.cuda.synchronize()
        self.a.record()
        return self

    def __exit__(self, *exc):
        self.b.record()
        self.b.synchronize()
        self.ms = self.a.elapsed_time(self.b)


def _first_token(logits: torch.Tensor) -> int:
    return int(logits.float().argmax().item())


def run_prefix(runner: FastRunner, cfg, args, dev):
    g = torch.Generator().manual_seed(7)
    P, S = args.prompt, args.share
    base = torch.randint(0, cfg.vocab_size, (P,), generator=g).tolist()
    other = base[:S] + torch.randint(0, cfg.vocab_size, (P - S,), generator=g).tolist()
    res = {"cold_ttft_ms": [], "warm_ttft_ms": [], "snapshot_ms": [], "restore_ms": []}
    tok_warm = tok_cold = None
    for it in range(args.warmup + args.reps):
        runner.reset(0)
        with _Timer() as t_cold:
            tok_cold_base = _first_token(runner.prefill(0, base, 0))
        runner.reset(0)
        runner.prefill(0, base[:S], 0)
        with _Timer() as t_snap:
            snap = runner.snapshot(0, S)
        runner.reset(0)
        runner.prefill(0, base, 0)  # the slot now holds a longer, different state
        with _Timer() as t_warm:
            runner.restore(0, snap)
            tok_warm = _first_token(runner.prefill(0, other[S:], S))
        with _Timer() as t_rest:
            runner.restore(0, snap)
        runner.reset(0)
        tok_cold = _first_token(runner.prefill(0, other, 0))
        del tok_cold_base
        if it >= args.warmup:
            res["cold_ttft_ms"].append(t_cold.ms)
            res["warm_ttft_ms"].append(t_warm.ms)
            res["snapshot_ms"].append(t_snap.ms)
            res["restore_ms"].append(t_rest.ms)
        snap_bytes = snap.nbytes
        del snap
    med = {k: statistics.median(v) for k, v in res.items()}
    med = dict(zip(med, _max_over_ranks(list(med.values()), dev)))
    return {"mode": "prefix", "prompt": P, "share": S, **{k: round(v, 3) for k, v in med.items()},
            "snapshot_mb": round(snap_bytes / 2**20, 1), "warm_first_token_matches_cold": tok_warm == tok_cold}


def run_concurrent(runner: FastRunner, cfg, args, dev):
    g = torch.Generator().manual_seed(11)
    R, P, D, gs = args.requests, args.prompt, args.decode, args.graph_steps
    prompts = [torch.randint(0, cfg.vocab_size, (P,), generator=g).tolist() for _ in range(R)]
    out = None
    for it in range(args.warmup + args.reps):
        firsts, ttft = [], []
        ev0 = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ev0.record()
        for r in range(R):
            runner.reset(r)
            firsts.append(_first_token(runner.prefill(r, prompts[r], 0)))
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            e.synchronize()
            ttft.append(ev0.elapsed_time(e))
        toks = firsts
        with _Timer() as t_dec:
            done = 1
            while done < D:
                n = min(gs, D - done)
                outs = runner.decode(list(range(R)), toks, n)
                toks = [o[-1] for o in outs]
                done += n
        if it >= args.warmup:
            vals = _max_over_ranks([statistics.median(ttft), t_dec.ms], dev)
            out = {"mode": "concurrent", "requests": R, "prompt": P, "decode": D, "ttft_p50_ms": round(vals[0], 2),
                   "decode_ms": round(vals[1], 2), "aggregate_decode_tok_s": round(R * (D - 1) / (vals[1] / 1e3), 1)}
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-next-80b-a3b")
    ap.add_argument("--mode", choices=["prefix", "concurrent"], default="prefix")
    ap.add_argument("--prompt", type=int, default=8192)
    ap.add_argument("--share", type=int, default=7680)
    ap.add_argument("--requests", type=int, default=4)
    ap.add_argument("--decode", type=int, default=256)
    ap.add_argument("--graph-steps", type=int, default=16)
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--ep", action="store_true", help="expert parallelism (whole experts per rank) for MoE layers")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    comm = None
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
        from ..parallel.tp import TPComm
        comm = TPComm(dist.group.WORLD, dev)
    cfg = get_preset(args.model)
    slots = args.requests + 1 if args.mode == "concurrent" else 2
    max_len = args.prompt + args.decode + 64
    model = FastModel.random(cfg, dev, seed=0, rank=rank, ws=world, max_slots=slots, max_len=max_len, comm=comm,
                             ep=args.ep)
    runner = FastRunner(model, graph_steps=args.graph_steps, prefill_chunk=args.prompt)
    res = run_prefix(runner, cfg, args, dev) if args.mode == "prefix" else run_concurrent(runner, cfg, args, dev)
    model.check_errors()
    if rank == 0:
        print(json.dumps({"model": cfg.name, "tp": world, "ep": args.ep, **res}))
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
