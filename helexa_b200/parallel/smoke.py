"""Tensor-parallel smoke check (the reference's `neuron --tp-smoke`, tp/worker_pool.rs
smoke path): start one process per rank, rendezvous, ping every rank, run a sanity
all-reduce through the collective backend and, on GPUs, one through this package's
peer-memory reduction, then print `status=ok` (or `status=error ...`) and exit 0 / 1.

  python -m helexa_b200.parallel.smoke --tp 2            # NCCL + P2P on GPUs 0..1
  python -m helexa_b200.parallel.smoke --tp 2 --cpu      # gloo ranks on the host
"""
from __future__ import annotations

import argparse
import os
import socket
import sys


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank: int, ws: int, port: int, cpu: bool, q) -> None:
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        if cpu:
            dist.init_process_group("gloo", rank=rank, world_size=ws)
            dev = torch.device("cpu")
        else:
            torch.cuda.set_device(rank)
            dev = torch.device("cuda", rank)
            dist.init_process_group("nccl", rank=rank, world_size=ws, device_id=dev)
        # ping: every rank reports its rank id
        ids = [None] * ws
        dist.all_gather_object(ids, rank)
        assert ids == list(range(ws)), ids
        # sanity all-reduce through the collective backend: sum of ones == ws
        t = torch.ones(4, device=dev)
        dist.all_reduce(t)
        assert torch.all(t == ws), t
        p2p = "skipped"
        if not cpu:
            from .tp import TPComm
            comm = TPComm(device=dev, mode="p2p1")
            x = torch.zeros(1, 256, dtype=torch.bfloat16, device=dev)
            part = torch.full((1, 256), float(rank + 1), dtype=torch.bfloat16, device=dev)
            comm.reduce_residual(part, x)
            torch.cuda.synchronize(dev)
            comm.check()
            want = ws * (ws + 1) / 2
            assert torch.all(x.float() == want), x
            comm.close()
            p2p = "ok"
        q.put((rank, "ok", p2p))
    except Exception as e:  # reported by the parent
        q.put((rank, f"error {type(e).__name__}: {e}", ""))
    finally:
        if dist.is_initialized():
            dist.destroy_process_group()


def run(ws: int, cpu: bool, timeout_s: float = 120.0) -> tuple[bool, str]:
    import queue

    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, ws, port, cpu, q)) for r in range(ws)]
    for p in procs:
        p.start()
    res = {}
    try:
        while len(res) < ws:
            r, status, p2p = q.get(timeout=timeout_s)
            res[r] = (status, p2p)
    except queue.Empty:
        for p in procs:
            p.kill()
        return False, f"status=error ranks {sorted(set(range(ws)) - set(res))} did not report within {timeout_s}s"
    for p in procs:
        p.join(30)
    bad = {r: s for r, (s, _) in res.items() if s != "ok"}
    if bad:
        return False, "status=error " + "; ".join(f"rank {r}: {s}" for r, s in sorted(bad.items()))
    return True, f"status=ok ranks={ws} backend={'gloo' if cpu else 'nccl'} p2p={res[0][1]}"


def main() -> None:
    ap = argparse.ArgumentParser(description="tensor-parallel smoke check")
    ap.add_argument("--tp", type=int, default=2)
    ap.add_argument("--cpu", action="store_true", help="gloo ranks on the host (no GPU)")
    args = ap.parse_args()
    ok, line = run(args.tp, args.cpu)
    print(line)
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
