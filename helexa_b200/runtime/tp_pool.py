"""Tensor-parallel model serving: one rank process per GPU behind the node API.

A `tensor_parallel = N` load (harness/candle.rs:4588-4826; pool spawn tp/mod.rs:
509-579) starts N rank processes (`python -m helexa_b200.runtime.tp_pool`), one per
device. They rendezvous over torch.distributed on 127.0.0.1 (NCCL for the model's
collectives plus a gloo control group), each builds its shard of the model behind a
runner, and then:

  rank 0     wraps its runner in `LeaderRunner` (every call is broadcast to the
             followers, then run locally) and serves runner calls that the node
             process sends over an authenticated local socket;
  rank 1..N  run `follower_loop`.

The node process sees a `RemoteRunner` with the ordinary runner interface, so the
engine, prefix cache, admission and HTTP layers are the single-GPU ones
(tp/mod.rs:866-997 serves every request through the pool the same way).

Failure handling. Every call on rank 0 runs under the step watchdog; a step that
exceeds `HELEXA_TP_STEP_TIMEOUT_S` makes the rank exit (deadman), so the node sees
the connection drop. A follower's exception is reported at the call boundary and
returned as an error. Either way `RemoteRunner` raises, the engine poisons the model
and the registry's recovery unloads it (killing every rank process) and reloads it
from the retained spec. Rank processes are tied to the node process with
PR_SET_PDEATHSIG, so they never outlive it.
"""
from __future__ import annotations

import importlib
import json
import os
import secrets
import signal
import socket
import subprocess
import sys
import threading
import time
import traceback
from datetime import timedelta
from multiprocessing.connection import Client, Listener

import torch

EXIT_INIT_FAILED = 71


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _die_with_parent() -> None:
    """Deliver SIGKILL to this process when its parent exits (Linux prctl)."""
    try:
        import ctypes
        ctypes.CDLL("libc.so.6", use_errno=True).prctl(1, signal.SIGKILL)  # PR_SET_PDEATHSIG
    except OSError:
        pass


# ---------------------------------------------------------------------------
# runner builders (run inside a rank process; named as "module:function")
# ---------------------------------------------------------------------------
def cuda_fast_runner(rank: int, ws: int, cfg_args: dict):
    """The production builder: this rank's FastModel shard on its GPU with the TP
    communicator, behind a FastRunner."""
    import torch.distributed as dist

    from ..models.fast import FastModel
    from ..parallel.tp import TPComm
    from ..weights.loader import resolve_source
    from .runner import FastRunner

    dev = torch.device("cuda", torch.cuda.current_device())
    src = resolve_source(cfg_args["source"])
    cfg = src.config
    comm = TPComm(dist.group.WORLD, dev)
    kw = dict(rank=rank, ws=ws, max_slots=cfg_args["max_slots"], max_len=cfg_args["max_len"], comm=comm)
    if src.kind == "preset":
        model = FastModel.random(cfg, dev, seed=0, **kw)
    elif src.kind == "gguf":
        from ..weights.gguf import GGUFFile
        model = FastModel.from_gguf(cfg, GGUFFile(src.path), dev, **kw)
    else:
        from ..weights.loader import SafetensorsDir
        model = FastModel.from_hf(cfg, SafetensorsDir(src.path).get, dev, **kw)
    if cfg_args.get("quant"):
        model.quantize_(cfg_args["quant"].upper())
    return FastRunner(model)


def cpu_ref_runner(rank: int, ws: int, cfg_args: dict):
    """CPU builder for host-side tests of the pool: every rank holds the full fp32
    reference model of a preset (no sharding), so the plumbing -- spawn, rendezvous,
    lockstep calls, snapshots, failure reporting, shutdown -- runs without a GPU.
    `fail_rank` / `fail_prefill_len` inject a host-side exception on that rank for a
    prefill of that many tokens."""
    from ..config import get_preset
    from ..models.reference import ReferenceModel
    from ..weights.random_init import random_weights
    from .runner import RefRunner

    cfg = get_preset(cfg_args.get("preset", "tiny-qwen3-next"))
    model = ReferenceModel(cfg, random_weights(cfg, seed=0), gdn_chunk_threshold=16)
    fail_rank, fail_len = cfg_args.get("fail_rank"), cfg_args.get("fail_prefill_len")

    class Runner(RefRunner):
        def prefill(self, slot, tokens, p0):
            if rank == fail_rank and len(tokens) == fail_len:
                raise RuntimeError(f"injected failure on rank {rank}")
            return super().prefill(slot, tokens, p0)

    return Runner(model, num_slots=cfg_args.get("max_slots", 3) - 1, max_len=cfg_args.get("max_len", 256))


# ---------------------------------------------------------------------------
# rank process
# ---------------------------------------------------------------------------
def _rank_main(args: dict) -> None:
    import torch.distributed as dist

    from .watchdog import StepWatchdog
    from .worker import LeaderRunner, follower_loop

    _die_with_parent()
    rank, ws = args["rank"], args["ws"]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(args["port"]))
    if args["backend"] == "nccl":
        torch.cuda.set_device(args["device"])
        dist.init_process_group("nccl", rank=rank, world_size=ws, device_id=torch.device("cuda", args["device"]),
                                timeout=timedelta(seconds=args["pg_timeout_s"]))
    else:
        dist.init_process_group("gloo", rank=rank, world_size=ws, timeout=timedelta(seconds=args["pg_timeout_s"]))
    # the control group idles between requests, so it never times out on its own; a
    # dead rank is handled by the node (connection drop -> poison -> kill the ranks)
    ctrl = dist.new_group(backend="gloo", timeout=timedelta(days=365))
    mod, fn = args["builder"].split(":")
    conn = None
    try:
        if rank == 0:
            conn = Client(("127.0.0.1", args["ctl_port"]), authkey=bytes.fromhex(args["authkey"]))
        local = getattr(importlib.import_module(mod), fn)(rank, ws, args["builder_args"])
    except Exception:
        if conn is not None:
            conn.send(("init_err", traceback.format_exc(limit=5)))
        raise
    if rank != 0:
        follower_loop(local, ctrl)
        return
    wd = StepWatchdog(on_timeout=lambda: os._exit(70))
    leader = LeaderRunner(local, ctrl, watchdog=wd)
    conn.send(("ready", {"num_slots": local.num_slots, "max_len": local.max_len, "vocab": local.vocab,
                         "greedy_on_device": bool(getattr(local, "greedy_on_device", False)),
                         "sample_on_device": bool(getattr(local, "sample_on_device", False))}))
    snaps: dict[int, object] = {}
    while True:
        try:
            msg = conn.recv()
        except (EOFError, OSError):
            break
        if msg[0] == "close":
            break
        _, method, a = msg
        try:
            if method == "snapshot":
                ref = leader.snapshot(*a)
                snaps[ref.sid] = ref
                out = (ref.sid, ref.length, ref.nbytes)
            elif method == "restore":
                slot, sid = a
                leader.restore(slot, snaps[sid])
                out = None
            elif method == "drop_snapshot":
                snaps.pop(a[0], None)
                leader.drop_snapshot(a[0])
                out = None
            else:
                out = getattr(leader, method)(*a)
                if isinstance(out, torch.Tensor):
                    # plain numpy over the socket: torch's own tensor pickling would pass
                    # shared-memory handles that the node cannot open
                    conn.send(("ok_tensor", out.float().cpu().numpy()))
                    continue
            conn.send(("ok", out))
        except Exception as e:
            conn.send(("err", f"{e!r}\n{traceback.format_exc(limit=4)}"))
    leader.shutdown()
    wd.close()
    dist.destroy_process_group()


# ---------------------------------------------------------------------------
# node side
# ---------------------------------------------------------------------------
class TPPoolError(RuntimeError):
    pass


class RemoteSnapshot:
    """Handle of a snapshot held by every rank (nbytes: per rank)."""

    def __init__(self, sid: int, length: int, nbytes: int):
        self.sid, self.length, self.nbytes = sid, length, nbytes


class RemoteRunner:
    """The runner interface, forwarded to rank 0 of a TP pool."""

    def __init__(self, procs: list[subprocess.Popen], conn, info: dict):
        self.procs, self.conn = procs, conn
        self.num_slots, self.max_len, self.vocab = info["num_slots"], info["max_len"], info["vocab"]
        self.greedy_on_device = info["greedy_on_device"]
        self.sample_on_device = info.get("sample_on_device", False)
        self._mu = threading.Lock()
        self.closed = False

    def _call(self, method: str, *args):
        with self._mu:
            if self.closed:
                raise TPPoolError("tensor-parallel pool is closed")
            try:
                self.conn.send(("call", method, args))
                status, out = self.conn.recv()
            except (EOFError, OSError) as e:
                codes = [p.poll() for p in self.procs]
                raise TPPoolError(f"rank 0 connection lost ({e!r}); rank exit codes {codes}") from e
        if status == "ok_tensor":
            return torch.from_numpy(out)
        if status != "ok":
            raise TPPoolError(out)
        return out

    def reset(self, slot):
        return self._call("reset", slot)

    def prefill(self, slot, tokens, p0):
        return self._call("prefill", slot, list(tokens), p0)

    def decode(self, slots, tokens, steps):
        return self._call("decode", list(slots), list(tokens), steps)

    def decode_logits(self, slots, tokens):
        return self._call("decode_logits", list(slots), list(tokens))

    def decode_sampled(self, slots, tokens, steps, params, histories, draws, seeds):
        return self._call("decode_sampled", list(slots), list(tokens), steps, list(params),
                          [list(h[-64:]) for h in histories], list(draws), list(seeds))

    def snapshot(self, slot, length):
        return RemoteSnapshot(*self._call("snapshot", slot, length))

    def restore(self, slot, snap: RemoteSnapshot):
        return self._call("restore", slot, snap.sid)

    def drop_snapshot(self, snap: RemoteSnapshot):
        if not self.closed:
            try:
                self._call("drop_snapshot", snap.sid)
            except TPPoolError:
                pass

    def close(self, timeout: float = 20.0):
        """Stop every rank: a clean shutdown first, then SIGKILL for stragglers."""
        with self._mu:
            if self.closed:
                return
            self.closed = True
            try:
                self.conn.send(("close",))
            except OSError:
                pass
        t0 = time.monotonic()
        for p in self.procs:
            try:
                p.wait(max(0.1, timeout - (time.monotonic() - t0)))
            except subprocess.TimeoutExpired:
                pass
        for p in self.procs:
            if p.poll() is None:
                p.kill()
                p.wait(10)
        try:
            self.conn.close()
        except OSError:
            pass


def spawn_pool(ws: int, builder: str, builder_args: dict, devices: list[int] | None = None,
               backend: str = "nccl", init_timeout_s: float = 900.0, pg_timeout_s: float = 600.0,
               env: dict | None = None) -> RemoteRunner:
    """Start `ws` rank processes and return the node-side runner of rank 0."""
    authkey = secrets.token_bytes(16)
    lis = Listener(("127.0.0.1", 0), authkey=authkey)
    port = _free_port()
    procs = []
    base_env = dict(os.environ, **(env or {}))
    root = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    base_env["PYTHONPATH"] = root + os.pathsep + base_env.get("PYTHONPATH", "")
    for r in range(ws):
        args = dict(rank=r, ws=ws, port=port, ctl_port=lis.address[1], authkey=authkey.hex(), backend=backend,
                    device=(devices or list(range(ws)))[r], builder=builder, builder_args=builder_args,
                    pg_timeout_s=pg_timeout_s)
        procs.append(subprocess.Popen([sys.executable, "-m", "helexa_b200.runtime.tp_pool", json.dumps(args)],
                                      env=base_env))
    conn = None
    accepted: list = []
    acc = threading.Thread(target=lambda: _accept(lis, accepted), daemon=True)
    acc.start()
    deadline = time.monotonic() + init_timeout_s
    try:
        while not accepted:
            dead = [p.returncode for p in procs if p.poll() is not None]
            if dead or time.monotonic() > deadline:
                raise TPPoolError(f"tensor-parallel ranks failed to start (exit codes {dead or 'timeout'})")
            acc.join(0.2)
        if isinstance(accepted[0], BaseException):
            raise TPPoolError(f"rank 0 connection failed: {accepted[0]!r}")
        conn = accepted[0]
        while not conn.poll(1.0):
            dead = [p.returncode for p in procs if p.poll() is not None]
            if dead or time.monotonic() > deadline:
                raise TPPoolError(f"tensor-parallel ranks failed to start (exit codes {dead or 'timeout'})")
        status, info = conn.recv()
        if status != "ready":
            raise TPPoolError(f"rank 0 failed to build its shard:\n{info}")
        return RemoteRunner(procs, conn, info)
    except BaseException as e:
        for p in procs:
            if p.poll() is None:
                p.kill()
        for p in procs:
            p.wait(10)
        if conn is not None:
            conn.close()
        raise
    finally:
        lis.close()


def _accept(lis: Listener, out: list) -> None:
    try:
        out.append(lis.accept())
    except BaseException as e:  # listener closed or bad auth
        out.append(e)


def build_tp_served_model(spec, src, cfg, devs_free: list[int]):
    """Registry entry for `tensor_parallel > 1`: spawn the pool, wrap it in the
    ordinary engine / admission / serving objects."""
    from .registry import LoadError, plan_max_len

    tp = spec.tensor_parallel
    devices = spec.devices or list(range(tp))
    if len(devices) != tp:
        raise LoadError(f"tensor_parallel={tp} needs {tp} devices, got {devices}", "bad_tensor_parallel")
    if torch.cuda.device_count() < max(devices) + 1:
        raise LoadError(f"devices {devices} are not all present ({torch.cuda.device_count()} visible)",
                        "device_unavailable")
    weights_per_rank = int(cfg.param_count() * 2 / tp)
    max_len = plan_max_len(cfg, spec, min(devs_free), weights_per_rank)  # tightest rank bounds KV
    if max_len < 256:
        raise LoadError(f"only {max_len} tokens of KV fit beside the weights", "insufficient_memory")
    runner = spawn_pool(tp, "helexa_b200.runtime.tp_pool:cuda_fast_runner",
                        {"source": spec.source, "max_slots": spec.max_batch + 1, "max_len": max_len,
                         "quant": spec.quant}, devices=devices)
    return serve_runner(spec, src, cfg, runner, devices, max_len)


def serve_runner(spec, src, cfg, runner, devices, max_len):
    """Engine + admission + ServedModel around an already-built (remote) runner."""
    from dataclasses import asdict

    from .admission import AdmissionConfig, AdmissionController
    from .engine import Engine
    from .prefix_cache import PrefixCache
    from .sampling import GenerationDefaults
    from .serving import ServedModel
    from .tokenizer import load_tokenizer

    tok = load_tokenizer(src.path, cfg.vocab_size)
    pc = PrefixCache(spec.prefix_cache_mb << 20, spec.prefix_cache_entries,
                     on_evict=runner.drop_snapshot) if spec.prefix_cache_mb else None
    engine = Engine(runner, prefix_cache=pc, im_start_id=tok.token_id("<|im_start|>"), max_batch=spec.max_batch)
    adm = AdmissionController(AdmissionConfig(max_in_flight=spec.max_in_flight or spec.max_batch,
                                              max_queue_depth=spec.max_queue_depth, max_wait_s=spec.max_wait_s,
                                              max_per_principal=spec.max_per_principal))
    kv_bpt = cfg.kv_bytes_per_token() // max(1, min(spec.tensor_parallel, cfg.num_key_value_heads or 1))
    adm.set_kv_budget_mb((kv_bpt * max_len * spec.max_batch) >> 20)
    defaults = GenerationDefaults.from_dir(src.path) if src.path and os.path.isdir(src.path) else \
        GenerationDefaults()
    sm = ServedModel(model_id=spec.model_id, engine=engine, tokenizer=tok, config=cfg, admission=adm,
                     defaults=defaults, devices=list(devices), tensor_parallel=spec.tensor_parallel,
                     spec=asdict(spec), kv_bytes_per_token=kv_bpt)
    if torch.cuda.is_available() and devices:
        from .registry import free_device_bytes
        sm.free_vram_mb = lambda: min(free_device_bytes(d) for d in devices) >> 20
    return sm


if __name__ == "__main__":
    try:
        _rank_main(json.loads(sys.argv[1]))
    except SystemExit:
        raise
    except BaseException:
        traceback.print_exc()
        sys.stderr.flush()
        os._exit(EXIT_INIT_FAILED)
