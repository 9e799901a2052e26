"""Tensor-parallel rank workers: every rank runs the same runner call in lockstep.

Rank 0 owns the engine. Each runner call it makes (prefill, decode, snapshot,
restore, reset, ...) is first broadcast to the follower ranks over a host control
group (gloo) and then executed locally; followers run `follower_loop`, executing the
same call on their shard, so the NCCL / peer-memory collectives inside the model line
up across ranks. This replaces the reference's newline-JSON RPC over child stdin with
a reply drain per step (tp/mod.rs:42-1572, tp/rpc.rs:313-570): here there are no
per-step replies, because every rank computes identical token ids (the lm_head and the
sampler are replicated).

Failure handling: the call is wrapped in the step watchdog; a follower that raises
reports the exception through the control group at the next call boundary and the
leader poisons the model.
"""
from __future__ import annotations

import traceback

import torch.distributed as dist

from .watchdog import StepWatchdog

SHUTDOWN = "__shutdown__"


class RankError(RuntimeError):
    pass


def _bcast(obj, group, src: int = 0):
    buf = [obj]
    dist.broadcast_object_list(buf, src=src, group=group)
    return buf[0]


class LeaderRunner:
    """Rank-0 proxy: forwards each call to the followers, then runs it locally."""

    def __init__(self, local, control_group, watchdog: StepWatchdog | None = None):
        self.local = local
        self.group = control_group
        self.wd = watchdog
        self.num_slots = local.num_slots
        self.max_len = local.max_len
        self.vocab = local.vocab
        self.greedy_on_device = getattr(local, "greedy_on_device", False)
        self.sample_on_device = getattr(local, "sample_on_device", False)
        self._snap_ids = 0
        self._snaps: dict[int, object] = {}

    def _call(self, method: str, *args):
        _bcast((method, args), self.group)
        if self.wd is None:
            out = getattr(self.local, method)(*args)
        else:
            with self.wd.step(method):
                out = getattr(self.local, method)(*args)
        # followers report failures at the call boundary
        status = [None] * dist.get_world_size(self.group)
        dist.all_gather_object(status, None, group=self.group)
        errs = [s for s in status if s]
        if errs:
            raise RankError("follower failed: " + errs[0])
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
        # every rank samples with the same seeds and counters from the same gathered
        # logits, so all ranks pick the same tokens
        return self._call("decode_sampled", list(slots), list(tokens), steps, list(params),
                          [list(h[-64:]) for h in histories], list(draws), list(seeds))

    def snapshot(self, slot, length):
        # every rank keeps its own shard of the snapshot under a shared id
        self._snap_ids += 1
        sid = self._snap_ids
        _bcast(("snapshot_store", (sid, slot, length)), self.group)
        local = self.local.snapshot(slot, length)
        self._snaps[sid] = local
        status = [None] * dist.get_world_size(self.group)
        dist.all_gather_object(status, None, group=self.group)
        return _SnapRef(sid, local, self)

    def restore(self, slot, snap):
        _bcast(("snapshot_restore", (snap.sid, slot)), self.group)
        self.local.restore(slot, snap.local)
        status = [None] * dist.get_world_size(self.group)
        dist.all_gather_object(status, None, group=self.group)
        errs = [s for s in status if s]
        if errs:
            raise RankError("follower failed: " + errs[0])

    def drop_snapshot(self, sid: int):
        self._snaps.pop(sid, None)
        _bcast(("snapshot_drop", (sid,)), self.group)
        status = [None] * dist.get_world_size(self.group)
        dist.all_gather_object(status, None, group=self.group)

    def shutdown(self):
        _bcast((SHUTDOWN, ()), self.group)


class _SnapRef:
    """Leader-side handle of a snapshot held by every rank; `nbytes` is per rank."""

    def __init__(self, sid, local, leader):
        self.sid = sid
        self.local = local
        self.leader = leader
        self.length = local.length

    @property
    def nbytes(self):
        return self.local.nbytes


def follower_loop(local, control_group) -> None:
    """Run on ranks 1..N-1 until the leader broadcasts a shutdown."""
    snaps: dict[int, object] = {}
    while True:
        method, args = _bcast(None, control_group)
        if method == SHUTDOWN:
            return
        err = None
        try:
            if method == "snapshot_store":
                sid, slot, length = args
                snaps[sid] = local.snapshot(slot, length)
            elif method == "snapshot_restore":
                sid, slot = args
                local.restore(slot, snaps[sid])
            elif method == "snapshot_drop":
                snaps.pop(args[0], None)
            else:
                getattr(local, method)(*args)
        except Exception as e:  # reported to the leader, which poisons the model
            err = f"rank {dist.get_rank()}: {e!r}\n{traceback.format_exc(limit=3)}"
        status = [None] * dist.get_world_size(control_group)
        dist.all_gather_object(status, err, group=control_group)
