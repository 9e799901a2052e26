"""TP rank-worker plumbing and the step watchdog, on CPU (gloo ranks, no GPU).

Mirrors the reference's host-only TP tests: worker lifecycle (tests/tp_worker_lifecycle.rs),
watchdog deadman timing (tp/mod.rs:1574-1642) and a failing rank poisoning the model.
"""
import os
import socket
import threading
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from helexa_b200.runtime.watchdog import StepTimeout, StepWatchdog


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model():
    from helexa_b200.config import get_preset
    from helexa_b200.models.reference import ReferenceModel
    from helexa_b200.weights.random_init import random_weights
    cfg = get_preset("tiny-qwen3-next")
    return ReferenceModel(cfg, random_weights(cfg, seed=0), gdn_chunk_threshold=16)


def _rank(rank, ws, port, q, fail_on):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        from helexa_b200.runtime.engine import Engine, FinishEvent
        from helexa_b200.runtime.prefix_cache import PrefixCache
        from helexa_b200.runtime.runner import RefRunner
        from helexa_b200.runtime.sampling import SamplingParams
        from helexa_b200.runtime.worker import LeaderRunner, follower_loop

        class Runner(RefRunner):
            def prefill(self, slot, tokens, p0):
                if fail_on and rank == 1 and len(tokens) == fail_on:
                    raise RuntimeError("injected rank failure")
                return super().prefill(slot, tokens, p0)

        local = Runner(_model(), num_slots=2, max_len=256)
        if rank == 0:
            leader = LeaderRunner(local, dist.group.WORLD)
            pc = PrefixCache(1 << 30, 4, on_evict=lambda s: leader.drop_snapshot(s.sid))
            eng = Engine(leader, prefix_cache=pc, im_start_id=999, snapshot_min_tokens=8)
            p = SamplingParams(temperature=0.0, repeat_penalty=1.0, max_tokens=4)
            res = []
            for prompt in ([5, 6, 7] * 6 + [999, 1, 2], [5, 6, 7] * 6 + [999, 1, 2, 8, 9, 999, 3]):
                toks, fin = eng.generate(prompt, p)
                res.append((toks, fin.reason, fin.cached_tokens))
            if fail_on:
                toks, fin = eng.generate(list(range(fail_on + 1)), p)
                res.append((toks, fin.reason, fin.error))
            eng.shutdown()
            if not eng.poisoned:
                leader.shutdown()
            st = local.states[0]
            q.put((0, res, [v.sum().item() for v in st.rec.values()]))
        else:
            follower_loop(local, dist.group.WORLD)
            st = local.states[0]
            q.put((1, None, [v.sum().item() for v in st.rec.values()]))
    finally:
        if not fail_on:
            dist.destroy_process_group()


def _launch(ws, fail_on=0):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_rank, args=(r, ws, port, q, fail_on)) for r in range(ws)]
    for p in ps:
        p.start()
    out = {}
    n = 1 if fail_on else ws
    for _ in range(n):
        r, res, sums = q.get(timeout=240)
        out[r] = (res, sums)
    for p in ps:
        p.join(5 if fail_on else 60)
        if p.is_alive():
            p.kill()
    return out


def test_leader_follower_lockstep_and_snapshots():
    out = _launch(2)
    res = out[0][0]
    assert res[0][1] == "length" and res[1][2] > 0          # second turn restored a snapshot
    assert out[0][1] == out[1][1]                           # follower state equals the leader's


def test_follower_failure_poisons_model():
    out = _launch(2, fail_on=10)  # the 11-token prompt prefills 10 tokens up to its snapshot cut
    toks, reason, err = out[0][0][-1]
    assert reason == "error" and "injected rank failure" in err


# ---- watchdog ------------------------------------------------------------------------
def test_watchdog_fires_and_aborts():
    aborted = threading.Event()
    wd = StepWatchdog(timeout_s=0.2, abort_deadline_s=5, on_timeout=aborted.set, on_deadman=lambda: None)
    with wd.step("fast"):
        time.sleep(0.01)
    assert not wd.fired.is_set()
    with pytest.raises(StepTimeout):
        with wd.step("slow"):
            time.sleep(0.6)
    assert aborted.is_set() and not wd.deadman_fired.is_set()
    with pytest.raises(StepTimeout):  # aborted communicator refuses further steps
        with wd.step("after"):
            pass
    wd.close()


def test_watchdog_deadman_when_abort_hangs():
    exited = threading.Event()
    wd = StepWatchdog(timeout_s=0.1, abort_deadline_s=0.3, on_timeout=lambda: time.sleep(5),
                      on_deadman=exited.set)
    t0 = time.monotonic()
    try:
        with wd.step("stuck"):
            exited.wait(3)
    except StepTimeout:
        pass
    assert exited.is_set() and wd.deadman_fired.is_set()
    assert 0.3 <= time.monotonic() - t0 < 3
    wd.close()
