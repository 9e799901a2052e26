"""Engine on the CPU reference runner: greedy parity, batching, prefix snapshots
(KV + GDN state restore must equal a cold prefill, arch/qwen3_5/snapshot.rs tests),
stop conditions and poisoning."""
import pytest
import torch

from helexa_b200.config import get_preset
from helexa_b200.models.reference import ReferenceModel
from helexa_b200.runtime.engine import Engine, FinishEvent
from helexa_b200.runtime.prefix_cache import PrefixCache
from helexa_b200.runtime.runner import RefRunner
from helexa_b200.runtime.sampling import SamplingParams


@pytest.fixture(scope="module")
def model():
    from helexa_b200.weights.random_init import random_weights
    from test_fast_model_gpu import _realistic
    cfg = get_preset("tiny-qwen3-next")
    torch.manual_seed(0)
    return ReferenceModel(cfg, _realistic(cfg, random_weights(cfg, seed=0, std=0.05)), gdn_chunk_threshold=16)


def _greedy_direct(m, prompt, n):
    st = m.new_state()
    lg = m.forward(torch.tensor(prompt), st)
    out = []
    for _ in range(n):
        t = int(lg.argmax())
        out.append(t)
        lg = m.forward(torch.tensor([t]), st)
    return out


def _params(n, **kw):
    return SamplingParams(temperature=0.0, repeat_penalty=1.0, max_tokens=n, **kw)


def test_engine_greedy_and_batching(model):
    eng = Engine(RefRunner(model, num_slots=3), max_batch=3)
    try:
        prompts = [[(7 * i + j) % 1000 for i in range(20 + 3 * j)] for j in range(3)]
        reqs = [eng.submit(p, _params(6)) for p in prompts]
        for p, r in zip(prompts, reqs):
            toks = []
            fin = None
            for ev in r.iter_events(timeout=120):
                if isinstance(ev, FinishEvent):
                    fin = ev
                else:
                    toks += ev.token_ids
            assert toks == _greedy_direct(model, p, 6)
            assert fin.reason == "length" and fin.completion_tokens == 6 and fin.prompt_tokens == len(p)
    finally:
        eng.shutdown()


def test_engine_prefix_snapshot_restore_equals_cold(model):
    im = 999
    pc = PrefixCache(budget_bytes=1 << 30, max_entries=4)
    eng = Engine(RefRunner(model, num_slots=2), prefix_cache=pc, im_start_id=im, snapshot_min_tokens=8)
    try:
        turn1 = [5, 6, 7] * 10 + [im] + [11, 12, 13]
        toks1, f1 = eng.generate(turn1, _params(4))
        assert f1.cached_tokens == 0 and len(pc) == 1
        turn2 = turn1 + toks1 + [im] + [21, 22]
        toks2, f2 = eng.generate(turn2, _params(4))
        assert f2.cached_tokens == len(turn1) - 3  # restored up to the first cut
        assert toks2 == _greedy_direct(model, turn2, 4)
        assert eng.stats["prefix_hits"] == 1
    finally:
        eng.shutdown()


def test_engine_stop_ids_and_cancel(model):
    eng = Engine(RefRunner(model, num_slots=2))
    try:
        prompt = list(range(30))
        ref = _greedy_direct(model, prompt, 8)
        toks, fin = eng.generate(prompt, _params(8, stop_token_ids=[ref[2]]))
        assert fin.reason == "stop" and toks == ref[:3]
        toks, fin = eng.generate(prompt, _params(8, stop_token_ids=[ref[2]], ignore_eos=True))
        assert fin.reason == "length" and toks == ref
    finally:
        eng.shutdown()


def test_engine_poisons_on_device_error(model):
    class Broken(RefRunner):
        def prefill(self, *a, **k):
            raise RuntimeError("CUDA error: an illegal memory access was encountered")

    eng = Engine(Broken(model, num_slots=1))
    req = eng.submit([1, 2, 3], _params(3))
    evs = list(req.iter_events(timeout=60))
    assert isinstance(evs[-1], FinishEvent) and evs[-1].reason == "error"
    assert eng.poisoned and "illegal memory access" in eng.poisoned
    with pytest.raises(Exception):
        eng.submit([1, 2], _params(2))
    eng.shutdown()
