"""Host-side runtime units: sampling precedence, prefix cache, admission control."""
import asyncio

import pytest
import torch

from helexa_b200.runtime.admission import AdmissionConfig, AdmissionController, AdmissionRejection
from helexa_b200.runtime.prefix_cache import PrefixCache, stable_snapshot_cut
from helexa_b200.runtime.sampling import GenerationDefaults, HostSampler, SamplingParams, apply_repeat_penalty


# ---- sampling -------------------------------------------------------------------
def test_sampling_precedence():
    d = GenerationDefaults(temperature=0.6, top_p=0.9, top_k=20, eos_token_ids=[7])
    p = SamplingParams.resolve({"temperature": 0.0, "max_tokens": 5}, d, eos_ids=[3])
    assert p.temperature == 0.0 and p.top_p == 0.9 and p.top_k == 20 and p.max_tokens == 5
    assert p.stop_token_ids == [3, 7]
    p2 = SamplingParams.resolve({}, GenerationDefaults())
    assert p2.temperature == 0.7 and p2.repeat_penalty == 1.1
    p3 = SamplingParams.resolve({"max_completion_tokens": 9, "repetition_penalty": 1.0}, d)
    assert p3.max_tokens == 9 and p3.repeat_penalty == 1.0


def test_repeat_penalty_and_sampler():
    lg = torch.tensor([2.0, -2.0, 1.0, 0.5])
    out = apply_repeat_penalty(lg, [0, 1], 2.0, 64)
    assert out.tolist() == [1.0, -4.0, 1.0, 0.5]
    s = HostSampler(SamplingParams(temperature=0.0, repeat_penalty=1.0))
    assert s.sample(lg, []) == 0
    s = HostSampler(SamplingParams(temperature=1.0, top_k=1, repeat_penalty=1.0, seed=3))
    assert all(s.sample(lg, []) == 0 for _ in range(10))
    s = HostSampler(SamplingParams(temperature=1.0, top_p=0.5, repeat_penalty=1.0, seed=3))
    assert all(s.sample(torch.tensor([5.0, 0.0, 0.0]), []) == 0 for _ in range(10))


# ---- prefix cache -------------------------------------------------------------------
def test_prefix_cache_longest_strict_match_and_ancestors():
    evicted = []
    pc = PrefixCache(budget_bytes=100, max_entries=3, on_evict=evicted.append)
    pc.insert([1, 2], "a", 10)
    pc.insert([1, 2, 3, 4], "b", 10)       # drops its ancestor [1, 2]
    assert evicted == ["a"] and len(pc) == 1
    assert pc.longest_match([1, 2, 3, 4]) is None          # strict prefix only
    assert pc.longest_match([1, 2, 3, 4, 5]).snapshot == "b"
    assert pc.longest_match([9, 9]) is None
    pc.insert([5], "c", 10)
    pc.insert([6], "d", 10)
    pc.insert([7], "e", 10)                 # entry cap 3 -> the least recently used ("b") goes
    assert len(pc) == 3
    assert "b" in evicted and "c" not in evicted
    pc.insert([8], "big", 1000)             # larger than the whole budget: refused
    assert "big" in evicted
    assert pc.remove_covering([6, 1]) == 1


def test_prefix_cache_byte_budget():
    pc = PrefixCache(budget_bytes=25, max_entries=10)
    for i in range(5):
        pc.insert([i], i, 10)
    assert pc.nbytes <= 25 and len(pc) == 2


def test_stable_snapshot_cut():
    assert stable_snapshot_cut([1, 9, 2, 9, 3, 4], 9) == 4
    assert stable_snapshot_cut([1, 2, 3], None) == 2


# ---- admission ------------------------------------------------------------------------
def _run(coro):
    return asyncio.run(coro)


def test_admission_queue_and_timeout():
    async def main():
        ctl = AdmissionController(AdmissionConfig(max_in_flight=1, max_queue_depth=1, max_wait_s=0.2))
        p1 = await ctl.enter("alice")
        waiter = asyncio.create_task(ctl.enter("bob"))
        await asyncio.sleep(0.01)
        assert ctl.queue_depth == 1
        with pytest.raises(AdmissionRejection) as e:
            await ctl.enter("carol")
        assert e.value.reason == "queue_full" and e.value.status == 503 and e.value.retry_after > 0
        with pytest.raises(AdmissionRejection) as e2:
            await waiter
        assert e2.value.reason == "timeout"
        p1.release()
        p2 = await ctl.enter("bob")
        p2.release()
        assert ctl.in_flight == 0 and ctl.rejections.queue_full == 1 and ctl.rejections.timeout == 1
    _run(main())


def test_admission_handoff_and_principal_cap():
    async def main():
        ctl = AdmissionController(AdmissionConfig(max_in_flight=1, max_queue_depth=4, max_wait_s=2,
                                                  max_per_principal=2))
        p1 = await ctl.enter("alice")
        w = asyncio.create_task(ctl.enter("alice"))
        await asyncio.sleep(0.01)
        with pytest.raises(AdmissionRejection) as e:
            await ctl.enter("alice")
        assert e.value.reason == "per_principal" and e.value.status == 429
        p1.release()
        p2 = await w
        assert ctl.in_flight == 1
        p2.release()
    _run(main())


def test_admission_anonymous_yields_to_identified():
    async def main():
        ctl = AdmissionController(AdmissionConfig(max_in_flight=2, max_queue_depth=4, max_wait_s=0.3))
        assert ctl.anon_max_in_flight == 1
        a1 = await ctl.enter(None)
        with pytest.raises(AdmissionRejection) as e:  # anonymous seat ceiling reached
            await ctl.enter(None)
        assert e.value.reason in ("anon_yield", "timeout")
        i1 = await ctl.enter("id")                     # identified takes the held-back seat
        a1.release()
        i1.release()
    _run(main())


def test_admission_kv_budget_and_close():
    async def main():
        ctl = AdmissionController(AdmissionConfig(max_in_flight=4, max_queue_depth=4, kv_max_wait_s=0.2))
        ctl.set_kv_budget_mb(100)
        with pytest.raises(AdmissionRejection) as e:
            await ctl.enter("x", kv_mb=200)
        assert e.value.reason == "kv_unservable" and e.value.retry_after == 0
        p = await ctl.enter("x", kv_mb=80)
        assert ctl.kv_available_mb() == 20
        with pytest.raises(AdmissionRejection) as e2:
            await ctl.enter("y", kv_mb=50)
        assert e2.value.reason == "kv_timeout"
        p.release()
        ctl.close()
        with pytest.raises(AdmissionRejection) as e3:
            await ctl.enter("z")
        assert e3.value.reason == "closed"
    _run(main())
