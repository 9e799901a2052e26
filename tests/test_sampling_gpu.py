"""The on-device sampler (csrc/sample_device.cu) against the host sampler's semantics:
greedy with repeat penalty, top-k = 1, empirical frequencies of temperature / top-k /
top-p draws against the renormalised softmax, seeded reproducibility, and the
sampled-decode graph of FastRunner against the host-sampled path."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _state(S, V, temp=1.0, top_k=0, top_p=1.0, penalty=1.0, seed=7):
    d = "cuda"
    return dict(temp=torch.full((S,), temp, device=d), top_k=torch.full((S,), top_k, dtype=torch.int32, device=d),
                top_p=torch.full((S,), top_p, device=d), penalty=torch.full((S,), penalty, device=d),
                seed=torch.full((S,), seed, dtype=torch.int64, device=d),
                ctr=torch.arange(S, dtype=torch.int64, device=d),
                hist=torch.zeros(S, 64, dtype=torch.int32, device=d), hist_n=torch.zeros(S, dtype=torch.int32, device=d),
                hist_at=torch.zeros(S, dtype=torch.int32, device=d),
                hist_cap=torch.full((S,), 64, dtype=torch.int32, device=d))


def _draw(logits_row, st, S):
    from helexa_b200 import ops
    V = logits_row.numel()
    lg = logits_row[None].repeat(S, 1).contiguous()
    slots = torch.arange(S, dtype=torch.int32, device="cuda")
    tok = torch.zeros(S, dtype=torch.int32, device="cuda")
    pos = torch.zeros(S, dtype=torch.int32, device="cuda")
    out = torch.zeros(S, 4, dtype=torch.int32, device="cuda")
    step = torch.zeros(S, dtype=torch.int32, device="cuda")
    ops.C.sample_step(lg, V, slots, st["temp"], st["top_k"], st["top_p"], st["penalty"], st["seed"], st["ctr"],
                      st["hist"], st["hist_n"], st["hist_at"], st["hist_cap"], tok, pos, out, step)
    torch.cuda.synchronize()
    assert torch.equal(out[:, 0], tok) and pos.tolist() == [1] * S
    return tok.long().cpu()


def test_greedy_with_penalty_and_topk1():
    torch.manual_seed(0)
    V = 5000
    lg = torch.randn(V, device="cuda")
    lg[17] = 10.0
    lg[23] = 9.5
    st = _state(1, V, temp=0.0, penalty=1.5)
    st["hist"][0, :3] = torch.tensor([17, 17, 4], dtype=torch.int32)
    st["hist_n"][0] = 3
    st["hist_at"][0] = 3
    # 17 is penalised once (10 / 1.5 < 9.5): the arg-max moves to 23
    assert int(_draw(lg, st, 1)[0]) == 23
    assert int(st["hist"][0, 3]) == 23 and int(st["hist_n"][0]) == 4
    st1 = _state(8, V, temp=0.8, top_k=1)
    assert (_draw(lg, st1, 8) == 17).all()


@pytest.mark.parametrize("top_k,top_p", [(0, 1.0), (3, 1.0), (0, 0.6), (5, 0.7)])
def test_frequencies_match_renormalised_softmax(top_k, top_p):
    torch.manual_seed(1)
    V, T, S = 12, 0.7, 4096
    lg = torch.randn(V, device="cuda") * 1.5
    probs = torch.softmax(lg.double().cpu() / T, -1)
    order = torch.argsort(probs, descending=True)
    keep = torch.zeros(V, dtype=torch.bool)
    if top_k:
        keep[order[:top_k]] = True
    else:
        keep[:] = True
    kept = probs * keep
    kept = kept / kept.sum()
    if top_p < 1.0:
        sp = kept[order]
        cum = torch.cumsum(sp, 0)
        k2 = torch.zeros(V, dtype=torch.bool)
        k2[order[(cum - sp) < top_p]] = True
        kept = kept * k2
        kept = kept / kept.sum()
    counts = torch.zeros(V)
    for rep in range(5):
        st = _state(S, V, temp=T, top_k=top_k, top_p=top_p, seed=100 + rep)
        t = _draw(lg, st, S)
        counts += torch.bincount(t, minlength=V).float()
    freq = counts / counts.sum()
    assert (freq[kept == 0] == 0).all(), (freq, kept)
    assert (freq - kept.float()).abs().max().item() < 0.02, (freq, kept)


def test_seeded_draws_repeat_and_large_vocab():
    torch.manual_seed(2)
    V = 151936
    lg = torch.randn(V, device="cuda") * 3
    a = _draw(lg, _state(16, V, temp=1.0, top_k=50, top_p=0.9, seed=5), 16)
    b = _draw(lg, _state(16, V, temp=1.0, top_k=50, top_p=0.9, seed=5), 16)
    assert torch.equal(a, b)
    top50 = set(torch.topk(lg, 50).indices.tolist())
    assert set(a.tolist()) <= top50


def test_fast_runner_sampled_graph_matches_host_penalised_greedy():
    from helexa_b200.config import get_preset
    from helexa_b200.models.fast import FastModel
    from helexa_b200.runtime.runner import FastRunner
    from helexa_b200.runtime.sampling import HostSampler, SamplingParams
    from helexa_b200.weights.random_init import random_weights
    cfg = get_preset("tiny-qwen3-next")
    fm = FastModel.from_hf(cfg, random_weights(cfg, seed=0, std=0.05), "cuda", max_slots=4, max_len=256)
    r = FastRunner(fm, graph_steps=4)
    prompt = torch.randint(0, cfg.vocab_size, (30,), generator=torch.Generator().manual_seed(3)).tolist()
    p = SamplingParams(temperature=0.0, repeat_penalty=1.3, repeat_last_n=64)
    r.reset(0)
    lg = r.prefill(0, prompt, 0)
    snap = r.snapshot(0, 30)
    hs = HostSampler(p)
    first = hs.sample(lg, prompt)
    hist = prompt + [first]
    dev = r.decode_sampled([0], [first], 6, [p], [hist], [0], [1])[0]
    r.reset(1)
    r.restore(1, snap)
    host, cur, h = [], first, list(hist)
    for _ in range(6):
        row = r.decode_logits([1], [cur])[0]
        cur = hs.sample(row, h)
        h.append(cur)
        host.append(cur)
    assert dev == host, (dev, host)
