"""Token-exact greedy parity of the reference model against HF transformers (CPU fp32).

Mirrors the reference's tiny Qwen3-Next parity test (crates/neuron/tests/qwen3_next_parity.rs)
on the benchmark's tiny config: hidden 256, [GDN x3, attention], 8 experts top-2 + shared.
"""
import pytest
import torch

from helexa_b200.config import get_preset
from helexa_b200.models.hf_oracle import build_hf_model, hf_greedy
from helexa_b200.models.reference import (ReferenceModel, delta_rule_chunked,
                                          delta_rule_recurrent, l2norm)
from helexa_b200.weights.random_init import random_weights


def _greedy(model, prompt, n):
    st = model.new_state()
    lg = model.forward(torch.tensor(prompt), st)
    out = []
    for _ in range(n):
        t = int(lg.argmax())
        out.append(t)
        lg = model.forward(torch.tensor([t]), st)
    return out


@pytest.mark.parametrize("name", ["tiny-qwen3-next", "tiny-qwen3", "tiny-qwen3-moe", "tiny-llama"])
def test_greedy_matches_hf(name):
    cfg = get_preset(name)
    w = random_weights(cfg, seed=0)
    g = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab_size, (32,), generator=g).tolist()
    hf = build_hf_model(cfg, w)
    want, margins = hf_greedy(hf, prompt, 16)
    got = _greedy(ReferenceModel(cfg, w), prompt, 16)
    # a step whose top-2 margin is under fp32 noise may legitimately flip; none do here
    for i, (a, b) in enumerate(zip(want, got)):
        if a != b:
            assert margins[i] < 1e-5, f"step {i}: {a} vs {b} with margin {margins[i]}"
            break


def test_chunked_delta_rule_matches_recurrent():
    torch.manual_seed(0)
    T, H, Dk, Dv = 150, 3, 16, 24
    q = l2norm(torch.randn(T, H, Dk)) * Dk ** -0.5
    # adversarial: strongly correlated keys (small perturbations of one direction)
    base = torch.randn(1, H, Dk)
    k = l2norm(base + 0.05 * torch.randn(T, H, Dk))
    v = torch.randn(T, H, Dv)
    g = -torch.rand(T, H) * 0.5
    beta = torch.rand(T, H)
    s0 = torch.randn(H, Dk, Dv) * 0.1
    o1, s1 = delta_rule_recurrent(q, k, v, g, beta, s0)
    o2, s2 = delta_rule_chunked(q, k, v, g, beta, s0, chunk=64)
    assert torch.allclose(o1, o2, atol=2e-4, rtol=1e-3)
    assert torch.allclose(s1, s2, atol=2e-4, rtol=1e-3)


def test_chunked_prefill_carries_conv_state():
    """Prefill in two chunks must equal one-shot prefill (conv state carried across)."""
    cfg = get_preset("tiny-qwen3-next")
    w = random_weights(cfg, seed=1)
    m = ReferenceModel(cfg, w, gdn_chunk_threshold=16)
    prompt = torch.randint(0, cfg.vocab_size, (100,), generator=torch.Generator().manual_seed(3))
    s1 = m.new_state()
    full = m.forward(prompt, s1)
    s2 = m.new_state()
    m.forward(prompt[:37], s2)
    part = m.forward(prompt[37:], s2)
    assert torch.allclose(full, part, atol=1e-4), (full - part).abs().max()
