"""The single-launch decode MoE block (router, top-k, experts, down, combine and the
fused cross-rank sum with grid barriers) against the three-kernel path, on random
weights: single rank, expert-parallel skipping, a one-rank exchange, batch > 1, and a
whole CUDA model decoding through it inside a captured graph."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(a, b, tol):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    assert err <= tol * max(1.0, b.abs().max().item()), err


def _weights(E, H, I, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    r = lambda *s: (torch.randn(*s, device="cuda", generator=g) * 0.05).bfloat16()  # noqa: E731
    router = r(E + 1, H)
    router[:E] *= 20  # decisive routing so both paths pick the same experts
    return router, r(E + 1, 2 * I, H), r(E + 1, H, I)


@pytest.mark.parametrize("B,E,k,H,I", [(1, 64, 6, 2048, 512), (3, 32, 4, 1024, 256), (8, 16, 2, 512, 128)])
def test_moe_fused_matches_three_kernels(B, E, k, H, I):
    from helexa_b200 import ops
    C = ops.C
    router, w_gu, w_d = _weights(E, H, I, 0)
    J = k + 1
    ln2 = torch.rand(H, device="cuda") + 0.5
    x = torch.randn(B, H, device="cuda").bfloat16()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    # three-kernel path
    rl = torch.zeros(B, E + 1, device="cuda")
    ids = torch.zeros(B, J, dtype=torch.int32, device="cuda")
    wts = torch.zeros(B, J, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    act = torch.zeros(B * J, I, device="cuda").bfloat16()
    want = x.clone()
    C.gemv_router(router, want, rl, ln2, 1e-6, E, k, True, True, ids, wts, cnt)
    C.gemv_experts(w_gu, want, ids.view(-1), act, ops.SILU_PAIR, J, ln2, 1e-6)
    C.moe_down(w_d, act, ids, wts, want, None)
    # fused
    got = x.clone()
    rl2 = torch.zeros(B, E + 1, device="cuda")
    act2 = torch.zeros(B * J, I, device="cuda").bfloat16()
    bar = torch.zeros(4, dtype=torch.int32, device="cuda")
    for _ in range(3):  # repeated calls: barrier epochs advance
        got = x.clone()
        C.moe_fused(got, ln2, 1e-6, router, w_gu, w_d, E, k, True, True, rl2, act2, bar, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and int(bar[1].item()) == 3
    _close(rl2, rl, 1e-3)
    _close(got, want, 2e-2)


def test_moe_fused_expert_parallel_and_single_rank_exchange():
    from helexa_b200 import ops
    C = ops.C
    B, E, k, H, I = 2, 32, 4, 1024, 256
    router, w_gu, w_d = _weights(E, H, I, 1)
    J = k
    ln2 = torch.rand(H, device="cuda") + 0.5
    x = torch.randn(B, H, device="cuda").bfloat16()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    e0, ne = 8, 8
    wgu_l, wd_l = w_gu[e0:e0 + ne].contiguous(), w_d[e0:e0 + ne].contiguous()
    # reference: only the local experts' routes contribute
    rl = torch.zeros(B, E, device="cuda")
    ids = torch.zeros(B, J, dtype=torch.int32, device="cuda")
    wts = torch.zeros(B, J, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    act = torch.zeros(B * J, I, device="cuda").bfloat16()
    want = x.clone()
    C.gemv_router(router[:E].contiguous(), want, rl, ln2, 1e-6, E, k, False, True, ids, wts, cnt)
    C.gemv_experts_ep(wgu_l, want, ids.view(-1), act, ops.SILU_PAIR, J, ln2, 1e-6, e0)
    words = 8 * 4096
    reg, _ = C.ipc_alloc(2 * words * 8, 0)
    ctr = torch.zeros(2, dtype=torch.int32, device="cuda")
    C.moe_down_ar_ep(wd_l, act, ids, wts, want, [reg.data_ptr()], 0, words, ctr, err, 1.0, e0)
    got = x.clone()
    rl2 = torch.zeros(B, E, device="cuda")
    act2 = torch.zeros(B * J, I, device="cuda").bfloat16()
    bar = torch.zeros(4, dtype=torch.int32, device="cuda")
    C.moe_fused(got, ln2, 1e-6, router[:E].contiguous(), wgu_l, wd_l, E, k, False, True, rl2, act2, bar, err, e0, ne,
                [reg.data_ptr()], 0, words, ctr, 1.0)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and int(ctr[0].item()) == 2
    _close(got, want, 2e-2)


def test_model_decodes_through_fused_moe_in_a_graph(monkeypatch):
    from helexa_b200.config import get_preset
    from helexa_b200.models.fast import FastModel
    from helexa_b200.weights.random_init import random_weights
    from test_fast_model_gpu import _realistic
    cfg = get_preset("tiny-qwen3-next")
    torch.manual_seed(0)
    w = _realistic(cfg, random_weights(cfg, seed=0, std=0.05))
    outs = []
    for fused in ("1", "0"):
        monkeypatch.setenv("HELEXA_MOE_FUSED", fused)  # the fused kernel is opt-in
        fm = FastModel.from_hf(cfg, w, "cuda", max_slots=1, max_len=256)
        assert fm.moe_fused == (fused == "1")
        prompt = torch.arange(40, dtype=torch.int32, device="cuda") * 7 % cfg.vocab_size
        lg = fm.prefill(0, prompt, 0)
        nb = fm.capture(1, steps=8)
        nb.slots.fill_(0)
        nb.tok.fill_(int(lg.argmax()))
        fm.replay(nb)
        torch.cuda.synchronize()
        assert fm.device_error() == 0
        outs.append((nb.out_tokens[0, :8].tolist(), nb.logits[0].clone()))
    assert outs[0][0] == outs[1][0]
    cos = torch.nn.functional.cosine_similarity(outs[0][1], outs[1][1], dim=0).item()
    assert cos > 0.999, cos
