"""Fused GEMV tails: router softmax/top-k and lm_head arg-max with step bookkeeping."""
import pytest
import torch

from helexa_b200.models import reference as R

pytestmark = pytest.mark.gpu


def _C():
    from helexa_b200 import ops
    return ops.C


def _close(a, b, tol):
    err = (a.float() - b.float()).abs().max().item()
    assert err <= tol * (b.float().abs().max().item() + 1e-6), err


@pytest.mark.parametrize("B", [1, 2, 4])
def test_router_tail(B):
    C = _C()
    torch.manual_seed(3)
    E, k, H = 512, 10, 2048
    router = (torch.randn(E + 1, H, device="cuda") * 0.05).bfloat16()
    x = torch.randn(B, H, device="cuda").bfloat16()
    nw = torch.rand(H, device="cuda") + 0.5
    logits = torch.zeros(B, E + 1, device="cuda")
    ids = torch.zeros(B, k + 1, dtype=torch.int32, device="cuda")
    wts = torch.zeros(B, k + 1, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    for _ in range(2):  # the election counter must reset itself
        C.gemv_router(router, x, logits, nw, 1e-6, E, k, True, True, ids, wts, cnt)
    torch.cuda.synchronize()
    xn = R.rms_norm(x, nw, 1e-6, 0.0).bfloat16().float()
    lg = xn @ router.float().t()
    _close(logits, lg, 1e-3)
    p = torch.softmax(logits[:, :E], -1)
    tv, ti = torch.topk(p, k, -1)
    assert torch.equal(ids[:, :k].long(), ti)
    _close(wts[:, :k], tv / tv.sum(-1, keepdim=True), 1e-4)
    _close(wts[:, k], torch.sigmoid(logits[:, E]), 1e-4)
    assert (ids[:, k] == E).all() and int(cnt) == 0


@pytest.mark.parametrize("B", [1, 4])
def test_lm_head_argmax_tail(B):
    C = _C()
    torch.manual_seed(4)
    V, H = 151936, 2048
    W = (torch.randn(V, H, device="cuda") * 0.05).bfloat16()
    x = torch.randn(B, H, device="cuda").bfloat16()
    nw = torch.rand(H, device="cuda") + 0.5
    best = torch.zeros(B, dtype=torch.int64, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    tok = torch.zeros(B, dtype=torch.int32, device="cuda")
    slots = torch.arange(B, dtype=torch.int32, device="cuda").flip(0).contiguous()
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = torch.zeros(B, 16, dtype=torch.int32, device="cuda")
    step = torch.zeros(B, dtype=torch.int32, device="cuda")
    logits = torch.empty(B, V, device="cuda")
    for rep in range(2):
        C.gemv_argmax(W, x, logits, nw, 1e-6, best, cnt, tok, slots, pos, out, step)
    torch.cuda.synchronize()
    xn = R.rms_norm(x, nw, 1e-6, 0.0).bfloat16().float()
    _close(logits, xn @ W.float().t(), 1e-3)
    assert torch.equal(tok.long(), logits.argmax(-1))
    assert pos.tolist() == [2] * B and step.tolist() == [2] * B
    assert torch.equal(out[:, 0], tok) and torch.equal(out[:, 1], tok)
    assert int(cnt) == 0 and int(best.abs().sum()) == 0
    # ties resolve to the lowest index
    W2 = torch.zeros(64, H, device="cuda").bfloat16()
    C.gemv_argmax(W2, x, None, nw, 1e-6, best, cnt, tok, None, None, None, None)
    torch.cuda.synchronize()
    assert tok.tolist() == [0] * B
