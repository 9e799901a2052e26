"""Streaming decode GEMV (csrc/sgemv.cu), every mode against fp32 torch references."""
import pytest
import torch

from helexa_b200.models import reference as R

pytestmark = pytest.mark.gpu


def _ops():
    from helexa_b200 import ops
    return ops


def _close(a, b, tol):
    err = (a.float() - b.float()).abs().max().item()
    assert err <= tol * (b.float().abs().max().item() + 1e-6), err


def _err():
    return torch.zeros(1, dtype=torch.int32, device="cuda")


@pytest.mark.parametrize("B", [1, 2, 4, 8])
@pytest.mark.parametrize("N,K", [(12352, 2048), (2048, 4096), (100, 256), (4096, 12288)])
def test_sgemv_dense_modes(B, N, K):
    ops = _ops()
    if not ops.sgemv_fits(ops.SG_STORE, K, B):
        pytest.skip("activations do not fit the shared-memory ring; the model uses the register GEMV")
    g = torch.Generator(device="cuda").manual_seed(0)
    W = (torch.randn(N, K, device="cuda", generator=g) * 0.05).bfloat16()
    x = torch.randn(B, K, device="cuda", generator=g).bfloat16()
    nw = torch.rand(K, device="cuda", generator=g) + 0.5
    e = _err()
    xn = R.rms_norm(x, nw, 1e-6, 0.0).bfloat16().float()
    ref = xn @ W.float().t()
    y = torch.empty(B, N, device="cuda", dtype=torch.bfloat16)
    ops.sgemv(ops.SG_STORE, W, x, y, norm=nw, eps=1e-6, err=e)
    _close(y, ref, 1e-2)
    yf = torch.empty(B, N, device="cuda")
    ops.sgemv(ops.SG_F32, W, x, yf, err=e)
    _close(yf, x.float() @ W.float().t(), 1e-3)
    res = torch.randn(B, N, device="cuda", generator=g).bfloat16()
    r2 = res.clone()
    ops.sgemv(ops.SG_RESID, W, x, r2, resid=r2, err=e)
    _close(r2, res.float() + x.float() @ W.float().t(), 2e-2)
    if N % 2 == 0:
        act = torch.empty(B, N // 2, device="cuda", dtype=torch.bfloat16)
        ops.sgemv(ops.SG_SILU, W, x, act, err=e)
        rr = x.float() @ W.float().t()
        _close(act, torch.nn.functional.silu(rr[:, 0::2]) * rr[:, 1::2], 3e-2)
    torch.cuda.synchronize()
    assert int(e) == 0


@pytest.mark.parametrize("B", [1, 2])
def test_sgemv_moe_router_experts_down(B):
    ops = _ops()
    torch.manual_seed(3)
    E, k, H, I = 64, 6, 1024, 256
    J = k + 1
    router = (torch.randn(E + 1, H, device="cuda") * 0.05).bfloat16()
    wgu = (torch.randn(E + 1, 2 * I, H, device="cuda") * 0.05).bfloat16()
    wd = (torch.randn(E + 1, H, I, device="cuda") * 0.05).bfloat16()
    x = torch.randn(B, H, device="cuda").bfloat16()
    nw = torch.rand(H, device="cuda") + 0.5
    e = _err()
    scratch = torch.zeros(B, E + 1, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    ids = torch.zeros(B, J, dtype=torch.int32, device="cuda")
    wts = torch.zeros(B, J, device="cuda")
    for rep in range(2):
        ops.sgemv(ops.SG_ROUTER, router, x, norm=nw, eps=1e-6, scratch=scratch, counter=cnt, out_ids=ids,
                  out_wts=wts, E=E, topk=k, shared=True, norm_topk=True, err=e)
    xn = R.rms_norm(x, nw, 1e-6, 0.0).bfloat16().float()
    lg = xn @ router.float().t()
    p = torch.softmax(lg[:, :E], -1)
    tv, ti = torch.topk(p, k, -1)
    assert torch.equal(ids[:, :k].long(), ti)
    _close(wts[:, :k], tv / tv.sum(-1, keepdim=True), 1e-3)
    _close(wts[:, k], torch.sigmoid(lg[:, E]), 1e-3)
    assert (ids[:, k] == E).all() and int(cnt) == 0
    act = torch.empty(B * J, I, device="cuda", dtype=torch.bfloat16)
    ops.sgemv(ops.SG_EXPERT, wgu, x, act, norm=nw, eps=1e-6, ids=ids.view(-1), J=J, err=e)
    for b in range(B):
        for j in range(J):
            y = xn[b] @ wgu[ids[b, j]].float().t()
            _close(act[b * J + j], torch.nn.functional.silu(y[0::2]) * y[1::2], 3e-2)
    xr = torch.randn(B, H, device="cuda").bfloat16()
    want = xr.float().clone()
    for b in range(B):
        for j in range(J):
            want[b] += wts[b, j] * (wd[ids[b, j]].float() @ act[b * J + j].float())
    ops.sgemv(ops.SG_MOEDOWN, wd, act, xr, resid=xr, ids=ids, wts=wts, J=J, err=e)
    _close(xr, want, 3e-2)
    torch.cuda.synchronize()
    assert int(e) == 0


@pytest.mark.parametrize("B", [1, 4])
def test_sgemv_lm_head_argmax(B):
    ops = _ops()
    torch.manual_seed(4)
    V, H = 151936, 2048
    W = (torch.randn(V, H, device="cuda") * 0.05).bfloat16()
    x = torch.randn(B, H, device="cuda").bfloat16()
    nw = torch.rand(H, device="cuda") + 0.5
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    amax = torch.zeros(sms * B * 2, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    tok = torch.zeros(B, dtype=torch.int32, device="cuda")
    slots = torch.arange(B, dtype=torch.int32, device="cuda")
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = torch.zeros(B, 16, dtype=torch.int32, device="cuda")
    step = torch.zeros(B, dtype=torch.int32, device="cuda")
    logits = torch.empty(B, V, device="cuda")
    e = _err()
    ops.sgemv(ops.SG_ARGMAX, W, x, logits, norm=nw, eps=1e-6, scratch=amax, counter=cnt, tok=tok, slots=slots,
              pos=pos, out_tokens=out, step=step, err=e)
    torch.cuda.synchronize()
    xn = R.rms_norm(x, nw, 1e-6, 0.0).bfloat16().float()
    ref = xn @ W.float().t()
    _close(logits, ref, 1e-3)
    assert torch.equal(tok.long(), logits.argmax(-1))
    assert pos.tolist() == [1] * B and step.tolist() == [1] * B and torch.equal(out[:, 0], tok)
    assert int(cnt) == 0 and int(e) == 0
