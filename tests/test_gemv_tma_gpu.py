"""The bulk-copy (TMA ring) decode GEMV engine against plain PyTorch fp32 references:
dense modes over batch sizes and row lengths (warp-per-row and split-K tiles), MoE
expert gate/up with SwiGLU (and expert-parallel skipping), the MoE down projection with
the weighted combine, the fused lm_head arg-max, and the single-rank exchange path."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from helexa_b200 import ops
    return ops.C


def _close(a, b, tol):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    assert err <= tol * max(1.0, b.abs().max().item()), err


def _err():
    return torch.zeros(1, dtype=torch.int32, device="cuda")


@pytest.mark.parametrize("B,N,K", [(1, 12352, 2048), (1, 2048, 4096), (2, 1000, 512), (3, 2048, 2048),
                                   (8, 4096, 1024), (1, 256, 12288), (1, 77, 25600)])
def test_dense_modes(B, N, K):
    from helexa_b200 import ops
    C = _C()
    torch.manual_seed(0)
    assert C.gemv_tma_ok(N, K, B, 1)
    W = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    x = torch.randn(B, K, device="cuda").bfloat16()
    nw = torch.rand(K, device="cuda") + 0.5
    err = _err()
    xn = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * nw).bfloat16()
    ref = xn.float() @ W.float().t()
    y = torch.empty(B, N, device="cuda").bfloat16()
    C.gemv_tma(W, x, y, ops.STORE_BF16, None, nw, 1e-6, err)
    _close(y, ref, 2e-2)
    yf = torch.empty(B, N, device="cuda")
    C.gemv_tma(W, x, yf, ops.STORE_F32, None, None, 0.0, err)
    _close(yf, x.float() @ W.float().t(), 1e-2)
    res = torch.randn(B, N, device="cuda").bfloat16()
    r2 = res.clone()
    C.gemv_tma(W, x, r2, ops.RESID_ADD, r2, None, 0.0, err)
    _close(r2, res.float() + x.float() @ W.float().t(), 2e-2)
    if N % 2 == 0:
        act = torch.empty(B, N // 2, device="cuda").bfloat16()
        C.gemv_tma(W, x, act, ops.SILU_PAIR, None, None, 0.0, err)
        full = x.float() @ W.float().t()
        _close(act, torch.nn.functional.silu(full[:, 0::2]) * full[:, 1::2], 3e-2)
    torch.cuda.synchronize()
    assert int(err.item()) == 0


@pytest.mark.parametrize("B,ep", [(1, False), (2, False), (1, True)])
def test_experts_and_moe_down(B, ep):
    C = _C()
    torch.manual_seed(1)
    E, k, H, I = 16, 10, 2048, 512
    J = k + 1
    Wgu = (torch.randn(E + 1, 2 * I, H, device="cuda") * 0.05).bfloat16()
    Wd = (torch.randn(E + 1, H, I, device="cuda") * 0.05).bfloat16()
    x = torch.randn(B, H, device="cuda").bfloat16()
    nw = torch.rand(H, device="cuda") + 0.5
    ids = torch.stack([torch.cat([torch.randperm(E)[:k], torch.tensor([E])]) for _ in range(B)]).int().cuda()
    wts = torch.rand(B, J, device="cuda")
    err = _err()
    e_base, e_count = (4, 8) if ep else (0, 0)
    Wgu_l = Wgu[e_base:e_base + e_count].contiguous() if ep else Wgu
    Wd_l = Wd[e_base:e_base + e_count].contiguous() if ep else Wd
    act = torch.zeros(B * J, I, device="cuda").bfloat16()
    C.gemv_tma_experts(Wgu_l, x, ids.view(-1), act, 2, J, nw, 1e-6, e_base, e_count, err)
    xn = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * nw).bfloat16().float()
    local = lambda e: (not ep) or (e_base <= e < e_base + e_count)  # noqa: E731
    for b in range(B):
        for j in range(J):
            e = int(ids[b, j])
            if not local(e):
                continue
            full = Wgu[e].float() @ xn[b]
            want = torch.nn.functional.silu(full[0::2].bfloat16().float()) * full[1::2].bfloat16().float()
            _close(act[b * J + j], want, 3e-2)
    x0 = torch.randn(B, H, device="cuda").bfloat16()
    xo = x0.clone()
    C.moe_down_tma(Wd_l, act, ids, wts, xo, None, e_base, e_count, err)
    want = x0.float().clone()
    for b in range(B):
        for j in range(J):
            e = int(ids[b, j])
            if local(e):
                a = (act[b * J + j].float() * wts[b, j]).bfloat16().float()
                want[b] += Wd[e].float() @ a
    _close(xo, want, 3e-2)
    part = torch.empty(B, H, device="cuda").bfloat16()
    C.moe_down_tma(Wd_l, act, ids, wts, x0, part, e_base, e_count, err)
    _close(part, want - x0.float(), 3e-2)
    torch.cuda.synchronize()
    assert int(err.item()) == 0


@pytest.mark.parametrize("B", [1, 3])
def test_argmax_step(B):
    C = _C()
    torch.manual_seed(2)
    V, K = 151936, 2048
    W = (torch.randn(V, K, device="cuda") * 0.05).bfloat16()
    x = torch.randn(B, K, device="cuda").bfloat16()
    nw = torch.rand(K, device="cuda") + 0.5
    best = torch.zeros(B, dtype=torch.int64, device="cuda")
    cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
    tok = torch.zeros(B, dtype=torch.int32, device="cuda")
    slots = torch.arange(B, dtype=torch.int32, device="cuda")
    pos = torch.zeros(B, dtype=torch.int32, device="cuda")
    out = torch.zeros(B, 4, dtype=torch.int32, device="cuda")
    step = torch.zeros(B, dtype=torch.int32, device="cuda")
    lg = torch.empty(B, V, device="cuda")
    err = _err()
    for it in range(2):  # self-resetting counters: a second call works the same
        C.gemv_tma_argmax(W, x, lg, nw, 1e-6, best, cnt, tok, slots, pos, out, step, 0, err)
        torch.cuda.synchronize()
        assert torch.equal(tok.long(), lg.argmax(-1))
        assert step.tolist() == [it + 1] * B and pos.tolist() == [it + 1] * B
    xn = (x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * nw).bfloat16()
    _close(lg, xn.float() @ W.float().t(), 1e-2)
    assert int(err.item()) == 0 and int(cnt.item()) == 0 and best.abs().sum() == 0


def test_single_rank_exchange_paths():
    from helexa_b200 import ops
    C = _C()
    torch.manual_seed(3)
    words = 8 * 4096
    reg, _ = C.ipc_alloc(2 * words * 8, 0)
    ctr = torch.zeros(2, dtype=torch.int32, device="cuda")
    err = _err()
    N, K = 2048, 1024
    W = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    for call in range(3):
        x = torch.randn(2, K, device="cuda").bfloat16()
        res = torch.randn(2, N, device="cuda").bfloat16()
        want = res.clone()
        C.gemv(W, x, want, ops.RESID_ADD, want, None, 0.0)
        got = res.clone()
        C.gemv_tma_ar(W, x, got, [reg.data_ptr()], 0, words, ctr, err, 1.0)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        _close(got, want.float(), 1e-2)
    assert int(ctr[0].item()) == 3 and int(ctr[1].item()) == 0


def test_missing_peer_times_out():
    C = _C()
    words = 8 * 4096
    mine, _ = C.ipc_alloc(2 * 2 * words * 8, 0)
    ghost, _ = C.ipc_alloc(2 * 2 * words * 8, 0)
    ctr = torch.zeros(2, dtype=torch.int32, device="cuda")
    err = _err()
    W = (torch.randn(2048, 512, device="cuda") * 0.05).bfloat16()
    x = torch.randn(1, 512, device="cuda").bfloat16()
    res = torch.randn(1, 2048, device="cuda").bfloat16()
    out = res.clone()
    C.gemv_tma_ar(W, x, out, [mine.data_ptr(), ghost.data_ptr()], 0, words, ctr, err, 0.005)
    torch.cuda.synchronize()
    assert int(err.item()) == 2001 and torch.equal(out, res)
