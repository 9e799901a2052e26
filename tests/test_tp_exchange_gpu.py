"""The fused decode exchange on one GPU.

(1) With one rank the kernels still run the whole exchange protocol (store the
(epoch, value) words, poll them, advance the call epoch), so repeated calls must match
the plain residual GEMV / MoE down / arg-max, across both receive parities.
(2) Bounded waits: a second "peer" region on the same GPU whose words nothing ever
writes stands in for a rank that never arrives. The kernel must give up after the
timeout, record 2000 + peer (fused path) or 1000 + peer (one-shot kernel), skip the
reduction, return, and make the next call return at once; the host then raises.
No kernel waits on another launch: the missing peer is simply memory nobody writes.
"""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from helexa_b200 import ops
    return ops.C


def _region(C, words):
    t, _ = C.ipc_alloc(2 * 2 * words * 8, 0)
    return t


def _tp_args(C, bases, rank, words, timeout_s):
    ctr = torch.zeros(2, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    return [bases, rank, words, ctr, err, timeout_s], err, ctr


def test_single_rank_exchange_matches_plain_kernels():
    from helexa_b200 import ops
    C = _C()
    torch.manual_seed(0)
    words = 8 * 4096
    reg = _region(C, words)
    args, err, ctr = _tp_args(C, [reg.data_ptr()], 0, words, 1.0)
    N, K = 2048, 1024
    W = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    for call in range(5):  # odd and even epochs: both receive parities
        B = 1 + call % 3
        x = torch.randn(B, K, device="cuda").bfloat16()
        res = torch.randn(B, N, device="cuda").bfloat16()
        want = res.clone()
        C.gemv(W, x, want, ops.RESID_ADD, want, None, 0.0)
        got = res.clone()
        C.gemv_ar(W, x, got, *args)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(got, want), (call, (got.float() - want.float()).abs().max())
    assert int(ctr[0].item()) == 5 and int(ctr[1].item()) == 0
    # MoE down with the exchange
    E, k, H, I, B = 16, 4, 512, 256, 2
    Wd = (torch.randn(E, H, I, device="cuda") * 0.05).bfloat16()
    act = torch.randn(B * k, I, device="cuda").bfloat16()
    ids = torch.randint(0, E, (B, k), dtype=torch.int32, device="cuda")
    wts = torch.rand(B, k, device="cuda")
    x0 = torch.randn(B, H, device="cuda").bfloat16()
    want, got = x0.clone(), x0.clone()
    C.moe_down(Wd, act, ids, wts, want, None)
    C.moe_down_ar(Wd, act, ids, wts, got, *args)
    torch.cuda.synchronize()
    assert int(err.item()) == 0 and torch.equal(got, want)
    # vocab-parallel arg-max with one slice = the plain fused arg-max
    V = 4096
    Wl = (torch.randn(V, K, device="cuda") * 0.05).bfloat16()
    nw = torch.rand(K, device="cuda") + 0.5
    xb = torch.randn(2, K, device="cuda").bfloat16()
    outs = []
    for fn in ("plain", "tp"):
        best = torch.zeros(2, dtype=torch.int64, device="cuda")
        cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
        tok = torch.zeros(2, dtype=torch.int32, device="cuda")
        slots = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
        pos = torch.zeros(2, dtype=torch.int32, device="cuda")
        ot = torch.zeros(2, 4, dtype=torch.int32, device="cuda")
        st = torch.zeros(2, dtype=torch.int32, device="cuda")
        lg = torch.zeros(2, V, device="cuda")
        if fn == "plain":
            C.gemv_argmax(Wl, xb, lg, nw, 1e-6, best, cnt, tok, slots, pos, ot, st)
        else:
            C.gemv_argmax_tp(Wl, xb, lg, nw, 1e-6, best, cnt, tok, slots, pos, ot, st, 0, *args)
        torch.cuda.synchronize()
        outs.append((tok.tolist(), pos.tolist(), ot[:, 0].tolist(), lg.argmax(-1).tolist()))
    assert int(err.item()) == 0
    assert outs[0] == outs[1] and outs[0][0] == outs[0][3]


def test_missing_peer_times_out_and_poisons():
    C = _C()
    torch.manual_seed(1)
    words = 8 * 4096
    mine, ghost = _region(C, words), _region(C, words)
    args, err, _ = _tp_args(C, [mine.data_ptr(), ghost.data_ptr()], 0, words, 0.005)
    N, K = 1024, 512
    W = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    x = torch.randn(1, K, device="cuda").bfloat16()
    res = torch.randn(1, N, device="cuda").bfloat16()
    out = res.clone()
    C.gemv_ar(W, x, out, *args)
    torch.cuda.synchronize()
    assert int(err.item()) == 2001            # peer 1 never arrived
    assert torch.equal(out, res)              # the reduction was skipped
    # later calls see the poisoned word and return without waiting
    t0 = time.perf_counter()
    for _ in range(20):
        C.gemv_ar(W, x, out, *args)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 0.1 and int(err.item()) == 2001
    E, H, I = 4, 256, 128
    Wd = (torch.randn(E, H, I, device="cuda") * 0.05).bfloat16()
    act = torch.randn(2, I, device="cuda").bfloat16()
    ids = torch.tensor([[0, 3]], dtype=torch.int32, device="cuda")
    wts = torch.rand(1, 2, device="cuda")
    args2, err2, _ = _tp_args(C, [mine.data_ptr(), ghost.data_ptr()], 0, words, 0.005)
    xx = torch.randn(1, H, device="cuda").bfloat16()
    C.moe_down_ar(Wd, act, ids, wts, xx.clone(), *args2)
    torch.cuda.synchronize()
    assert int(err2.item()) == 2001


def test_oneshot_missing_peer_times_out():
    from helexa_b200.parallel.tp import TPError
    C = _C()
    data_bytes = 1 << 16
    a, _ = C.ipc_alloc(4096 + 2 * data_bytes, 0)
    b, _ = C.ipc_alloc(4096 + 2 * data_bytes, 0)
    epoch = torch.zeros(2, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    p = torch.randn(1024, device="cuda").bfloat16()
    x = torch.randn(1024, device="cuda").bfloat16()
    x0 = x.clone()
    C.ar_oneshot([a.data_ptr(), b.data_ptr()], 0, p, x, None, data_bytes, epoch, err, 1, 0.005)
    torch.cuda.synchronize()
    assert int(err.item()) == 1001 and torch.equal(x, x0)

    from helexa_b200.parallel.tp import TPComm
    c = TPComm.__new__(TPComm)  # TPComm.check reads the same error word
    c.mode, c.rank, c.timeout_s, c.err = "p2p", 0, 0.005, err
    with pytest.raises(TPError):
        TPComm.check(c)
