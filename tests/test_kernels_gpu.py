"""Numerics of each CUDA kernel against a plain PyTorch fp32 reference of the same op."""
import pytest
import torch

from helexa_b200.models import reference as R

pytestmark = pytest.mark.gpu


def _C():
    from helexa_b200 import ops
    return ops.C


def _close(a, b, tol):
    err = (a.float() - b.float()).abs().max().item()
    scale = b.float().abs().max().item() + 1e-6
    assert err <= tol * scale, f"max err {err} vs scale {scale}"


@pytest.mark.parametrize("B", [1, 2, 4, 5])
@pytest.mark.parametrize("N,K", [(2048, 4096), (12352, 2048), (100, 256)])
def test_gemv_modes(B, N, K):
    from helexa_b200 import ops
    C = _C()
    g = torch.Generator(device="cuda").manual_seed(0)
    W = torch.randn(N, K, device="cuda", generator=g).bfloat16() * 0.05
    x = torch.randn(B, K, device="cuda", generator=g).bfloat16()
    nw = (torch.rand(K, device="cuda", generator=g) + 0.5).float()
    ref = x.float() @ W.float().t()
    y = torch.empty(B, N, device="cuda", dtype=torch.float32)
    C.gemv(W, x, y, ops.STORE_F32, None, None, 0.0)
    _close(y, ref, 1e-3)
    # norm prologue
    xn = R.rms_norm(x, nw, 1e-6, 0.0).bfloat16().float()
    C.gemv(W, x, y, ops.STORE_F32, None, nw, 1e-6)
    _close(y, xn @ W.float().t(), 1e-2)
    # residual epilogue in place
    res = torch.randn(B, N, device="cuda", generator=g).bfloat16()
    r2 = res.clone()
    C.gemv(W, x, r2, ops.RESID_ADD, r2, None, 0.0)
    _close(r2, res.float() + ref, 2e-2)
    if N % 2 == 0:
        act = torch.empty(B, N // 2, device="cuda", dtype=torch.bfloat16)
        C.gemv(W, x, act, ops.SILU_PAIR, None, None, 0.0)
        _close(act, torch.nn.functional.silu(ref[:, 0::2]) * ref[:, 1::2], 2e-2)


def test_moe_topk_and_down():
    C = _C()
    torch.manual_seed(0)
    B, E, k, H, I = 3, 64, 6, 512, 128
    logits = torch.randn(B, E + 1, device="cuda")
    ids = torch.zeros(B, k + 1, dtype=torch.int32, device="cuda")
    wts = torch.zeros(B, k + 1, device="cuda")
    C.moe_topk(logits, E, k, True, True, ids, wts)
    p = torch.softmax(logits[:, :E], -1)
    tv, ti = torch.topk(p, k, -1)
    assert torch.equal(ids[:, :k].long(), ti)
    _close(wts[:, :k], tv / tv.sum(-1, keepdim=True), 1e-5)
    assert (ids[:, k] == E).all()
    _close(wts[:, k], torch.sigmoid(logits[:, E]), 1e-5)
    Wd = (torch.randn(E + 1, H, I, device="cuda") * 0.05).bfloat16()
    act = torch.randn(B * (k + 1), I, device="cuda").bfloat16()
    x = torch.randn(B, H, device="cuda").bfloat16()
    want = x.float().clone()
    for b in range(B):
        for j in range(k + 1):
            want[b] += wts[b, j] * (Wd[ids[b, j]].float() @ act[b * (k + 1) + j].float())
    C.moe_down(Wd, act, ids, wts, x, None)
    _close(x, want, 2e-2)


@pytest.mark.parametrize("Dk,Hk,Hv", [(128, 4, 8), (32, 4, 8)])
def test_gdn_decode_matches_recurrent(Dk, Hk, Hv):
    C = _C()
    torch.manual_seed(1)
    Dv, K, S = Dk, 4, 3
    kd, vd = Hk * Dk, Hv * Dv
    Cc = 2 * kd + vd
    B = 2
    slots = torch.tensor([2, 0], dtype=torch.int32, device="cuda")
    pos = torch.tensor([5, 0, 9], dtype=torch.int32, device="cuda")
    conv_w = torch.randn(Cc, K, device="cuda") * 0.3
    ring = (torch.randn(S, Cc, K, device="cuda")).bfloat16()
    rec = torch.randn(S, Hv, Dk, Dv, device="cuda") * 0.1
    A_log = torch.randn(Hv, device="cuda") * 0.5
    dt_bias = torch.randn(Hv, device="cuda") * 0.5
    nw = torch.rand(Dv, device="cuda") + 0.5
    proj = torch.randn(B, 2 * kd + 2 * vd + 2 * Hv, device="cuda").bfloat16()
    out = torch.empty(B, vd, device="cuda", dtype=torch.bfloat16)
    ring0, rec0 = ring.clone(), rec.clone()
    C.gdn_decode(proj, conv_w, ring, rec, A_log, dt_bias, nw, slots, pos, out, Hk, Hv, Dk, Dv, 1e-6)
    r = Hv // Hk
    for b in range(B):
        s = int(slots[b]); p = int(pos[s])
        x = proj[b].float()
        mixed = x[:Cc]
        prev = torch.stack([ring0[s][:, (p - 3 + j) % K].float() if p - 3 + j >= 0 else torch.zeros(Cc, device="cuda")
                            for j in range(3)], 1)
        y, _ = R.causal_conv1d(mixed[None], conv_w, prev)
        y = y[0].bfloat16().float()
        q = y[:kd].view(Hk, Dk).repeat_interleave(r, 0)
        k = y[kd:2 * kd].view(Hk, Dk).repeat_interleave(r, 0)
        v = y[2 * kd:].view(Hv, Dv)
        z = x[2 * kd + vd:2 * kd + 2 * vd].view(Hv, Dv)
        bb = x[2 * kd + 2 * vd:2 * kd + 2 * vd + Hv]
        aa = x[2 * kd + 2 * vd + Hv:]
        g, beta = R.gdn_gating(aa, bb, A_log, dt_bias)
        q = R.l2norm(q) * Dk ** -0.5
        k = R.l2norm(k)
        o, S1 = R.delta_rule_recurrent(q[None], k[None], v[None], g[None], beta[None], rec0[s])
        _close(rec[s], S1, 1e-4)
        want = R.gated_rms_norm(o[0], z, nw, 1e-6).reshape(-1)
        _close(out[b], want, 3e-2)
        assert torch.equal(ring[s][:, p % K], proj[b, :Cc])


@pytest.mark.parametrize("D,Hq,Hkv,gated,L,ns", [(256, 16, 2, True, 700, 16), (256, 16, 2, True, 1900, 152),
                                                 (128, 32, 8, False, 1500, 12), (64, 4, 2, True, 3, 5),
                                                 (128, 64, 4, False, 999, 8), (256, 8, 4, True, 64, 40)])
def test_attn_decode(D, Hq, Hkv, gated, L, ns):
    """Split counts cover 8-, 4- and 1-CTA clusters, 19 cluster partials, more splits
    than keys, and 16 query heads per kv head."""
    C = _C()
    torch.manual_seed(2)
    S, maxlen, B = 2, 2048, 2
    rot = D // 4 if gated else D
    slots = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
    pos = torch.tensor([L - 1, L // 2], dtype=torch.int32, device="cuda")
    kc = torch.randn(S, Hkv, maxlen, D, device="cuda").bfloat16()
    vc = torch.randn(S, Hkv, maxlen, D, device="cuda").bfloat16()
    qw = 2 * D if gated else D
    proj = torch.randn(B, Hq * qw + 2 * Hkv * D, device="cuda").bfloat16()
    qn = torch.rand(D, device="cuda") + 0.5
    kn = torch.rand(D, device="cuda") + 0.5
    theta = 1e7
    inv = 1.0 / (theta ** (torch.arange(0, rot, 2, dtype=torch.int64).float() / rot)).cuda()
    part_o = torch.empty(B, Hq, ns, D, device="cuda")
    part_ml = torch.empty(B, Hq, ns, 2, device="cuda")
    cnt = torch.zeros(B, Hkv, dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hq * D, device="cuda", dtype=torch.bfloat16)
    kc0, vc0 = kc.clone(), vc.clone()
    for rep in range(2):  # second launch checks the self-resetting counters
        kc.copy_(kc0); vc.copy_(vc0)
        C.attn_decode(proj, qn, kn, inv, kc, vc, slots, pos, part_o, part_ml, cnt, out, Hq, Hkv, D, rot, gated, 1e-6)
        assert int(cnt.abs().sum()) == 0
        for b in range(B):
            s = int(slots[b]); p = int(pos[s])
            x = proj[b]
            q = x[:Hq * qw].view(Hq, qw)[:, :D]
            gate = x[:Hq * qw].view(Hq, qw)[:, D:] if gated else None
            k = x[Hq * qw:Hq * qw + Hkv * D].view(Hkv, D)
            v = x[Hq * qw + Hkv * D:].view(Hkv, D)
            q = R.rms_norm(q, qn, 1e-6, 0.0).bfloat16().float()
            k = R.rms_norm(k, kn, 1e-6, 0.0).bfloat16().float()
            cos, sin = R.rope_cos_sin(torch.tensor([p], device="cuda"), rot, theta)
            q = R.apply_rope(q[None], cos, sin)[0]
            k = R.apply_rope(k[None], cos, sin)[0]
            _close(kc[s, :, p], k, 2e-2)
            assert torch.equal(vc[s, :, p], v)
            Kf = kc0[s, :, :p + 1].float().clone()
            Vf = vc0[s, :, :p + 1].float().clone()
            Kf[:, p], Vf[:, p] = k, v.float()
            Kr = Kf.repeat_interleave(Hq // Hkv, 0)
            Vr = Vf.repeat_interleave(Hq // Hkv, 0)
            sc = torch.einsum("hd,hld->hl", q, Kr) / D ** 0.5
            o = torch.einsum("hl,hld->hd", torch.softmax(sc, -1), Vr)
            if gated:
                o = o * torch.sigmoid(gate.float())
            _close(out[b].view(Hq, D), o, 3e-2)


def test_embed_and_argmax():
    C = _C()
    E = torch.randn(1000, 256, device="cuda").bfloat16()
    tok = torch.tensor([5, 999, 0], dtype=torch.int32, device="cuda")
    x = torch.empty(3, 256, device="cuda", dtype=torch.bfloat16)
    C.embed(E, tok, x)
    assert torch.equal(x, E[tok.long()])
    logits = torch.randn(3, 151936, device="cuda")
    logits[1, 7] = logits[1, 9] = 100.0
    pos = torch.zeros(4, dtype=torch.int32, device="cuda")
    slots = torch.tensor([3, 1, 2], dtype=torch.int32, device="cuda")
    out = torch.zeros(3, 8, dtype=torch.int32, device="cuda")
    step = torch.zeros(3, dtype=torch.int32, device="cuda")
    C.argmax_step(logits, tok, slots, pos, out, step)
    assert torch.equal(tok.long(), logits.argmax(-1))
    assert int(tok[1]) == 7
    assert pos.tolist() == [0, 1, 1, 1] and step.tolist() == [1, 1, 1]
    assert torch.equal(out[:, 0], tok)


@pytest.mark.parametrize("T,p0,D", [(200, 0, 128), (70, 5, 128), (33, 0, 32), (130, 64, 32), (513, 0, 64),
                                    (1000, 7, 128)])
def test_gdn_prefill_matches_reference(T, p0, D):
    C = _C()
    torch.manual_seed(7)
    Hk, Hv, K = 2, 4, 4
    kd, vd = Hk * D, Hv * D
    Cc = 2 * kd + vd
    proj = torch.randn(T, 2 * kd + 2 * vd + 2 * Hv, device="cuda").bfloat16()
    conv_w = torch.randn(Cc, K, device="cuda") * 0.3
    ring = torch.randn(Cc, K, device="cuda").bfloat16()
    A_log = torch.randn(Hv, device="cuda") * 0.5
    dt_bias = torch.randn(Hv, device="cuda") * 0.5
    nw = torch.rand(D, device="cuda") + 0.5
    S0 = torch.randn(Hv, D, D, device="cuda") * 0.05
    S = S0.clone()
    out = torch.empty(T, vd, device="cuda", dtype=torch.bfloat16)
    C.gdn_prefill(proj, conv_w, ring, A_log, dt_bias, nw, S, out, Hk, Hv, D, p0, 1e-6)
    # reference
    prev = torch.stack([ring[:, (p0 - 3 + j) % K].float() if p0 - 3 + j >= 0 else torch.zeros(Cc, device="cuda")
                        for j in range(3)], 1)
    y, _ = R.causal_conv1d(proj[:, :Cc].float(), conv_w, prev)
    y = y.bfloat16().float()
    r = Hv // Hk
    q = R.l2norm(y[:, :kd].view(T, Hk, D).repeat_interleave(r, 1)) * D ** -0.5
    k = R.l2norm(y[:, kd:2 * kd].view(T, Hk, D).repeat_interleave(r, 1))
    v = y[:, 2 * kd:].view(T, Hv, D)
    z = proj[:, Cc:Cc + vd].float().view(T, Hv, D)
    bb = proj[:, Cc + vd:Cc + vd + Hv].float()
    aa = proj[:, Cc + vd + Hv:].float()
    g, beta = R.gdn_gating(aa, bb, A_log, dt_bias)
    o, S1 = R.delta_rule_recurrent(q, k, v, g, beta, S0)
    want = R.gated_rms_norm(o, z, nw, 1e-6).reshape(T, vd)
    _close(S, S1, 2e-2)
    _close(out, want, 3e-2)


@pytest.mark.parametrize("T,p0,D,Hq,Hkv", [(200, 0, 256, 16, 2), (70, 33, 128, 8, 8), (1, 100, 64, 4, 2),
                                          (300, 129, 256, 4, 1), (64, 0, 128, 4, 4), (700, 50, 256, 4, 2),
                                          (1030, 0, 128, 8, 2)])
def test_attn_prefill_matches_fp32(T, p0, D, Hq, Hkv):
    """Causal GQA prefill over the cache (keys 0..p0+T-1) against an fp32 softmax of the
    same bf16 inputs; covers partial query tiles, an earlier prefix (p0 > 0), a single
    token, grouped query heads and both CTA shapes (4 and 8 warps)."""
    C = _C()
    torch.manual_seed(11)
    L, maxlen = p0 + T, p0 + T + 37
    q = torch.randn(T, Hq * D, device="cuda").bfloat16()
    kc = torch.randn(Hkv, maxlen, D, device="cuda").bfloat16()
    vc = torch.randn(Hkv, maxlen, D, device="cuda").bfloat16()
    out = torch.empty(T, Hq * D, device="cuda", dtype=torch.bfloat16)
    C.attn_prefill(q, kc, vc, out, Hq, p0, D ** -0.5)
    torch.cuda.synchronize()
    G = Hq // Hkv
    qf = q.float().view(T, Hq, D).transpose(0, 1)                       # [Hq, T, D]
    kf = kc[:, :L].float().repeat_interleave(G, 0)                       # [Hq, L, D]
    vf = vc[:, :L].float().repeat_interleave(G, 0)
    sc = torch.einsum("htd,hld->htl", qf, kf) * D ** -0.5
    mask = torch.arange(L, device="cuda")[None, :] <= (p0 + torch.arange(T, device="cuda"))[:, None]
    sc = sc.masked_fill(~mask[None], float("-inf"))
    want = torch.einsum("htl,hld->htd", torch.softmax(sc, -1), vf).transpose(0, 1).reshape(T, Hq * D)
    _close(out, want, 2e-2)
