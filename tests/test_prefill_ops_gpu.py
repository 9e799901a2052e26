"""Prefill element-wise kernels against plain PyTorch fp32 references of the same op:
fused residual add + RMSNorm, q/k-norm + partial RoPE + KV append, conv-ring update,
the attention kernel's sigmoid-gate epilogue, and the fused TP reduction kernel run
with one rank (add + norm + store into the exported h buffer)."""
import pytest
import torch

from helexa_b200.models.reference import apply_rope, rope_cos_sin

pytestmark = pytest.mark.gpu


def _C():
    from helexa_b200 import ops
    return ops.C


def _close(a, b, tol):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    assert err <= tol * max(1.0, b.abs().max().item()), err


@pytest.mark.parametrize("T,H", [(37, 2048), (5, 4096), (16, 5120), (300, 256)])
def test_add_rmsnorm(T, H):
    C = _C()
    torch.manual_seed(0)
    x = torch.randn(T, H, device="cuda").bfloat16()
    o = torch.randn(T, H, device="cuda").bfloat16()
    w = torch.rand(H, device="cuda") + 0.5
    xs = (x.float() + o.float()).bfloat16()
    want = xs.float() * torch.rsqrt(xs.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w
    h = torch.empty_like(x)
    x2 = x.clone()
    C.add_rmsnorm(x2, o, w, h, 1e-6)
    assert torch.equal(x2, xs)
    _close(h, want, 1e-2)
    h2 = torch.empty_like(x)
    C.add_rmsnorm(x, None, w, h2, 1e-6)  # norm only, x untouched
    want2 = x.float() * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6) * w
    _close(h2, want2, 1e-2)


@pytest.mark.parametrize("D,Hq,Hkv,rot,gated,norm", [(256, 4, 2, 64, True, True), (128, 8, 2, 128, False, True),
                                                     (64, 4, 2, 16, True, False)])
def test_qk_rope_kv(D, Hq, Hkv, rot, gated, norm):
    C = _C()
    torch.manual_seed(1)
    T, p0, maxlen = 50, 7, 128
    qw = 2 * D if gated else D
    qkv = torch.randn(T, Hq * qw + 2 * Hkv * D, device="cuda").bfloat16()
    qn = torch.rand(D, device="cuda") + 0.5 if norm else None
    kn = torch.rand(D, device="cuda") + 0.5 if norm else None
    inv = (1.0 / (1e6 ** (torch.arange(0, rot, 2, dtype=torch.int64).float() / rot))).cuda()
    kc = torch.zeros(Hkv, maxlen, D, device="cuda").bfloat16()
    vc = torch.zeros_like(kc)
    q = torch.empty(T, Hq * D, device="cuda").bfloat16()
    C.qk_rope_kv(qkv, Hq, Hkv, D, qw, qn, kn, inv, rot, kc, vc, p0, q, 1e-6)
    qp = qkv[:, :Hq * qw].view(T, Hq, qw)[..., :D].float()
    k = qkv[:, Hq * qw:Hq * qw + Hkv * D].view(T, Hkv, D).float()
    v = qkv[:, Hq * qw + Hkv * D:].view(T, Hkv, D)

    def rms(t, w):
        return (t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + 1e-6) * w).bfloat16().float()
    if norm:
        qp, k = rms(qp, qn), rms(k, kn)
    cos, sin = rope_cos_sin(torch.arange(p0, p0 + T, device="cuda"), rot, 1e6, inv)
    _close(q.view(T, Hq, D), apply_rope(qp, cos, sin), 1e-2)
    _close(kc[:, p0:p0 + T].transpose(0, 1), apply_rope(k, cos, sin), 1e-2)
    assert torch.equal(vc[:, p0:p0 + T].transpose(0, 1), v)
    assert kc[:, :p0].abs().sum() == 0 and kc[:, p0 + T:].abs().sum() == 0


def test_conv_ring_update():
    C = _C()
    Cc, K = 96, 4
    for T, p0 in [(10, 0), (2, 5), (1, 9), (7, 3)]:
        proj = torch.randn(T, Cc + 20, device="cuda").bfloat16()
        ring = torch.randn(Cc, K, device="cuda").bfloat16()
        want = ring.clone()
        for p in range(max(p0, p0 + T - K), p0 + T):
            want[:, p % K] = proj[p - p0, :Cc]
        C.conv_ring_update(proj, ring, p0)
        assert torch.equal(ring, want)


def test_attn_prefill_gate_epilogue():
    C = _C()
    torch.manual_seed(2)
    T, D, Hq, Hkv = 100, 128, 4, 2
    q = torch.randn(T, Hq * D, device="cuda").bfloat16()
    kc = torch.randn(Hkv, 256, D, device="cuda").bfloat16()
    vc = torch.randn(Hkv, 256, D, device="cuda").bfloat16()
    qkv = torch.randn(T, Hq * 2 * D, device="cuda").bfloat16()
    plain = torch.empty(T, Hq * D, device="cuda").bfloat16()
    C.attn_prefill(q, kc, vc, plain, Hq, 0, D ** -0.5)
    gated = torch.empty_like(plain)
    C.attn_prefill(q, kc, vc, gated, Hq, 0, D ** -0.5, qkv[:, D:], 2 * D)
    gate = qkv.view(T, Hq, 2 * D)[..., D:].reshape(T, Hq * D)
    _close(gated, plain.float() * torch.sigmoid(gate.float()), 1e-2)


def test_rs_norm_ag_single_rank():
    """One rank: the fused reduction kernel is add + norm, reading the partial from the
    exported staging buffer and writing h into the exported h buffer."""
    C = _C()
    torch.manual_seed(3)
    T, H = 64, 2048
    flag = C.rs_norm_ag_flag_bytes()
    nb = T * H * 2
    region, _ = C.ipc_alloc(flag + 2 * nb, 0)
    stage = region[flag:flag + nb].view(torch.bfloat16).view(T, H)
    hbuf = region[flag + nb:flag + 2 * nb].view(torch.bfloat16).view(T, H)
    ctr = torch.zeros(2, dtype=torch.int32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    w = torch.rand(H, device="cuda") + 0.5
    for call in range(3):
        x = torch.randn(T, H, device="cuda").bfloat16()
        stage.copy_(torch.randn(T, H, device="cuda").bfloat16())
        want_x, want_h = x.clone(), torch.empty_like(x)
        C.add_rmsnorm(want_x, stage, w, want_h, 1e-6)
        C.rs_norm_ag([region.data_ptr()], 0, flag, flag + nb, x, w, 1e-6, ctr, err, 1.0, 16)
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert torch.equal(x, want_x) and torch.equal(hbuf, want_h)
    assert int(ctr[0].item()) == 3
