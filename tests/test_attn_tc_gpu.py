"""tcgen05/TMEM attention prefill against an fp32 softmax of the same bf16 inputs:
partial query tiles, an earlier prefix (p0 > 0), a single token, grouped query heads,
head dims 64 / 128 / 256, long rows that trigger the lazy O rescale, and the sigmoid
output gate in the epilogue."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(a, b, tol):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    assert err <= tol * max(1.0, b.abs().max().item()), err


def _ref(q, kc, vc, T, p0, Hq, Hkv, D):
    L, G = p0 + T, Hq // Hkv
    qf = q.float().view(T, Hq, D).transpose(0, 1)
    kf = kc[:, :L].float().repeat_interleave(G, 0)
    vf = vc[:, :L].float().repeat_interleave(G, 0)
    sc = torch.einsum("htd,hld->htl", qf, kf) * D ** -0.5
    mask = torch.arange(L, device="cuda")[None, :] <= (p0 + torch.arange(T, device="cuda"))[:, None]
    sc = sc.masked_fill(~mask[None], float("-inf"))
    return torch.einsum("htl,hld->htd", torch.softmax(sc, -1), vf).transpose(0, 1).reshape(T, Hq * D)


@pytest.mark.parametrize("T,p0,D,Hq,Hkv,qs", [(200, 0, 256, 16, 2, 1.0), (70, 33, 128, 8, 8, 1.0),
                                             (1, 100, 64, 4, 2, 1.0), (300, 129, 256, 4, 1, 1.0),
                                             (1030, 0, 128, 8, 2, 1.0), (777, 300, 256, 4, 2, 6.0),
                                             (2048, 0, 256, 2, 1, 1.0)])
def test_attn_prefill_tc_matches_fp32(T, p0, D, Hq, Hkv, qs):
    from helexa_b200 import ops
    C = ops.C
    torch.manual_seed(11)
    maxlen = p0 + T + 37
    q = (torch.randn(T, Hq * D, device="cuda") * qs).bfloat16()  # qs > 1: peaked rows, frequent rescales
    kc = torch.randn(Hkv, maxlen, D, device="cuda").bfloat16()
    vc = torch.randn(Hkv, maxlen, D, device="cuda").bfloat16()
    out = torch.full((T, Hq * D), float("nan"), device="cuda", dtype=torch.bfloat16)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.attn_prefill_tc(q, kc, vc, out, Hq, p0, D ** -0.5, None, 0, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    _close(out, _ref(q, kc, vc, T, p0, Hq, Hkv, D), 2e-2)


def test_attn_prefill_tc_gate_matches_mma_kernel():
    from helexa_b200 import ops
    C = ops.C
    torch.manual_seed(12)
    T, D, Hq, Hkv = 300, 256, 4, 2
    q = torch.randn(T, Hq * D, device="cuda").bfloat16()
    kc = torch.randn(Hkv, 512, D, device="cuda").bfloat16()
    vc = torch.randn(Hkv, 512, D, device="cuda").bfloat16()
    qkv = torch.randn(T, Hq * 2 * D, device="cuda").bfloat16()
    a = torch.empty(T, Hq * D, device="cuda").bfloat16()
    b = torch.empty_like(a)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    C.attn_prefill(q, kc, vc, a, Hq, 0, D ** -0.5, qkv[:, D:], 2 * D)
    C.attn_prefill_tc(q, kc, vc, b, Hq, 0, D ** -0.5, qkv[:, D:], 2 * D, err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    _close(b, a, 2e-2)
