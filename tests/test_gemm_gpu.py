"""tcgen05 GEMM (plain and grouped) against an fp32 torch matmul of the same bf16 inputs."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _C():
    from helexa_b200 import ops
    return ops.C


def _err():
    return torch.zeros(1, dtype=torch.int32, device="cuda")


def _check(got, want, tol=1e-2):
    err = (got.float() - want).abs().max().item()
    assert err <= tol * (want.abs().max().item() + 1e-6), err


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 512, 2048), (8192, 1024, 2048), (77, 2048, 4096),
                                   (1000, 520, 136)])
def test_gemm_bf16(M, N, K):
    torch.manual_seed(0)
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    e = _err()
    _C().gemm(A, B, C, 0, e)
    torch.cuda.synchronize()
    assert int(e) == 0
    _check(C, A.float() @ B.float().t())


def test_gemm_f32_and_swiglu():
    torch.manual_seed(1)
    M, N, K = 500, 1024, 2048
    A = torch.randn(M, K, device="cuda").bfloat16()
    B = (torch.randn(N, K, device="cuda") * 0.05).bfloat16()
    e = _err()
    Cf = torch.empty(M, N, device="cuda")
    _C().gemm(A, B, Cf, 2, e)
    ref = A.float() @ B.float().t()
    _check(Cf, ref, 1e-3)
    Cs = torch.empty(M, N // 2, device="cuda", dtype=torch.bfloat16)
    _C().gemm(A, B, Cs, 1, e)
    torch.cuda.synchronize()
    _check(Cs, torch.nn.functional.silu(ref[:, 0::2]) * ref[:, 1::2], 2e-2)
    assert int(e) == 0


def test_gemm_grouped():
    torch.manual_seed(2)
    G, N, K = 5, 384, 512
    counts = [0, 130, 7, 256, 1]
    A = torch.randn(sum(counts), K, device="cuda").bfloat16()
    B = (torch.randn(G * N, K, device="cuda") * 0.05).bfloat16()
    tiles, row = [], 0
    for g, c in enumerate(counts):
        for m0 in range(0, c, 128):
            tiles.append([row + m0, g * N, min(128, c - m0), row + m0])
        row += c
    t = torch.tensor(tiles, dtype=torch.int32, device="cuda")
    C = torch.zeros(sum(counts), N, device="cuda", dtype=torch.bfloat16)
    e = _err()
    _C().gemm_grouped(A, B, C, t, N, 0, e)
    torch.cuda.synchronize()
    assert int(e) == 0
    row = 0
    for g, c in enumerate(counts):
        if c:
            _check(C[row:row + c], A[row:row + c].float() @ B[g * N:(g + 1) * N].float().t())
        row += c


@pytest.mark.parametrize("shared", [True, False])
def test_moe_route_prefill_and_grouped_dev(shared):
    """Device routing (top-k, plan, gather) + grouped GEMMs with a device tile count
    against a per-token fp32 loop over the selected experts."""
    torch.manual_seed(3)
    T, H, E, k, I = 300, 256, 16, 4, 128
    G, J = E + int(shared), k + int(shared)
    C = _C()
    hn = torch.randn(T, H, device="cuda").bfloat16()
    logits = torch.randn(T, E + 8, device="cuda") * 3
    w_gu = (torch.randn(G, 2 * I, H, device="cuda") * 0.05).bfloat16()
    w_d = (torch.randn(G, H, I, device="cuda") * 0.05).bfloat16()
    i32 = dict(dtype=torch.int32, device="cuda")
    ids, rows = torch.empty(T, J, **i32), torch.empty(T, J, **i32)
    wts = torch.empty(T, J, device="cuda")
    counts, offsets, cursor = torch.zeros(G, **i32), torch.empty(G, **i32), torch.empty(G, **i32)
    tiles, ntiles = torch.empty((T * J + 127) // 128 + G, 4, **i32), torch.empty(1, **i32)
    A = torch.empty(T * J, H, device="cuda", dtype=torch.bfloat16)
    C.moe_route_prefill(logits, E, k, shared, True, hn, ids, wts, rows, counts, offsets, cursor, tiles, ntiles, A,
                        0, 0)
    act = torch.empty(T * J, I, device="cuda", dtype=torch.bfloat16)
    e = _err()
    C.gemm_grouped_dev(A, w_gu.view(-1, H), act, tiles, ntiles, 2 * I, 1, e)
    y = torch.empty(T * J, H, device="cuda", dtype=torch.bfloat16)
    C.gemm_grouped_dev(act, w_d.view(-1, I), y, tiles, ntiles, H, 0, e)
    out = torch.zeros(T, H, device="cuda", dtype=torch.bfloat16)
    C.moe_combine(y, rows, wts, out)
    torch.cuda.synchronize()
    assert int(e) == 0
    probs = torch.softmax(logits[:, :E], -1)
    tv, ti = torch.topk(probs, k, -1)
    tv = tv / tv.sum(-1, keepdim=True)
    assert torch.equal(ids[:, :k].long(), ti)
    assert torch.allclose(wts[:, :k], tv, atol=1e-5)
    assert sorted(rows.flatten().tolist()) == list(range(T * J))
    assert torch.equal(A[rows.long()].view(T, J, H), hn[:, None].expand(T, J, H))
    ref = torch.zeros(T, H, device="cuda")
    for t in range(T):
        sel = [(int(ti[t, j]), float(tv[t, j])) for j in range(k)]
        if shared:
            sel.append((E, float(torch.sigmoid(logits[t, E]))))
        for g, w in sel:
            hgu = hn[t].float() @ w_gu[g].float().t()
            a = torch.nn.functional.silu(hgu[0::2]) * hgu[1::2]
            ref[t] += w * (a.bfloat16().float() @ w_d[g].float().t())
    _check(out, ref, 3e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("gtype", ["Q8_0", "Q4_K", "Q6_K"])
@pytest.mark.parametrize("epi", [0, 1, 2])
def test_gemm_fused_dequant_matches_dequantized_gemm(gtype, epi):
    """The GEMM that dequantizes GGUF blocks in its producer warps gives the same result
    as dequantizing the whole weight to bf16 and running the bf16 GEMM (same bf16 B
    values, same accumulation order), on ragged M and N."""
    from helexa_b200 import ops
    from helexa_b200.models.fast import GGUF_Q4_K, GGUF_Q6_K, GGUF_Q8_0, QWeight
    C = ops.C
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(5)
    M, N, K = 300, 544, 768
    w = (torch.randn(N, K, device=dev, generator=g) * 0.05).bfloat16()
    t = {"Q8_0": GGUF_Q8_0, "Q4_K": GGUF_Q4_K, "Q6_K": GGUF_Q6_K}[gtype]
    qw = QWeight(C.gguf_quant(w, t), t, K)
    x = torch.randn(M, K, device=dev, generator=g).bfloat16()
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    n_out = N // 2 if epi == 1 else N
    dt = torch.float32 if epi == 2 else torch.bfloat16
    ref = torch.empty(M, n_out, dtype=dt, device=dev)
    C.gemm(x, qw.dequant(C), ref, epi, err)
    got = torch.empty(M, n_out, dtype=dt, device=dev)
    C.gemm_q(x, qw.raw, qw.type, K, got, epi, err)
    torch.cuda.synchronize()
    assert err.item() == 0
    assert (got.float() - ref.float()).abs().max().item() <= 1e-2 * ref.float().abs().max().item()
