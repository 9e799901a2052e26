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
