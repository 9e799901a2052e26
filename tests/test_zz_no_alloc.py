"""The allocation-free attention-decode entry point, called through its C symbol.

`hx_attn_decode_noalloc` serves callers that cannot allocate device memory when they
call in (a host framework that owns every allocation, or a plain C/C++ caller with no
caching allocator): its split-K scratch is a fixed device array inside the library.
This test loads the symbol with ctypes, runs it twice in a row and checks both
results against the regular `attn_decode` op within the tolerance the kernel tests
use. It lives in its own file, collected last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from helexa_b200 import ops
    lib = ctypes.CDLL(ops.C.__file__)
    f = lib.hx_attn_decode_noalloc
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    f.argtypes = [P, I, P, P, P, P, P, I, P, P, P, I, I, I, I, I, I, F, I, P]
    f.restype = I
    lib.hx_noalloc_error.restype = ctypes.c_char_p
    return lib, f


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("D,Hq,Hkv,gated,L", [(256, 16, 2, True, 700), (128, 32, 8, False, 1500)])
def test_noalloc_matches_attn_decode(D, Hq, Hkv, gated, L):
    from helexa_b200 import ops
    lib, f = _lib()
    torch.manual_seed(5)
    S, maxlen, B, ns = 2, 2048, 2, 16
    rot = D // 4 if gated else D
    slots = torch.tensor([1, 0], dtype=torch.int32, device="cuda")
    pos = torch.tensor([L - 1, L // 3], dtype=torch.int32, device="cuda")
    kc0 = torch.randn(S, Hkv, maxlen, D, device="cuda").bfloat16()
    vc0 = torch.randn(S, Hkv, maxlen, D, device="cuda").bfloat16()
    qw = 2 * D if gated else D
    qn = torch.rand(D, device="cuda") + 0.5
    kn = torch.rand(D, device="cuda") + 0.5
    inv = (1.0 / (1e7 ** (torch.arange(0, rot, 2, dtype=torch.int64).float() / rot))).cuda()
    stream = torch.cuda.current_stream()
    for call in range(2):
        proj = torch.randn(B, Hq * qw + 2 * Hkv * D, device="cuda").bfloat16()
        # existing entry point, with caller-provided scratch
        kc, vc = kc0.clone(), vc0.clone()
        part_o = torch.empty(B, Hq, ns, D, device="cuda")
        part_ml = torch.empty(B, Hq, ns, 2, device="cuda")
        cnt = torch.zeros(B, Hkv, dtype=torch.int32, device="cuda")
        want = torch.empty(B, Hq * D, device="cuda", dtype=torch.bfloat16)
        ops.C.attn_decode(proj, qn, kn, inv, kc, vc, slots, pos, part_o, part_ml, cnt, want, Hq, Hkv, D, rot,
                          gated, 1e-6)
        # allocation-free entry point through the exported C symbol
        kc2, vc2 = kc0.clone(), vc0.clone()
        got = torch.full((B, Hq * D), float("nan"), device="cuda", dtype=torch.bfloat16)
        rc = f(_p(proj), proj.shape[1], _p(qn), _p(kn), _p(inv), _p(kc2), _p(vc2), maxlen, _p(slots), _p(pos),
               _p(got), B, Hq, Hkv, D, rot, int(gated), 1e-6, ns, ctypes.c_void_p(stream.cuda_stream))
        assert rc == 0, lib.hx_noalloc_error()
        torch.cuda.synchronize()
        err = (got.float() - want.float()).abs().max().item()
        assert err <= 3e-2 * want.float().abs().max().item(), (call, err)
        assert torch.equal(kc2, kc) and torch.equal(vc2, vc)


def test_noalloc_rejects_oversized_request():
    lib, f = _lib()
    z = ctypes.c_void_p(0)
    # B*Hq*nsplit*D far beyond the fixed scratch: refused before any launch
    rc = f(z, 0, z, z, z, z, z, 16, z, z, z, 64, 64, 8, 256, 64, 1, 1e-6, 256, z)
    assert rc == 1004  # HX_NOALLOC_E_SCRATCH: never a cudaError_t value
    assert b"scratch too small" in lib.hx_noalloc_error()
