"""tcgen05 GEMM throughput vs cuBLAS (torch.matmul) on prefill-shaped problems.

  python -m helexa_b200.bench.gemm_bench [--shapes 8192x12352x2048,...]
Times with CUDA events after warm-up; inputs exceed L2 for the large shapes.
"""
from __future__ import annotations

import argparse
import json

import torch

DEFAULT = "8192x12352x2048,8192x2048x4096,8192x9216x2048,8192x151936x2048,16384x8192x8192"


def bench(fn, iters=20, warm=5):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    e1.synchronize()
    return e0.elapsed_time(e1) / iters


def main():
    from .. import ops
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default=DEFAULT)
    args = ap.parse_args()
    C = ops.C
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    for s in args.shapes.split(","):
        M, N, K = (int(v) for v in s.split("x"))
        A = torch.randn(M, K, device="cuda", dtype=torch.bfloat16)
        B = torch.randn(N, K, device="cuda", dtype=torch.bfloat16) * 0.05
        Cm = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        ms = bench(lambda: C.gemm(A, B, Cm, 0, err))
        ms_ref = bench(lambda: torch.matmul(A, B.t()))
        ref = torch.matmul(A, B.t())
        rel = ((Cm.float() - ref.float()).norm() / ref.float().norm()).item()
        fl = 2.0 * M * N * K
        print(json.dumps({"M": M, "N": N, "K": K, "ms": round(ms, 4), "tflops": round(fl / ms / 1e9, 1),
                          "cublas_ms": round(ms_ref, 4), "cublas_tflops": round(fl / ms_ref / 1e9, 1),
                          "rel_err_vs_cublas": round(rel, 5), "err_flag": int(err.item())}))
        del A, B, Cm, ref
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()


def quant_main(argv=None):
    """Quantized weights at prefill: dequantize-in-the-GEMM (`gemm_q`) against
    dequantize-to-bf16-then-GEMM, over M, for one Qwen3-32B-shaped projection.

      python -c "from helexa_b200.bench.gemm_bench import quant_main; quant_main()"
    """
    from .. import ops
    from ..models.fast import GGUF_Q4_K, GGUF_Q6_K, GGUF_Q8_0, QWeight
    ap = argparse.ArgumentParser()
    ap.add_argument("--n", type=int, default=10240)
    ap.add_argument("--k", type=int, default=5120)
    ap.add_argument("--ms", default="16,64,128,256,512,1024")
    args = ap.parse_args(argv)
    C = ops.C
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    W = torch.randn(args.n, args.k, device="cuda", dtype=torch.bfloat16) * 0.05
    for name, t in (("Q4_K", GGUF_Q4_K), ("Q6_K", GGUF_Q6_K), ("Q8_0", GGUF_Q8_0)):
        qw = QWeight(C.gguf_quant(W, t), t, args.k)
        for M in (int(m) for m in args.ms.split(",")):
            A = torch.randn(M, args.k, device="cuda", dtype=torch.bfloat16)
            out = torch.empty(M, args.n, device="cuda", dtype=torch.bfloat16)
            t_fused = bench(lambda: C.gemm_q(A, qw.raw, qw.type, args.k, out, 0, err))
            t_scratch = bench(lambda: C.gemm(A, qw.dequant(C), out, 0, err))
            print(json.dumps({"type": name, "M": M, "N": args.n, "K": args.k, "fused_ms": round(t_fused, 4),
                              "scratch_ms": round(t_scratch, 4)}))
    assert err.item() == 0
