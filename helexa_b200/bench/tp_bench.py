"""Two-or-more-rank microbenchmark of the tensor-parallel reductions (CUDA events, max
over ranks). Decode (in CUDA graphs): the plain residual GEMV, the GEMV with the
cross-rank reduction fused into its epilogue, and the separate one-shot P2P kernel.
Prefill (T=8192 x H=2048 bf16, one row-parallel output): the fused reduce-scatter +
residual + RMSNorm + all-gather kernel against NCCL all-reduce + the add/norm kernel.

  python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
      -m helexa_b200.bench.tp_bench
"""
import json
import os

import torch
import torch.distributed as dist

rank = int(os.environ["RANK"]); ws = int(os.environ["WORLD_SIZE"])
torch.cuda.set_device(rank); dev = torch.device("cuda", rank)
dist.init_process_group("nccl", device_id=dev)
from helexa_b200 import ops  # noqa: E402
from helexa_b200.parallel.tp import TPComm  # noqa: E402
C = ops.C
comm = TPComm(device=dev, mode="p2p")
def t(fn, n=100):
    for _ in range(3): fn()
    torch.cuda.synchronize(); dist.barrier()
    g = torch.cuda.CUDAGraph(); s = torch.cuda.Stream(); s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            for _ in range(n): fn()
    torch.cuda.current_stream().wait_stream(s); g.replay(); torch.cuda.synchronize(); dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(); g.replay(); e1.record(); e1.synchronize()
    return e0.elapsed_time(e1) / n * 1e3
res = {}
for N, K in [(2048, 4096 // ws), (2048, 2048)]:
    W = (torch.randn(N, K, device=dev) * 0.02).bfloat16(); inp = torch.randn(1, K, device=dev).bfloat16()
    x = torch.zeros(1, N, device=dev).bfloat16()
    res[f"gemv_resid_{N}x{K}_case{len(res)}"] = t(lambda: C.gemv(W, inp, x, ops.RESID_ADD, x, None, 0.0))
    res[f"gemv_ar_{N}x{K}"] = t(lambda: C.gemv_ar(W, inp, x, *comm.fused_args()))
    part = torch.zeros(1, N, device=dev).bfloat16()
    res[f"ar_oneshot_{N}"] = t(lambda: C.ar_oneshot(comm.bases, rank, part.view(-1), x.view(-1), None, comm.data_bytes, comm.epoch, comm.err, 1, 5.0))
def t_eager(fn, n=20):
    for _ in range(3): fn()
    torch.cuda.synchronize(); dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n): fn()
    e1.record(); e1.synchronize()
    return e0.elapsed_time(e1) / n * 1e3
T, H = 8192, 2048
stage, hbuf = comm.prefill_region(T, H)
stage.copy_(torch.randn(T * H, device=dev).bfloat16())
xs = torch.randn(T, H, device=dev).bfloat16(); w = torch.rand(H, device=dev) + 0.5
res[f"prefill_rs_norm_ag_{T}x{H}"] = t_eager(lambda: comm.rs_norm_ag(xs, w, 1e-6))
# the same step through NVLink multicast (switch-side reduction, multicast stores)
g = torch.Generator(device=dev).manual_seed(7)
part0 = torch.randn(T * H, device=dev, generator=g).bfloat16()
x0 = torch.randn(T, H, device=dev, generator=torch.Generator(device=dev).manual_seed(8)).bfloat16()
stage.copy_(part0); xa = x0.clone(); comm.rs_norm_ag(xa, w, 1e-6); torch.cuda.synchronize(); dist.barrier()
h_p2p = hbuf.view(T, H).clone()
comm.nvls, comm._pf_elems = True, 0
stage2, hbuf2 = comm.prefill_region(T, H)
res["nvls_available"] = float(comm.pf_mc != 0)
if comm.pf_mc:
    stage2.copy_(part0); xb = x0.clone(); comm.rs_norm_ag(xb, w, 1e-6); torch.cuda.synchronize(); dist.barrier()
    res["nvls_vs_p2p_max_abs_diff"] = (hbuf2.view(T, H).float() - h_p2p.float()).abs().max().item()
    res[f"prefill_rs_norm_ag_nvls_{T}x{H}"] = t_eager(lambda: comm.rs_norm_ag(xs, w, 1e-6))
elif rank == 0:
    print("nvls unavailable:", comm.nvls_error)
o = torch.randn(T, H, device=dev).bfloat16(); hh = torch.empty_like(o)
def nccl_path():
    dist.all_reduce(o)
    C.add_rmsnorm(xs, o, w, hh, 1e-6)
res[f"prefill_nccl_allreduce_add_norm_{T}x{H}"] = t_eager(nccl_path)
res["prefill_bytes_over_nvlink_per_rank_MB"] = 2 * (ws - 1) / ws * T * H * 2 / 1e6
comm.check()
r = torch.tensor(list(res.values()), device=dev); dist.all_reduce(r, op=dist.ReduceOp.MAX)
if rank == 0: print(json.dumps({k: round(v, 2) for k, v in zip(res, r.tolist())}))
comm.close(); dist.destroy_process_group()
