"""Tensor-parallel sharding on CPU ranks (gloo, world size 2 and 4).

Each rank builds its shard of the fused layout (column/row splits, GDN head split,
per-expert intermediate split, KV-head replication when ranks > KV heads) and runs
the torch-op prefill; the all-reduced result must equal the single-rank model, as
the reference checks its TP MoE partial sums on CPU (tp/tp_qwen3_5.rs:2466-2496).
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, ws, port, name, q, ep=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        import helexa_b200.models.fast as F
        from helexa_b200.config import get_preset
        from helexa_b200.parallel.tp import TPComm
        from helexa_b200.weights.random_init import random_weights
        from test_fast_model_gpu import _realistic
        F._allow_cpu_prefill = True
        cfg = get_preset(name)
        torch.manual_seed(0)
        w = _realistic(cfg, random_weights(cfg, seed=0, std=0.05))
        comm = TPComm(device=torch.device("cpu"))
        fm = F.FastModel.from_hf(cfg, w, "cpu", rank=rank, ws=ws, max_slots=1, max_len=128, comm=comm, ep=ep)
        prompt = torch.randint(0, cfg.vocab_size, (70,), generator=torch.Generator().manual_seed(1)).int()
        out = fm.prefill(0, prompt, 0)
        # a numpy copy travels by value (a tensor would be shared through the child's
        # resource sharer, which goes away when the child exits)
        q.put((rank, out.float().numpy()))
        dist.barrier()  # no rank tears gloo down while a peer's last message is in flight
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("name,ws,ep", [("tiny-qwen3-next", 2, False), ("tiny-qwen3-next", 4, False),
                                        ("tiny-qwen3-moe", 2, False), ("tiny-qwen3-moe", 2, True),
                                        ("tiny-qwen3-moe", 4, True), ("tiny-qwen3-moe-wide", 8, True),
                                        ("tiny-qwen3-moe-wide", 8, False)])
def test_tp_matches_single_rank(name, ws, ep):
    """Tensor-parallel (and, with ep, expert-parallel MoE) prefill on gloo ranks against
    the single-rank model."""
    import helexa_b200.models.fast as F
    from helexa_b200.config import get_preset
    from helexa_b200.weights.random_init import random_weights
    from test_fast_model_gpu import _realistic
    F._allow_cpu_prefill = True
    try:
        cfg = get_preset(name)
        torch.manual_seed(0)
        w = _realistic(cfg, random_weights(cfg, seed=0, std=0.05))
        fm = F.FastModel.from_hf(cfg, w, "cpu", max_slots=1, max_len=128)
        prompt = torch.randint(0, cfg.vocab_size, (70,), generator=torch.Generator().manual_seed(1)).int()
        want = fm.prefill(0, prompt, 0)
    finally:
        F._allow_cpu_prefill = False
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, ws, port, name, q, ep)) for r in range(ws)]
    for p in procs:
        p.start()
    res = {r: torch.from_numpy(a) for r, a in (q.get(timeout=300) for _ in range(ws))}
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    coss = [torch.nn.functional.cosine_similarity(res[r].float(), want.float(), dim=0).item() for r in range(ws)]
    # ranks sum bf16 partials, so rounding differs from the single-rank model and can
    # flip a near-tied expert choice; a sharding error drives the cosine far lower
    assert min(coss) > 0.985, coss
    assert torch.equal(res[0], res[ws - 1])
