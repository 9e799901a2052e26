"""GGUF: host k-quant codecs (C++), container write/read, GPU fused-dequant GEMV."""
import os

import numpy as np
import pytest
import torch

from helexa_b200.weights import gguf as G


def _C():
    from helexa_b200 import ops
    return ops.C


@pytest.mark.parametrize("gt,tol", [(G.Q8_0, 0.01), (G.Q4_K, 0.12), (G.Q6_K, 0.03)])
def test_host_quant_roundtrip(gt, tol):
    torch.manual_seed(0)
    x = torch.randn(4 * 256 * 8) * 0.02
    raw = _C().gguf_quant_host(x, gt)
    bb, bv = G.BLOCK[gt]
    assert raw.numel() == x.numel() // bv * bb
    y = _C().gguf_dequant_host(raw, gt, x.numel())
    rel = ((y - x).norm() / x.norm()).item()
    assert rel < tol, rel
    # quantizing the decoded values again is (almost) a fixed point
    y2 = _C().gguf_dequant_host(_C().gguf_quant_host(y, gt), gt, x.numel())
    assert ((y2 - y).norm() / y.norm()).item() < tol


def test_q6k_block_layout_by_hand():
    """Decode one hand-built Q6_K block: every value must land in its documented slot."""
    b = np.zeros(210, dtype=np.uint8)
    q = (np.arange(256) % 64).astype(np.int64)       # unsigned 6-bit codes
    sc = np.arange(1, 17, dtype=np.int8)
    for half in range(2):
        qq = q[128 * half:128 * half + 128]
        for l in range(32):
            q1, q2, q3, q4 = qq[l], qq[l + 32], qq[l + 64], qq[l + 96]
            b[64 * half + l] = (q1 & 15) | ((q3 & 15) << 4)
            b[64 * half + l + 32] = (q2 & 15) | ((q4 & 15) << 4)
            b[128 + 32 * half + l] = (q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6)
    b[192:208] = sc.view(np.uint8)
    b[208:210] = np.frombuffer(np.float16(0.5).tobytes(), dtype=np.uint8)
    y = _C().gguf_dequant_host(torch.from_numpy(b.copy()), G.Q6_K, 256).numpy()
    want = np.array([0.5 * sc[j // 16] * (q[j] - 32) for j in range(256)], dtype=np.float32)
    np.testing.assert_allclose(y, want)


def test_gguf_file_roundtrip(tmp_path):
    torch.manual_seed(1)
    w = torch.randn(64, 512) * 0.02
    n = torch.randn(512) * 0.02 + 1
    path = os.path.join(tmp_path, "m.gguf")
    meta = {"general.architecture": "qwen3", "general.name": "tiny", "qwen3.block_count": 1,
            "qwen3.embedding_length": 512, "qwen3.attention.head_count": 4, "qwen3.attention.head_count_kv": 2,
            "qwen3.feed_forward_length": 1024, "qwen3.context_length": 4096}
    G.write_gguf(path, meta, [("blk.0.attn_q.weight", w, G.Q4_K), ("blk.0.attn_norm.weight", n, G.F32),
                              ("blk.0.attn_k.weight", w, G.Q6_K), ("blk.0.attn_v.weight", w, G.Q8_0)])
    g = G.GGUFFile(path)
    assert g.meta["general.name"] == "tiny" and g.tensors["blk.0.attn_q.weight"].shape == (64, 512)
    assert torch.equal(g.tensor("blk.0.attn_norm.weight"), n)
    for name, tol in (("blk.0.attn_q.weight", 0.12), ("blk.0.attn_k.weight", 0.03), ("blk.0.attn_v.weight", 0.01)):
        assert ((g.tensor(name) - w).norm() / w.norm()).item() < tol
    cfg = g.model_config()
    assert cfg.hidden_size == 512 and cfg.num_key_value_heads == 2 and cfg.head_dim == 128
    assert G.hf_to_gguf_name("model.layers.3.mlp.down_proj.weight") == "blk.3.ffn_down.weight"
    assert g.hf_get("model.layers.0.self_attn.q_proj.weight").shape == (64, 512)
    g.close()


@pytest.mark.gpu
@pytest.mark.parametrize("gt", [G.Q8_0, G.Q4_K, G.Q6_K, 114])
@pytest.mark.parametrize("B,mode", [(1, 0), (2, 1), (1, 2), (4, 3), (8, 0)])
def test_gguf_gemv_and_dequant(gt, B, mode):
    """Decode GEMV straight from the block bytes (the wide 16-byte-per-lane kernels for
    Q4_K and padded Q6_K = type 114) and the prefill dequantization, against the host
    codec's dequantized weights."""
    C = _C()
    torch.manual_seed(2)
    N, K = 384, 2048 + 256 * (gt == 114)
    w = torch.randn(N, K) * 0.02
    host_t = G.Q6_K if gt == 114 else gt
    raw = C.gguf_quant_host(w.view(-1), host_t).view(N, -1).cuda()
    wd = C.gguf_dequant_host(raw.cpu().view(-1), host_t, N * K).view(N, K).cuda()
    if gt == 114:
        raw = C.gguf_pad_q6k(raw)
        assert raw.shape[1] == K // 256 * 224
    out = torch.empty(N, K, dtype=torch.bfloat16, device="cuda")
    C.gguf_dequant(raw, gt, K, out)
    torch.testing.assert_close(out.float(), wd, atol=1e-3, rtol=1e-2)
    x = torch.randn(B, K, device="cuda").bfloat16()
    ref = x.float() @ wd.t()
    if mode == 2:
        y = torch.empty(B, N // 2, device="cuda", dtype=torch.bfloat16)
        want = torch.nn.functional.silu(ref[:, 0::2]) * ref[:, 1::2]
    elif mode == 3:
        y = torch.empty(B, N, device="cuda")
        want = ref
    else:
        y = torch.zeros(B, N, device="cuda", dtype=torch.bfloat16)
        want = ref
    C.gguf_gemv(raw, gt, K, x, y, mode, y if mode == 1 else None, None, 0.0)
    torch.cuda.synchronize()
    err = (y.float() - want).abs().max().item()
    assert err <= 2e-2 * want.abs().max().item() + 1e-3, err


@pytest.mark.gpu
@pytest.mark.parametrize("gt,tol", [(G.Q8_0, 0.01), (G.Q4_K, 0.12), (G.Q6_K, 0.03)])
def test_device_quantizer_matches_host_codec(gt, tol):
    """In-situ quantization on the GPU writes the host codec's block bytes, and the
    decoded weights stay within the codec tolerance of the input."""
    C = _C()
    torch.manual_seed(4)
    N, K = 96, 1024
    w = (torch.randn(N, K) * 0.03).bfloat16()
    host = C.gguf_quant_host(w.float().view(-1), gt).view(N, -1)
    dev = C.gguf_quant(w.cuda(), gt).cpu()
    assert dev.shape == host.shape
    wd = C.gguf_dequant_host(dev.reshape(-1), gt, N * K).view(N, K)
    wh = C.gguf_dequant_host(host.reshape(-1), gt, N * K).view(N, K)
    rel = (wd - w.float()).norm() / w.float().norm()
    assert rel < tol, rel
    assert torch.equal(wd, wh)
    assert torch.equal(dev, host)


@pytest.mark.gpu
@pytest.mark.parametrize("name,scheme", [("tiny-qwen3", "Q8_0"), ("tiny-qwen3", "Q4_K_M"),
                                         ("tiny-qwen3-next", "Q6_K")])
def test_quantized_model_matches_dequantized_weights(name, scheme):
    """A quantized FastModel (fused-dequant decode GEMVs, dequant-then-GEMM prefill)
    against the same model holding the dequantized bf16 weights: prefill logits and
    teacher-forced graph decode logits agree."""
    from helexa_b200.config import get_preset
    from helexa_b200.models.fast import FastModel, QWeight
    from helexa_b200.weights.random_init import random_weights
    cfg = get_preset(name)
    w = random_weights(cfg, seed=0, std=0.05)
    dev = torch.device("cuda", 0)
    q = FastModel.from_hf(cfg, w, dev, max_slots=1, max_len=128)
    q.quantize_(scheme)
    nq = sum(isinstance(t, QWeight) for lw in q.layers for t in lw.values())
    assert nq > 0
    ref = FastModel.from_hf(cfg, w, dev, max_slots=1, max_len=128)
    for lq, lr in zip(q.layers, ref.layers):
        for k, t in lq.items():
            if isinstance(t, QWeight):
                lr[k] = t.dequant(q.C)
    prompt = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(1)).int().to(dev)
    out = []
    first = None
    for m in (q, ref):
        lg = m.prefill(0, prompt, 0).float()
        first = int(lg.argmax()) if first is None else first  # both models decode the same token
        nb = m.capture(1, steps=1)
        nb.slots.fill_(0)
        nb.tok.fill_(first)
        m.replay(nb)
        torch.cuda.synchronize()
        out.append((lg, nb.logits[0].float().clone()))
    cos = torch.nn.functional.cosine_similarity
    assert cos(out[0][0], out[1][0], dim=0).item() > 0.999
    # decode GEMVs quantize their input rows to int8 blocks: ~0.3% per-value error
    assert cos(out[0][1], out[1][1], dim=0).item() > 0.995
    assert q.weight_bytes() < ref.weight_bytes()


def _write_tiny_gguf(path, inter=768, layers=2):
    """A Q4_K_M-style dense Qwen3 file: q/k/o/gate/up Q4_K, v/down Q6_K, f32 norms,
    Q8_0 embedding, Q6_K output. hidden 256, 4 heads of 64 (2 kv heads)."""
    import dataclasses

    from helexa_b200.config import get_preset
    from helexa_b200.weights.random_init import random_weights
    cfg = dataclasses.replace(get_preset("tiny-qwen3"), intermediate_size=inter, num_hidden_layers=layers,
                              layer_types=None, tie_word_embeddings=False)
    w = random_weights(cfg, seed=2, std=0.05)
    types = {"attn_q": G.Q4_K, "attn_k": G.Q4_K, "attn_v": G.Q6_K, "attn_output": G.Q4_K, "ffn_gate": G.Q4_K,
             "ffn_up": G.Q4_K, "ffn_down": G.Q6_K}
    tensors = []
    for hf, t in w.items():
        gname = G.hf_to_gguf_name(hf)
        kind = gname.split(".")[-2] if gname.startswith("blk.") else gname
        if t.dim() == 1:
            gt = G.F32
        elif gname == "token_embd.weight":
            gt = G.Q8_0
        elif gname == "output.weight":
            gt = G.Q6_K
        else:
            gt = types[kind]
        tensors.append((gname, t, gt))
    meta = {"general.architecture": "qwen3", "general.name": "tiny-gguf", "qwen3.block_count": layers,
            "qwen3.embedding_length": cfg.hidden_size, "qwen3.attention.head_count": cfg.num_attention_heads,
            "qwen3.attention.head_count_kv": cfg.num_key_value_heads, "qwen3.attention.key_length": cfg.head_dim,
            "qwen3.feed_forward_length": inter, "qwen3.context_length": 4096, "qwen3.vocab_size": cfg.vocab_size,
            "qwen3.attention.layer_norm_rms_epsilon": cfg.rms_norm_eps, "qwen3.rope.freq_base": cfg.rope_theta}
    G.write_gguf(path, meta, tensors)
    return cfg


@pytest.mark.parametrize("ws", [1, 2])
def test_native_gguf_layout_matches_dequantized(tmp_path, ws):
    """QuantLayer keeps block rows (no host dequantization): dequantizing its per-rank
    pieces gives exactly the fused layout built from the dequantized checkpoint,
    including the uneven superblock split of down_proj (3 superblocks over 2 ranks) and
    the segmented q|k|v (Q4_K q/k, Q6_K v)."""
    from helexa_b200.models import layout
    path = os.path.join(tmp_path, "m.gguf")
    _write_tiny_gguf(path)
    g = G.GGUFFile(path)
    cfg = g.model_config()
    ql = G.QuantLayer(g)

    def deq(t):
        if isinstance(t, G.QuantRows):
            return G._dequant_rows(t)
        if isinstance(t, list):
            return torch.cat([deq(p) for p in t], 0)
        return t.float()
    sizes = []
    for r in range(ws):
        dims = layout.local_dims(cfg, r, ws, inter_block=256)
        sizes.append(dims.inter)
        want = layout.fuse_layer(cfg, dims, 1, g.hf_get, dtype=torch.float32)
        got = ql.layer(cfg, dims, 1)
        assert isinstance(got["w_gu"], G.QuantRows) and isinstance(got["w_d"], G.QuantRows)
        assert isinstance(got["w_qkv"], list) and len(got["w_qkv"]) == 2  # q|k Q4_K, v Q6_K
        for k, t in want.items():
            assert torch.equal(deq(got[k]), t.float()), (r, k)
    assert sum(sizes) == 768 and all(s % 256 == 0 for s in sizes)
    g.close()


@pytest.mark.gpu
def test_native_gguf_model_matches_dequantized(tmp_path):
    """FastModel.from_gguf serves the block rows (fused-dequant decode GEMVs, segmented
    q|k|v) and matches the model built from the dequantized checkpoint."""
    from helexa_b200.models.fast import FastModel, QWeight, QWeightCat
    path = os.path.join(tmp_path, "m.gguf")
    _write_tiny_gguf(path)
    g = G.GGUFFile(path)
    cfg = g.model_config()
    dev = torch.device("cuda", 0)
    q = FastModel.from_gguf(cfg, g, dev, max_slots=1, max_len=128)
    assert isinstance(q.layers[0]["w_qkv"], QWeightCat) and isinstance(q.layers[0]["w_d"], QWeight)
    ref = FastModel.from_hf(cfg, g.hf_get, dev, max_slots=1, max_len=128)
    prompt = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(1)).int().to(dev)
    out = []
    for m in (q, ref):
        lg = m.prefill(0, prompt, 0).float()
        nb = m.capture(1, steps=4)
        nb.slots.fill_(0)
        nb.tok.fill_(int(lg.argmax()))
        m.replay(nb)
        torch.cuda.synchronize()
        out.append((lg, nb.logits[0].float().clone()))
    cos = torch.nn.functional.cosine_similarity
    assert cos(out[0][0], out[1][0], dim=0).item() > 0.999
    assert cos(out[0][1], out[1][1], dim=0).item() > 0.995
    assert q.weight_bytes() < ref.weight_bytes()
    g.close()


@pytest.mark.gpu
@pytest.mark.parametrize("gt", [G.Q4_K, G.Q6_K])
@pytest.mark.parametrize("B,ep", [(1, False), (2, False), (2, True)])
def test_quantized_expert_kernels(gt, B, ep):
    """gate/up SwiGLU by route and down + weighted combine + residual straight from the
    block rows, against fp32 math on the dequantized stacks (expert parallel: routes to
    experts outside the rank's range contribute nothing)."""
    C = _C()
    torch.manual_seed(5)
    E, I, H, J = 6, 256, 512, 3
    wgu = torch.randn(E * 2 * I, H) * 0.02
    wd = torch.randn(E * H, I) * 0.02
    raw_gu = C.gguf_quant_host(wgu.view(-1), gt).view(E * 2 * I, -1).cuda()
    raw_d = C.gguf_quant_host(wd.view(-1), gt).view(E * H, -1).cuda()
    dq_gu = C.gguf_dequant_host(raw_gu.cpu().view(-1), gt, wgu.numel()).view(E, 2 * I, H)
    dq_d = C.gguf_dequant_host(raw_d.cpu().view(-1), gt, wd.numel()).view(E, H, I)
    t = gt
    if gt == G.Q6_K:
        raw_gu, raw_d, t = C.gguf_pad_q6k(raw_gu), C.gguf_pad_q6k(raw_d), 114
    x = torch.randn(B, H).bfloat16()
    ids = torch.randint(0, E, (B * J,), dtype=torch.int32)
    wts = torch.rand(B * J)
    e_base, e_count = (2, 3) if ep else (0, 0)
    act = torch.zeros(B * J, I, dtype=torch.bfloat16, device="cuda")
    # expert parallel: the rank holds experts [e_base, e_base + e_count) only
    lgu = raw_gu[e_base * 2 * I:(e_base + e_count) * 2 * I] if ep else raw_gu
    ld = raw_d[e_base * H:(e_base + e_count) * H] if ep else raw_d
    C.gguf_experts(lgu, t, H, x.cuda(), ids.cuda(), act, J, None, 0.0, e_base, e_count)
    xo = x.cuda().clone()
    C.gguf_moe_down(ld, t, I, act, ids.cuda(), wts.cuda(), xo, J, e_base, e_count)
    torch.cuda.synchronize()
    want_act = torch.zeros(B * J, I)
    want = x.float().clone()
    for r in range(B * J):
        e = int(ids[r])
        if ep and not (e_base <= e < e_base + e_count):
            continue
        h = dq_gu[e] @ x[r // J].float()
        a = torch.nn.functional.silu(h[0::2]) * h[1::2]
        want_act[r] = a
        want[r // J] += wts[r] * (dq_d[e] @ a)
    local = [r for r in range(B * J) if not ep or e_base <= int(ids[r]) < e_base + e_count]
    if local:
        err = (act.float().cpu()[local] - want_act[local]).abs().max().item()
        assert err <= 3e-2 * want_act[local].abs().max().item() + 1e-3, err
    err = (xo.float().cpu() - want).abs().max().item()
    assert err <= 3e-2 * (want - x.float()).abs().max().item() + 2e-2, err


@pytest.mark.gpu
def test_quantized_experts_model_matches_dequantized():
    """A MoE model with in-situ quantized expert stacks (decode: integer-dot expert
    kernels; prefill: dequantized scratch + grouped GEMM) follows the same model run
    on the dequantized stacks."""
    import dataclasses
    from helexa_b200.config import get_preset
    from helexa_b200.models.fast import FastModel, QExperts
    from helexa_b200.weights.random_init import random_weights
    cfg = dataclasses.replace(get_preset("tiny-qwen3-next"), moe_intermediate_size=256,
                              shared_expert_intermediate_size=256)
    w = random_weights(cfg, seed=0, std=0.05)
    q = FastModel.from_hf(cfg, w, "cuda", max_slots=1, max_len=128)
    q.quantize_("Q4_K_M")
    moe = [i for i in range(cfg.num_hidden_layers) if cfg.layer_uses_moe(i)]
    assert all(isinstance(q.layers[i]["w_gu"], QExperts) for i in moe)
    ref = FastModel.from_hf(cfg, w, "cuda", max_slots=1, max_len=128)
    ref.quantize_("Q4_K_M", experts=False)
    for i in moe:
        for k in ("w_gu", "w_d"):
            ref.layers[i][k] = q.layers[i][k].dequant(q.C).clone()
    prompt = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(1)).int().cuda()
    out, first = [], None
    for m in (q, ref):
        lg = m.prefill(0, prompt, 0).float()
        first = int(lg.argmax()) if first is None else first
        nb = m.capture(1, steps=1)
        nb.slots.fill_(0)
        nb.tok.fill_(first)
        m.replay(nb)
        torch.cuda.synchronize()
        out.append((lg, nb.logits[0].float().clone()))
    cos = torch.nn.functional.cosine_similarity
    assert cos(out[0][0], out[1][0], dim=0).item() > 0.9999
    assert cos(out[0][1], out[1][1], dim=0).item() > 0.995
    assert q.weight_bytes() < ref.weight_bytes()


def _write_tiny_moe_gguf(path, layers=2):
    """A qwen3moe file: attention Q4_K (v Q6_K), expert stacks gate/up Q4_K and down
    Q6_K as [E, rows, cols] tensors, f32 router and norms."""
    import dataclasses

    from helexa_b200.config import get_preset
    from helexa_b200.weights.random_init import random_weights
    cfg = dataclasses.replace(get_preset("tiny-qwen3-moe"), num_hidden_layers=layers, layer_types=None,
                              moe_intermediate_size=256, tie_word_embeddings=False)
    w = random_weights(cfg, seed=3, std=0.05)
    types = {"attn_q": G.Q4_K, "attn_k": G.Q4_K, "attn_v": G.Q6_K, "attn_output": G.Q4_K}
    tensors = []
    for hf, t in w.items():
        if ".experts." in hf:
            continue
        gname = G.hf_to_gguf_name(hf)
        kind = gname.split(".")[-2] if gname.startswith("blk.") else gname
        gt = G.F32 if t.dim() == 1 or kind == "ffn_gate_inp" else \
            G.Q8_0 if gname == "token_embd.weight" else G.Q6_K if gname == "output.weight" else types[kind]
        tensors.append((gname, t, gt))
    E = cfg.num_experts
    for i in range(layers):
        for proj, gt in (("gate_proj", G.Q4_K), ("up_proj", G.Q4_K), ("down_proj", G.Q6_K)):
            st = torch.stack([w[f"model.layers.{i}.mlp.experts.{e}.{proj}.weight"] for e in range(E)])
            tensors.append((f"blk.{i}.ffn_{proj.split('_')[0]}_exps.weight", st, gt))
    meta = {"general.architecture": "qwen3moe", "general.name": "tiny-moe-gguf", "qwen3moe.block_count": layers,
            "qwen3moe.embedding_length": cfg.hidden_size, "qwen3moe.attention.head_count": cfg.num_attention_heads,
            "qwen3moe.attention.head_count_kv": cfg.num_key_value_heads,
            "qwen3moe.attention.key_length": cfg.head_dim, "qwen3moe.feed_forward_length": cfg.intermediate_size,
            "qwen3moe.expert_count": E, "qwen3moe.expert_used_count": cfg.num_experts_per_tok,
            "qwen3moe.expert_feed_forward_length": cfg.moe_intermediate_size, "qwen3moe.context_length": 4096,
            "qwen3moe.attention.layer_norm_rms_epsilon": cfg.rms_norm_eps, "qwen3moe.rope.freq_base": cfg.rope_theta}
    G.write_gguf(path, meta, tensors)
    return cfg, w


def test_moe_gguf_names_and_expert_slices(tmp_path):
    """qwen3moe files: the config comes back as a MoE config, HF expert names resolve to
    slices of the [E, rows, cols] stacks, and the native layer keeps the stacks as
    interleaved block rows."""
    import os
    from helexa_b200.models import layout
    path = os.path.join(tmp_path, "moe.gguf")
    cfg0, w = _write_tiny_moe_gguf(path)
    g = G.GGUFFile(path)
    cfg = g.model_config()
    assert cfg.family == "qwen3_moe" and cfg.num_experts == cfg0.num_experts and cfg.moe_intermediate_size == 256
    e1 = g.hf_get("model.layers.1.mlp.experts.2.down_proj.weight")
    want = w["model.layers.1.mlp.experts.2.down_proj.weight"]
    assert e1.shape == want.shape and (e1 - want).norm() / want.norm() < 0.05
    dims = layout.local_dims(cfg, 0, 1)
    lay = G.QuantLayer(g).layer(cfg, dims, 0)
    gu, dn = lay["w_gu"], lay["w_d"]
    E, I, H = cfg.num_experts, cfg.moe_intermediate_size, cfg.hidden_size
    assert isinstance(gu, G.QuantExperts) and (gu.G, gu.R, gu.K) == (E, 2 * I, H) and gu.gtype == G.Q4_K
    assert isinstance(dn, G.QuantExperts) and (dn.G, dn.R, dn.K) == (E, H, I) and dn.gtype == G.Q6_K
    # row 2r of expert e is gate row r, row 2r + 1 is up row r
    rb = gu.raw.shape[1]
    gate = g.raw("blk.0.ffn_gate_exps.weight").view(E, I, rb)
    up = g.raw("blk.0.ffn_up_exps.weight").view(E, I, rb)
    assert torch.equal(gu.raw[(3 * 2 * I) + 2 * 5], gate[3, 5]) and torch.equal(gu.raw[3 * 2 * I + 2 * 5 + 1], up[3, 5])
    g.close()


@pytest.mark.gpu
def test_native_moe_gguf_matches_dequantized(tmp_path):
    import os
    from helexa_b200.models.fast import FastModel, QExperts
    path = os.path.join(tmp_path, "moe.gguf")
    _write_tiny_moe_gguf(path)
    g = G.GGUFFile(path)
    cfg = g.model_config()
    dev = torch.device("cuda", 0)
    q = FastModel.from_gguf(cfg, g, dev, max_slots=1, max_len=128)
    assert isinstance(q.layers[0]["w_gu"], QExperts)
    ref = FastModel.from_hf(cfg, g.hf_get, dev, max_slots=1, max_len=128)
    prompt = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(1)).int().to(dev)
    out, first = [], None
    for m in (q, ref):
        lg = m.prefill(0, prompt, 0).float()
        first = int(lg.argmax()) if first is None else first
        nb = m.capture(1, steps=1)
        nb.slots.fill_(0)
        nb.tok.fill_(first)
        m.replay(nb)
        torch.cuda.synchronize()
        out.append((lg, nb.logits[0].float().clone()))
    cos = torch.nn.functional.cosine_similarity
    assert cos(out[0][0], out[1][0], dim=0).item() > 0.999
    assert cos(out[0][1], out[1][1], dim=0).item() > 0.995
    assert q.weight_bytes() < ref.weight_bytes()
    g.close()


def test_moe_gguf_serves_on_cpu(tmp_path):
    """A qwen3moe GGUF loads through the registry on the CPU (experts split out of the
    stacks into the reference model) and answers a chat request."""
    import os
    from fastapi.testclient import TestClient
    from helexa_b200.server.app import create_app
    path = os.path.join(tmp_path, "moe.gguf")
    _write_tiny_moe_gguf(path)
    with TestClient(create_app()) as c:
        r = c.post("/models/load", json={"model_id": "m", "source": path, "device": "cpu", "max_batch": 1,
                                         "max_len": 256})
        assert r.status_code == 200, r.text
        r = c.post("/v1/chat/completions", json={"model": "m", "messages": [{"role": "user", "content": "hi"}],
                                                 "max_tokens": 3, "temperature": 0})
        assert r.status_code == 200, r.text
        assert r.json()["usage"]["completion_tokens"] >= 1
