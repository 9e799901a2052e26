"""Per-rank fused weight layout used by the CUDA model.

HF checkpoints store one tensor per projection; the decode kernels want as few
weight streams per layer as possible, so each rank's weights are re-laid out once
at load time:

  GDN      w_in   [2*kd + 2*vd + 2*Hv, H]   rows = q | k | v | z | b | a (local heads)
                                             (de-interleaves the checkpoint's per-key-head
                                             `in_proj_qkvz` / `in_proj_ba` groups, cf.
                                             tp/tp_qwen3_5.rs:2501-2577 split_fused_qkvz)
           conv_w [C, K] f32 (C = local q|k|v channels), out_w [H, vd]
  attn     w_qkv  [Hq*qw + 2*Hkv*D, H]      rows = q(+gate per head) | k | v
           o_w    [H, Hq*D]
  MoE      router [E(+1), H]                 last row = shared_expert_gate when present
           w_gu   [E(+1), 2*I, H]            rows interleaved gate0, up0, gate1, up1, ...
           w_d    [E(+1), H, I]              the shared expert is appended as expert E
  MLP      w_gu   [2*I, H] interleaved, w_d [H, I]
  norms    f32, with the "(1+w)" offset folded in

Tensor parallelism (Megatron column/row split, tp/tp_linear.rs:151-294): column
shards take row blocks, row-parallel shards take column blocks, GDN shards by key
heads (value heads follow, tp/tp_qwen3_5.rs:133-161), attention by query heads with
KV heads replicated when ws > Hkv (the reference refuses that case,
tp/tp_qwen3_5.rs:564-569), MoE experts along the intermediate dim
(tp/tp_qwen3_5.rs:797-808).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..config import ModelConfig


@dataclass
class LocalDims:
    ws: int
    rank: int
    H: int
    hq: int = 0
    hkv: int = 0
    kv_head0: int = 0     # first global kv head this rank holds
    D: int = 0
    qw: int = 0           # per-head q-proj width (2D when gated)
    hk: int = 0
    hv: int = 0
    dk: int = 0
    dv: int = 0
    inter: int = 0        # dense MLP shard
    inter0: int = 0       # first intermediate column of this rank's shard
    moe_inter: int = 0    # per-expert shard
    shared_inter: int = 0
    ep: bool = False      # expert parallel: whole experts e0 .. e0 + e_local - 1 on this rank
    e0: int = 0
    e_local: int = 0

    @property
    def gdn_kd(self) -> int:
        return self.hk * self.dk

    @property
    def gdn_vd(self) -> int:
        return self.hv * self.dv

    @property
    def gdn_conv(self) -> int:
        return 2 * self.gdn_kd + self.gdn_vd

    @property
    def gdn_in_rows(self) -> int:
        return 2 * self.gdn_kd + 2 * self.gdn_vd + 2 * self.hv

    @property
    def qkv_rows(self) -> int:
        return self.hq * self.qw + 2 * self.hkv * self.D


def block_split(n: int, block: int, ws: int, rank: int) -> tuple[int, int]:
    """(start, size) of rank's share of n columns split on `block` boundaries: whole
    blocks, as even as possible (the first n/block mod ws ranks get one block more).
    With block = 1 and n divisible by ws this is the even Megatron split."""
    nb = n // block
    lo = rank * nb // ws
    hi = (rank + 1) * nb // ws
    return lo * block, (hi - lo) * block


def local_dims(cfg: ModelConfig, rank: int = 0, ws: int = 1, ep: bool = False, inter_block: int = 1) -> LocalDims:
    """Per-rank shard sizes. With `ep` (expert parallelism, ws > 1) each rank holds
    whole experts E/ws .. instead of an intermediate slice of every expert; attention,
    GDN and dense layers stay tensor-parallel. `inter_block`: the dense MLP's
    intermediate dim splits on multiples of this (256 for k-quant GGUF weights, whose
    row-parallel down projection must hold whole superblocks: Qwen3-32B's 25600 over 8
    ranks gives 12 or 13 superblocks per rank)."""
    d = LocalDims(ws=ws, rank=rank, H=cfg.hidden_size)
    if cfg.num_full_layers:
        if cfg.num_attention_heads % ws:
            raise ValueError(f"{cfg.num_attention_heads} query heads do not split over {ws} ranks")
        d.hq = cfg.num_attention_heads // ws
        d.D = cfg.head_dim
        d.qw = 2 * cfg.head_dim if cfg.attn_output_gate else cfg.head_dim
        if cfg.num_key_value_heads >= ws:
            if cfg.num_key_value_heads % ws:
                raise ValueError("kv heads do not split evenly")
            d.hkv = cfg.num_key_value_heads // ws
            d.kv_head0 = rank * d.hkv
        else:
            if ws % cfg.num_key_value_heads:
                raise ValueError("ranks must be a multiple of kv heads for replication")
            d.hkv = 1
            d.kv_head0 = rank * cfg.num_key_value_heads // ws
    if cfg.num_linear_layers:
        if cfg.linear_num_key_heads % ws:
            raise ValueError(f"{cfg.linear_num_key_heads} GDN key heads do not split over {ws} ranks")
        d.hk = cfg.linear_num_key_heads // ws
        d.hv = cfg.linear_num_value_heads // ws
        d.dk, d.dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
    if cfg.intermediate_size:
        if cfg.intermediate_size % inter_block:
            raise ValueError(f"intermediate {cfg.intermediate_size} is not a multiple of {inter_block}")
        d.inter0, d.inter = block_split(cfg.intermediate_size, inter_block, ws, rank)
    if cfg.num_experts and ep and ws > 1:
        if cfg.num_experts % ws:
            raise ValueError(f"{cfg.num_experts} experts do not split over {ws} ranks")
        if cfg.shared_expert_intermediate_size:
            raise ValueError("expert parallelism needs a model without a shared expert")
        d.ep, d.e_local = True, cfg.num_experts // ws
        d.e0 = rank * d.e_local
        d.moe_inter = cfg.moe_intermediate_size
    elif cfg.num_experts:
        if cfg.moe_intermediate_size % ws:
            raise ValueError("moe_intermediate_size does not split")
        d.moe_inter = cfg.moe_intermediate_size // ws
        d.shared_inter = cfg.shared_expert_intermediate_size // ws
    return d


def _rows(t: torch.Tensor, n: int, i: int) -> torch.Tensor:
    step = t.shape[0] // n
    return t[i * step:(i + 1) * step]


def _cols(t: torch.Tensor, n: int, i: int) -> torch.Tensor:
    step = t.shape[1] // n
    return t[:, i * step:(i + 1) * step]


def interleave_rows(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """[I, H] x2 -> [2I, H] with rows g0, u0, g1, u1, ..."""
    return torch.stack([g, u], 1).reshape(-1, g.shape[1])


def norm_f32(cfg: ModelConfig, w: torch.Tensor) -> torch.Tensor:
    return w.float() + cfg.norm_offset


def fuse_layer(cfg: ModelConfig, dims: LocalDims, i: int, get, dtype=torch.bfloat16) -> dict[str, torch.Tensor]:
    """Build the fused tensors of layer i for this rank. `get(name)` returns an HF tensor."""
    ws, r = dims.ws, dims.rank
    p = f"model.layers.{i}."
    out: dict[str, torch.Tensor] = {
        "ln1": norm_f32(cfg, get(p + "input_layernorm.weight")),
        "ln2": norm_f32(cfg, get(p + "post_attention_layernorm.weight")),
    }
    if cfg.is_linear(i):
        q = p + "linear_attn."
        Hk, Hv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        Dk, Dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        rr = Hv // Hk
        W = get(q + "in_proj_qkvz.weight").view(Hk, 2 * Dk + 2 * rr * Dv, -1)
        Wba = get(q + "in_proj_ba.weight").view(Hk, 2 * rr, -1)
        ks = slice(r * dims.hk, (r + 1) * dims.hk)
        Wl, Wbal = W[ks], Wba[ks]
        Hd = W.shape[-1]
        wq = Wl[:, :Dk].reshape(-1, Hd)
        wk = Wl[:, Dk:2 * Dk].reshape(-1, Hd)
        wv = Wl[:, 2 * Dk:2 * Dk + rr * Dv].reshape(-1, Hd)
        wz = Wl[:, 2 * Dk + rr * Dv:].reshape(-1, Hd)
        wb = Wbal[:, :rr].reshape(-1, Hd)
        wa = Wbal[:, rr:].reshape(-1, Hd)
        out["w_in"] = torch.cat([wq, wk, wv, wz, wb, wa], 0).to(dtype).contiguous()
        cw = get(q + "conv1d.weight").reshape(cfg.gdn_conv_dim, -1)
        kd = cfg.gdn_key_dim
        cq = cw[:kd].view(Hk, Dk, -1)[ks].reshape(-1, cw.shape[1])
        ck = cw[kd:2 * kd].view(Hk, Dk, -1)[ks].reshape(-1, cw.shape[1])
        cv = cw[2 * kd:].view(Hv, Dv, -1)[r * dims.hv:(r + 1) * dims.hv].reshape(-1, cw.shape[1])
        out["conv_w"] = torch.cat([cq, ck, cv], 0).float().contiguous()
        vs = slice(r * dims.hv, (r + 1) * dims.hv)
        out["A_log"] = get(q + "A_log").float()[vs].contiguous()
        out["dt_bias"] = get(q + "dt_bias").float()[vs].contiguous()
        out["gnorm"] = get(q + "norm.weight").float().contiguous()
        out["out_w"] = _cols(get(q + "out_proj.weight"), ws, r).to(dtype).contiguous()
    else:
        q = p + "self_attn."
        D = cfg.head_dim
        Wq = get(q + "q_proj.weight").view(cfg.num_attention_heads, dims.qw, -1)
        Wq = Wq[r * dims.hq:(r + 1) * dims.hq].reshape(-1, Wq.shape[-1])
        Wk = get(q + "k_proj.weight").view(cfg.num_key_value_heads, D, -1)
        Wv = get(q + "v_proj.weight").view(cfg.num_key_value_heads, D, -1)
        kv = slice(dims.kv_head0, dims.kv_head0 + dims.hkv)
        Wk = Wk[kv].reshape(-1, Wk.shape[-1])
        Wv = Wv[kv].reshape(-1, Wv.shape[-1])
        out["w_qkv"] = torch.cat([Wq, Wk, Wv], 0).to(dtype).contiguous()
        out["o_w"] = _cols(get(q + "o_proj.weight"), ws, r).to(dtype).contiguous()
        if cfg.qk_norm:
            out["q_norm"] = norm_f32(cfg, get(q + "q_norm.weight")).contiguous()
            out["k_norm"] = norm_f32(cfg, get(q + "k_norm.weight")).contiguous()
    m = p + "mlp."
    if cfg.layer_uses_moe(i):
        E = cfg.num_experts
        rw = [get(m + "gate.weight")]
        has_shared = cfg.shared_expert_intermediate_size > 0
        if has_shared:
            rw.append(get(m + "shared_expert_gate.weight"))
        out["router"] = torch.cat(rw, 0).to(dtype).contiguous()
        gus, ds = [], []
        # expert parallel: this rank's whole experts; tensor parallel: a slice of each
        experts, es, er = (range(dims.e0, dims.e0 + dims.e_local), 1, 0) if dims.ep else (range(E), ws, r)
        for e in experts:
            pre = m + f"experts.{e}."
            gus.append(interleave_rows(_rows(get(pre + "gate_proj.weight"), es, er),
                                       _rows(get(pre + "up_proj.weight"), es, er)))
            ds.append(_cols(get(pre + "down_proj.weight"), es, er))
        if has_shared:
            if cfg.shared_expert_intermediate_size != cfg.moe_intermediate_size:
                raise ValueError("the fused expert stack needs shared_expert_intermediate_size == "
                                 "moe_intermediate_size")
            pre = m + "shared_expert."
            gus.append(interleave_rows(_rows(get(pre + "gate_proj.weight"), ws, r),
                                       _rows(get(pre + "up_proj.weight"), ws, r)))
            ds.append(_cols(get(pre + "down_proj.weight"), ws, r))
        out["w_gu"] = torch.stack(gus).to(dtype).contiguous()
        out["w_d"] = torch.stack(ds).to(dtype).contiguous()
    else:
        i0, i1 = dims.inter0, dims.inter0 + dims.inter
        out["w_gu"] = interleave_rows(get(m + "gate_proj.weight")[i0:i1],
                                      get(m + "up_proj.weight")[i0:i1]).to(dtype).contiguous()
        out["w_d"] = get(m + "down_proj.weight")[:, i0:i1].to(dtype).contiguous()
    return out


def layer_shapes(cfg: ModelConfig, dims: LocalDims, i: int) -> dict[str, tuple[tuple[int, ...], torch.dtype]]:
    """Shapes/dtypes of fuse_layer's output, for direct random init on the device."""
    H = dims.H
    bf, f32 = torch.bfloat16, torch.float32
    s: dict[str, tuple[tuple[int, ...], torch.dtype]] = {"ln1": ((H,), f32), "ln2": ((H,), f32)}
    if cfg.is_linear(i):
        s.update(w_in=((dims.gdn_in_rows, H), bf), conv_w=((dims.gdn_conv, cfg.linear_conv_kernel_dim), f32),
                 A_log=((dims.hv,), f32), dt_bias=((dims.hv,), f32), gnorm=((dims.dv,), f32),
                 out_w=((H, dims.gdn_vd), bf))
    else:
        s.update(w_qkv=((dims.qkv_rows, H), bf), o_w=((H, dims.hq * dims.D), bf))
        if cfg.qk_norm:
            s.update(q_norm=((dims.D,), f32), k_norm=((dims.D,), f32))
    if cfg.layer_uses_moe(i):
        extra = 1 if cfg.shared_expert_intermediate_size else 0
        ne = dims.e_local if dims.ep else cfg.num_experts + extra
        s.update(router=((cfg.num_experts + extra, H), bf),
                 w_gu=((ne, 2 * dims.moe_inter, H), bf),
                 w_d=((ne, H, dims.moe_inter), bf))
    else:
        s.update(w_gu=((2 * dims.inter, H), bf), w_d=((H, dims.inter), bf))
    return s
