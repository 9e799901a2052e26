"""The CUDA model: fused per-rank weights, slot-pooled sequence state and a
graph-captured decode step built from the sm_100a kernels in csrc/.

State lives in preallocated pools indexed by a slot id, so batched decode works on
any subset of live sequences without the reference's assemble/extract copies
(harness/engine.rs:691-877, arch/qwen3_5/snapshot.rs:200-311):

  pos       int32 [S]                 position of each slot's next token
  kc, vc    bf16  [S, Hkv, maxlen, D] per full-attention layer (contiguous, never
                                      re-concatenated -- the ref's ConcatKvCache
                                      reallocates on every append, full_attn.rs:156)
  conv      bf16  [S, C, K]           GDN conv inputs, ring indexed by position % K
  rec       f32   [S, Hv, Dk, Dv]     GDN recurrent state

A decode step (one token for each of B slots) is: embed -> per layer
{norm-fused GEMV, fused token mixer, residual GEMV, MoE/MLP} -> norm-fused lm_head
GEMV -> on-device arg-max that advances the slot positions. Every launch reads its
dynamic inputs (token ids, slots, positions) from device memory, so the whole step
is captured once per batch size and replayed.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Callable

import torch

from .. import ops
from ..config import ModelConfig
from . import layout


# Tests of the prefill layout logic (pure torch ops) may build the model on the CPU.
_allow_cpu_prefill = False


class PhaseTimer:
    """Accumulates device time per named phase from CUDA events (mark() starts a phase)."""

    def __init__(self):
        self.events: list[tuple[str, torch.cuda.Event]] = []

    def mark(self, name: str):
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.events.append((name, e))

    def totals(self) -> dict[str, float]:
        self.mark("_end")
        self.events[-1][1].synchronize()
        out: dict[str, float] = {}
        for (n, a), (_, b) in zip(self.events, self.events[1:]):
            out[n] = out.get(n, 0.0) + a.elapsed_time(b)
        self.events = []
        return {k: round(v, 3) for k, v in out.items()}


@dataclass
class DecodeBuffers:
    B: int
    tok: torch.Tensor          # int32 [B] current input token -> next token
    slots: torch.Tensor        # int32 [B]
    x: torch.Tensor            # bf16 [B, H] residual stream
    proj_gdn: torch.Tensor | None
    gdn_out: torch.Tensor | None
    proj_attn: torch.Tensor | None
    attn_out: torch.Tensor | None
    part_o: torch.Tensor | None
    part_ml: torch.Tensor | None
    counters: torch.Tensor | None
    rlogits: torch.Tensor | None
    ids: torch.Tensor | None
    wts: torch.Tensor | None
    act_moe: torch.Tensor | None   # bf16 [B*J, moe_inter]
    act_mlp: torch.Tensor | None   # bf16 [B, inter]
    partial: torch.Tensor      # bf16 [B, H] row-parallel partial sums (TP)
    logits: torch.Tensor       # f32 [B, V]
    out_tokens: torch.Tensor   # int32 [B, cap]
    step: torch.Tensor         # int32 [B]
    best: torch.Tensor         # int64 [B] packed arg-max words (self-resetting)
    counter: torch.Tensor      # int32 [1] last-CTA election (self-resetting)
    err: torch.Tensor          # int32 [1] bounded-wait error code
    graph: torch.cuda.CUDAGraph | None = None
    graph_steps: int = 0
    sgraph: torch.cuda.CUDAGraph | None = None    # sampled decode (on-device sampler)
    sgraph_steps: int = 0
    logits_full: torch.Tensor | None = None       # f32 [B, V] (vocab-parallel gather target)
    _gather_buf: torch.Tensor | None = None


class SamplerState:
    """Per-slot parameters and penalty history of the on-device sampler
    (csrc/sample_device.cu), read by the captured sampled-decode graphs."""

    HIST = 64

    def __init__(self, slots: int, device):
        f32, i32, i64 = torch.float32, torch.int32, torch.int64
        self.temp = torch.zeros(slots, dtype=f32, device=device)
        self.top_k = torch.zeros(slots, dtype=i32, device=device)
        self.top_p = torch.ones(slots, dtype=f32, device=device)
        self.penalty = torch.ones(slots, dtype=f32, device=device)
        self.seed = torch.zeros(slots, dtype=i64, device=device)
        self.ctr = torch.zeros(slots, dtype=i64, device=device)
        self.hist = torch.zeros(slots, self.HIST, dtype=i32, device=device)
        self.hist_n = torch.zeros(slots, dtype=i32, device=device)
        self.hist_at = torch.zeros(slots, dtype=i32, device=device)
        self.hist_cap = torch.full((slots,), self.HIST, dtype=i32, device=device)

    def tensors(self):
        return (self.temp, self.top_k, self.top_p, self.penalty, self.seed, self.ctr, self.hist, self.hist_n,
                self.hist_at, self.hist_cap)

    def set_slot(self, slot: int, temperature: float, top_k: int, top_p: float, penalty: float, last_n: int,
                 seed: int, draws: int, history: list[int]):
        """Load one sequence's sampling parameters and its last `last_n` tokens."""
        cap = max(1, min(int(last_n), self.HIST))
        h = list(history[-cap:]) if penalty != 1.0 else []
        self.temp[slot] = float(temperature)
        self.top_k[slot] = int(top_k)
        self.top_p[slot] = float(top_p)
        self.penalty[slot] = float(penalty)
        self.seed[slot] = int(seed) & ((1 << 63) - 1)
        self.ctr[slot] = int(draws)
        row = torch.zeros(self.HIST, dtype=torch.int32)
        if h:
            row[:len(h)] = torch.tensor(h, dtype=torch.int32)
        self.hist[slot].copy_(row, non_blocking=False)
        self.hist_n[slot] = len(h)
        self.hist_at[slot] = len(h) % cap
        self.hist_cap[slot] = cap

    def snapshot(self):
        return [t.clone() for t in self.tensors()]

    def restore(self, saved):
        for t, v in zip(self.tensors(), saved):
            t.copy_(v)


# GGUF type ids (ggml): the block formats the kernels read
GGUF_Q8_0, GGUF_Q4_K, GGUF_Q6_K = 8, 12, 14
GGUF_Q6_K_PADDED = 114  # device-side Q6_K with superblocks padded to 224 bytes
_GGUF_BLOCK = {GGUF_Q8_0: (34, 32), GGUF_Q4_K: (144, 256), GGUF_Q6_K: (210, 256)}
# quantization schemes -> type per fused weight (Q4_K_M: ffn_down in Q6_K, the rest Q4_K;
# the fused [q|k|v] projection keeps one type, so attn_v is Q4_K here)
QUANT_SCHEMES = {
    "Q8_0": {"*": GGUF_Q8_0},
    "Q6_K": {"*": GGUF_Q6_K},
    "Q4_K": {"*": GGUF_Q4_K},
    "Q4_K_M": {"*": GGUF_Q4_K, "w_d": GGUF_Q6_K},
}


class DeviceError(RuntimeError):
    """A kernel's bounded wait ran out (code 1000+peer / 2000+peer: a tensor-parallel
    peer never arrived; other codes: a GEMM pipeline wait)."""

    def __init__(self, code: int):
        what = f"tensor-parallel peer {code % 1000} never arrived" if code >= 1000 else "GEMM pipeline wait ran out"
        super().__init__(f"device error {code}: {what}")
        self.code = code


class QWeight:
    """One linear weight held as GGUF block rows on the device (uint8 [N, row_bytes]):
    decode reads it through the fused-dequant GEMV, prefill dequantizes it to bf16
    for the tensor-core GEMM (the reference's QMatMul / dequant-then-GEMM switch,
    tp/tp_linear.rs:76-139)."""

    def __init__(self, raw: torch.Tensor, gtype: int, K: int):
        if gtype == GGUF_Q6_K and raw.is_cuda:
            # 210-byte Q6_K superblocks -> a 224-byte stride (same bytes, 16-byte aligned)
            # so the wide-load GEMV can read them
            raw, gtype = ops.C.gguf_pad_q6k(raw.contiguous()), GGUF_Q6_K_PADDED
        self.raw, self.type, self.K = raw, gtype, K

    @property
    def shape(self):
        return (self.raw.shape[0], self.K)

    def nbytes(self) -> int:
        return self.raw.numel()

    def dequant(self, C) -> torch.Tensor:
        out = torch.empty(self.raw.shape[0], self.K, dtype=torch.bfloat16, device=self.raw.device)
        C.gguf_dequant(self.raw, self.type, self.K, out)
        return out


class QWeightCat:
    """Row segments of different GGUF block types forming one projection (Q4_K_M keeps
    attn_v in Q6_K beside Q4_K q/k): the decode GEMV runs once per segment into a
    column slice of the output; prefill dequantizes and concatenates."""

    def __init__(self, parts: list):
        self.parts = parts

    @property
    def shape(self):
        return (sum(p.shape[0] for p in self.parts), self.parts[0].shape[1])

    def nbytes(self) -> int:
        return sum(_tbytes(p) for p in self.parts)

    def dequant(self, C) -> torch.Tensor:
        return torch.cat([p.dequant(C) if isinstance(p, QWeight) else p for p in self.parts], 0)


class QExperts:
    """Stacked MoE expert weights [G, R, K] held as GGUF block rows (uint8 [G * R,
    row_bytes]; G = routed experts plus the shared expert at index E). Decode reads
    them through the quantized expert kernels (gguf_experts / gguf_moe_down); prefill
    dequantizes the whole stack into a bf16 scratch shared by every layer and runs the
    grouped tcgen05 GEMM on it (the reference's moe_gemm_gguf serves these blocks,
    tp/tp_qwen3_5.rs:1153-1231)."""

    def __init__(self, raw: torch.Tensor, gtype: int, G: int, R: int, K: int):
        if gtype == GGUF_Q6_K and raw.is_cuda:
            raw, gtype = ops.C.gguf_pad_q6k(raw.contiguous()), GGUF_Q6_K_PADDED
        self.raw, self.type, self.G, self.R, self.K = raw, gtype, G, R, K

    @property
    def shape(self):
        return (self.G, self.R, self.K)

    def nbytes(self) -> int:
        return self.raw.numel()

    def expert_bytes(self) -> int:
        return self.raw.numel() // self.G

    def dequant(self, C, out: torch.Tensor | None = None) -> torch.Tensor:
        """bf16 [G, R, K] (into `out`'s storage when given)."""
        n = self.G * self.R * self.K
        if out is None or out.numel() < n:
            out = torch.empty(n, dtype=torch.bfloat16, device=self.raw.device)
        v = out.view(-1)[:n].view(self.G * self.R, self.K)
        C.gguf_dequant(self.raw, self.type, self.K, v)
        return v.view(self.G, self.R, self.K)


def _extra_launches(w) -> int:
    """Launches a quantized weight adds over one GEMV: the activation quantization in
    front of each integer-dot GEMV, one GEMV per row segment, and for expert stacks
    the quantization in front of the down projection as well."""
    if isinstance(w, QExperts):
        return 2
    if isinstance(w, QWeightCat):
        return len(w.parts) - 1 + sum(_extra_launches(p) for p in w.parts)
    if isinstance(w, QWeight):
        return 1 if w.type in (GGUF_Q4_K, GGUF_Q6_K_PADDED) and w.K % 256 == 0 else 0
    return 0


def _tbytes(t) -> int:
    if isinstance(t, (QWeight, QWeightCat, QExperts)):
        return t.nbytes()
    return t.numel() * t.element_size()


class FastModel:
    """CUDA inference model for Qwen3 / Qwen3-MoE / Qwen3-Next on one rank."""

    def __init__(self, cfg: ModelConfig, layers: list[dict[str, torch.Tensor]], embed: torch.Tensor,
                 lm_head: torch.Tensor, final_norm: torch.Tensor, dims: layout.LocalDims,
                 device: torch.device, max_slots: int = 4, max_len: int = 16384, comm=None,
                 attn_splits: int | None = None):
        if device.type != "cuda" and not _allow_cpu_prefill:
            raise ValueError("FastModel runs on CUDA only; use ReferenceModel on the CPU")
        self.cfg, self.dims, self.device = cfg, dims, device
        self.layers, self.embed_w, self.lm_head, self.final_norm = layers, embed, lm_head, final_norm
        self.max_slots, self.max_len = max_slots, max_len
        self._xscratch = None  # bf16 scratch for dequantized expert stacks (prefill)
        self.comm = comm  # parallel.TPComm or None (single rank)
        self.C = ops.C if device.type == "cuda" else None
        # vocab-parallel lm_head under the fused TP path: each rank streams V / ws rows per
        # decode step and the arg-max keys are exchanged (instead of every rank streaming
        # the whole 151936 x hidden matrix)
        V = cfg.vocab_size
        self.vocab_parallel = bool(comm is not None and dims.ws > 1 and getattr(comm, "fused", False)
                                   and V % dims.ws == 0)
        self.v_off = 0
        if self.vocab_parallel:
            vl = V // dims.ws
            self.v_off = dims.rank * vl
            self.lm_head = lm_head[self.v_off:self.v_off + vl].contiguous()
        self.v_local = self.lm_head.shape[0]
        self.inv_freq = cfg.rope_inv_freq().to(device)
        self.has_shared = cfg.shared_expert_intermediate_size > 0
        sm = torch.cuda.get_device_properties(device).multi_processor_count if device.type == "cuda" else 1
        self.sms = sm
        # split-K width of decode attention (None: per batch size, see _splits_for)
        self.attn_splits = attn_splits
        # ---- state pools -------------------------------------------------
        self.pos = torch.zeros(max_slots, dtype=torch.int32, device=device)
        self.kc: dict[int, torch.Tensor] = {}
        self.vc: dict[int, torch.Tensor] = {}
        self.conv: dict[int, torch.Tensor] = {}
        self.rec: dict[int, torch.Tensor] = {}
        for i in range(cfg.num_hidden_layers):
            if cfg.is_linear(i):
                self.conv[i] = torch.zeros(max_slots, dims.gdn_conv, cfg.linear_conv_kernel_dim,
                                           dtype=torch.bfloat16, device=device)
                self.rec[i] = torch.zeros(max_slots, dims.hv, dims.dk, dims.dv, dtype=torch.float32,
                                          device=device)
            else:
                shp = (max_slots, dims.hkv, max_len, dims.D)
                self.kc[i] = torch.zeros(shp, dtype=torch.bfloat16, device=device)
                self.vc[i] = torch.zeros(shp, dtype=torch.bfloat16, device=device)
        self._bufs: dict[int, DecodeBuffers] = {}
        # decode GEMV engine: "ld" (register-staged loads, csrc/gemv.cu; default: measured
        # 3.9-5.5 TB/s on the 80B shapes in isolation) or "tma" (bulk-copy ring,
        # csrc/gemv_tma.cu; 1.4-3.0 TB/s on the same shapes, kept as an option)
        self.gemv_engine = os.environ.get("HELEXA_GEMV", "ld")
        # attention prefill: "tc" (tcgen05/TMEM, csrc/attn_prefill_tc.cu) or "mma"
        # (mma.sync tiles, csrc/attn_prefill.cu)
        self.attn_engine = os.environ.get("HELEXA_ATTN_PREFILL", "tc")
        self.gemm_dequant = os.environ.get("HELEXA_GEMM_DEQUANT", "scratch")
        self._tma_ok_cache: dict = {}
        self.sampler = SamplerState(max_slots, device) if device.type == "cuda" else None
        # multimodal rotary (vision-language configs): per-frequency axis map, and per slot
        # the rotary position minus the cache index (negative after an image)
        self.mrope = bool(cfg.mrope_section)
        self.rope_delta = torch.zeros(max_slots, dtype=torch.int32, device=device)
        self._rope_delta_host = [0] * max_slots
        self.mrope_axes = None
        if self.mrope:
            from .mrope import mrope_axis_map
            self.mrope_axes = mrope_axis_map(cfg.rotary_dim // 2, cfg.mrope_section, cfg.mrope_interleaved).to(device)
        # decode MoE block as one persistent kernel (router, top-k, experts, down and the TP
        # exchange with grid barriers, csrc/moe_fused.cu) instead of three launches. Off by
        # default: the 80B decode step measured 4.39 ms with it vs 3.95 ms with the three
        # kernels (HELEXA_MOE_FUSED=1 turns it on)
        self.moe_fused = os.environ.get("HELEXA_MOE_FUSED", "0") == "1" and cfg.num_experts > 0
        self._moe_bar = torch.zeros(4, dtype=torch.int32, device=device) if device.type == "cuda" else None
        if self.C is not None:
            self._gemm_err()  # allocated before any graph capture
        self.prefill_timer = None  # optional PhaseTimer (CUDA events per prefill phase)

    # ------------------------------------------------------------------
    # construction
    # ------------------------------------------------------------------
    @classmethod
    def from_hf(cls, cfg: ModelConfig, get: Callable[[str], torch.Tensor] | dict, device,
                rank: int = 0, ws: int = 1, ep: bool = False, **kw) -> "FastModel":
        """Load from HF-layout tensors (a dict or a name -> tensor callable). `ep`: the
        MoE layers are expert-parallel over the ranks (whole experts per rank)."""
        if isinstance(get, dict):
            get = get.__getitem__
        device = torch.device(device)
        dims = layout.local_dims(cfg, rank, ws, ep)
        layers = []
        for i in range(cfg.num_hidden_layers):
            fl = layout.fuse_layer(cfg, dims, i, get)
            layers.append({k: v.to(device) for k, v in fl.items()})
        embed = get("model.embed_tokens.weight").to(device=device, dtype=torch.bfloat16).contiguous()
        lm = embed if cfg.tie_word_embeddings else get("lm_head.weight").to(device=device, dtype=torch.bfloat16)
        fn = layout.norm_f32(cfg, get("model.norm.weight")).to(device)
        return cls(cfg, layers, embed, lm.contiguous(), fn, dims, device, **kw)

    @classmethod
    def from_gguf(cls, cfg: ModelConfig, g, device, rank: int = 0, ws: int = 1, **kw) -> "FastModel":
        """Serve a GGUF file as GGUF: quantized projections go to the device as their
        block rows (no host dequantization, no re-quantization) and run through the
        fused-dequant GEMVs at decode and dequant-then-tcgen05-GEMM at prefill; tensor
        parallel shards are cut on block boundaries (weights/gguf.py QuantLayer)."""
        from ..weights.gguf import QuantExperts, QuantLayer, QuantRows, quant_block_of
        if cfg.family not in ("qwen3", "llama", "qwen3_moe"):
            # hybrid (GDN) GGUF files: dequantize on load
            return cls.from_hf(cfg, g.hf_get, device, rank=rank, ws=ws, **kw)
        device = torch.device(device)
        dense = [i for i in range(cfg.num_hidden_layers) if not cfg.layer_uses_moe(i)]
        blk = max([quant_block_of(g, f"blk.{i}.ffn_down.weight") for i in dense] or [1])
        dims = layout.local_dims(cfg, rank, ws, ep=kw.pop("ep", False), inter_block=blk)
        ql = QuantLayer(g)

        def dev(t):
            if isinstance(t, QuantExperts):
                return QExperts(t.raw.contiguous().to(device), t.gtype, t.G, t.R, t.K)
            if isinstance(t, QuantRows):
                return QWeight(t.raw.contiguous().to(device), t.gtype, t.K)
            if isinstance(t, list):
                return QWeightCat([dev(p) for p in t])
            return t.to(device=device, dtype=torch.float32 if t.dtype == torch.float32 and t.dim() == 1
                        else torch.bfloat16).contiguous()
        layers = [{k: dev(v) for k, v in ql.layer(cfg, dims, i).items()} for i in range(cfg.num_hidden_layers)]
        C = ops.C

        def table(name):  # embedding / lm_head: dequantized to bf16 on the device
            t = g.tensors[name]
            if t.gtype in (8, 12, 14):
                q = ql._raw2d(name)
                return QWeight(q.raw.contiguous().to(device), q.gtype, q.K).dequant(C)
            return g.tensor(name).to(device=device, dtype=torch.bfloat16).contiguous()
        embed = table("token_embd.weight")
        lm = embed if "output.weight" not in g.tensors else table("output.weight")
        fn = layout.norm_f32(cfg, g.tensor("output_norm.weight")).to(device)
        m = cls(cfg, layers, embed, lm.contiguous(), fn, dims, device, **kw)
        m.quant = "gguf"
        return m

    @classmethod
    def random(cls, cfg: ModelConfig, device, seed: int = 0, rank: int = 0, ws: int = 1, std: float = 0.02,
               ep: bool = False, **kw) -> "FastModel":
        """Random-init N(0, std) directly in the fused layout on the device (large models)."""
        device = torch.device(device)
        dims = layout.local_dims(cfg, rank, ws, ep)
        g = torch.Generator(device=device).manual_seed(seed + 7919 * rank)

        def mk(shape, dtype):
            t = torch.empty(shape, dtype=dtype, device=device)
            return t.normal_(0.0, std, generator=g)

        layers = []
        for i in range(cfg.num_hidden_layers):
            lw = {}
            for name, (shape, dtype) in layout.layer_shapes(cfg, dims, i).items():
                t = mk(shape, dtype)
                if name in ("ln1", "ln2", "q_norm", "k_norm"):
                    t += cfg.norm_offset
                lw[name] = t
            layers.append(lw)
        embed = mk((cfg.vocab_size, cfg.hidden_size), torch.bfloat16)
        lm = embed if cfg.tie_word_embeddings else mk((cfg.vocab_size, cfg.hidden_size), torch.bfloat16)
        fn = mk((cfg.hidden_size,), torch.float32) + cfg.norm_offset
        return cls(cfg, layers, embed, lm, fn, dims, device, **kw)

    def weight_bytes(self) -> int:
        n = sum(_tbytes(t) for lw in self.layers for t in lw.values())
        n += self.embed_w.numel() * 2 + (0 if self.lm_head is self.embed_w else self.lm_head.numel() * 2)
        return n

    def decode_bytes_per_token(self) -> int:
        """Weight bytes a bs=1 decode step streams (active experts only)."""
        cfg, n = self.cfg, 0
        for i, lw in enumerate(self.layers):
            for k, t in lw.items():
                if k in ("w_gu", "w_d") and cfg.layer_uses_moe(i):
                    per = t.expert_bytes() if isinstance(t, QExperts) else t[0].numel() * t.element_size()
                    n += per * (cfg.num_experts_per_tok + (1 if self.has_shared else 0))
                else:
                    n += _tbytes(t)
        return n + self.lm_head.numel() * 2 + self.cfg.hidden_size * 2

    # ------------------------------------------------------------------
    # decode
    # ------------------------------------------------------------------
    def _splits_for(self, B: int) -> int:
        """Decode-attention split count: about one 128-thread CTA per SM over all
        (sequence, kv head) pairs (measured best at 8K context: 64-104 splits per kv
        head for 2 kv heads), a multiple of 8 so the splits form 8-CTA clusters that
        merge on chip, leaving few partials for the final cross-cluster merge."""
        if self.attn_splits:
            return self.attn_splits
        want = self.sms // max(1, B * max(1, self.dims.hkv))
        return max(8, min(256, (want + 7) // 8 * 8))

    def buffers(self, B: int, out_cap: int = 4096) -> DecodeBuffers:
        if B in self._bufs:
            return self._bufs[B]
        cfg, d, dev = self.cfg, self.dims, self.device
        bf, f32, i32 = torch.bfloat16, torch.float32, torch.int32
        z = lambda *s, dt=bf: torch.zeros(*s, dtype=dt, device=dev)  # noqa: E731
        J = cfg.num_experts_per_tok + (1 if self.has_shared else 0)
        any_mlp = any(not cfg.layer_uses_moe(i) for i in range(cfg.num_hidden_layers))
        nb = DecodeBuffers(
            B=B, tok=z(B, dt=i32), slots=torch.arange(B, dtype=i32, device=dev), x=z(B, d.H),
            proj_gdn=z(B, d.gdn_in_rows) if cfg.num_linear_layers else None,
            gdn_out=z(B, d.gdn_vd) if cfg.num_linear_layers else None,
            proj_attn=z(B, d.qkv_rows) if cfg.num_full_layers else None,
            attn_out=z(B, d.hq * d.D) if cfg.num_full_layers else None,
            part_o=z(B, d.hq, self._splits_for(B), d.D, dt=f32) if cfg.num_full_layers else None,
            part_ml=z(B, d.hq, self._splits_for(B), 2, dt=f32) if cfg.num_full_layers else None,
            counters=z(B, max(1, d.hkv), dt=i32) if cfg.num_full_layers else None,
            rlogits=z(B, cfg.num_experts + (1 if self.has_shared else 0), dt=f32) if cfg.num_experts else None,
            ids=z(B, J, dt=i32) if cfg.num_experts else None,
            wts=z(B, J, dt=f32) if cfg.num_experts else None,
            act_moe=z(B * J, d.moe_inter) if cfg.num_experts else None,
            act_mlp=z(B, d.inter) if any_mlp else None,
            partial=z(B, d.H),
            logits=z(B, self.v_local, dt=f32), out_tokens=z(B, out_cap, dt=i32), step=z(B, dt=i32),
            best=z(B, dt=torch.int64), counter=z(1, dt=i32), err=z(1, dt=i32))
        self._bufs[B] = nb
        return nb

    _moe_fused_ok = False

    def _moe_fused_call(self, lw, nb: DecodeBuffers, E: int, k: int, J: int):
        d, cfg = self.dims, self.cfg
        e_base, e_count = (d.e0, lw["w_gu"].shape[0]) if d.ep else (0, 0)
        tp = {}
        err = self._gemm_err()
        if self.comm is not None and d.ws > 1:
            bases, rank, slots_, ctr, err, tmo = self.comm.fused_args()
            tp = dict(bases=bases, rank=rank, slot_elems=slots_, ctr=ctr, timeout_s=tmo)
        self.C.moe_fused(nb.x, lw["ln2"], cfg.rms_norm_eps, lw["router"], lw["w_gu"], lw["w_d"], E, k,
                         self.has_shared, cfg.norm_topk_prob, nb.rlogits, nb.act_moe, self._moe_bar, err,
                         e_base, e_count, **tp)
        self._moe_fused_ok = True

    def _tma(self, N: int, K: int, x_rows: int, groups: int = 1) -> bool:
        if self.gemv_engine != "tma" or self.C is None:
            return False
        key = (N, K, x_rows, groups)
        if key not in self._tma_ok_cache:
            self._tma_ok_cache[key] = bool(self.C.gemv_tma_ok(N, K, x_rows, groups))
        return self._tma_ok_cache[key]

    def _row_parallel(self, W, inp, nb: DecodeBuffers):
        """x += W . inp, summed across TP ranks when the layer is sharded."""
        if self.comm is None or self.dims.ws == 1:
            self._gemv(W, inp, nb.x, ops.RESID_ADD, nb.x, None, 0.0)
        elif self.comm.fused and not isinstance(W, (QWeight, QWeightCat)):
            if self._tma(W.shape[0], W.shape[1], nb.B):
                self.C.gemv_tma_ar(W, inp, nb.x, *self.comm.fused_args())
            else:
                self.C.gemv_ar(W, inp, nb.x, *self.comm.fused_args())
        else:
            self._gemv(W, inp, nb.partial, ops.STORE_BF16, None, None, 0.0)
            self.comm.reduce_residual(nb.partial, nb.x)

    def _decode_layer(self, i: int, nb: DecodeBuffers):
        C, cfg, d, lw = self.C, self.cfg, self.dims, self.layers[i]
        eps = cfg.rms_norm_eps
        if cfg.is_linear(i):
            self._gemv(lw["w_in"], nb.x, nb.proj_gdn, ops.STORE_BF16, None, lw["ln1"], eps)
            C.gdn_decode(nb.proj_gdn, lw["conv_w"], self.conv[i], self.rec[i], lw["A_log"], lw["dt_bias"],
                         lw["gnorm"], nb.slots, self.pos, nb.gdn_out, d.hk, d.hv, d.dk, d.dv, eps)
            self._row_parallel(lw["out_w"], nb.gdn_out, nb)
        else:
            self._gemv(lw["w_qkv"], nb.x, nb.proj_attn, ops.STORE_BF16, None, lw["ln1"], eps)
            C.attn_decode(nb.proj_attn, lw.get("q_norm"), lw.get("k_norm"), self.inv_freq, self.kc[i], self.vc[i],
                          nb.slots, self.pos, nb.part_o, nb.part_ml, nb.counters, nb.attn_out, d.hq, d.hkv, d.D,
                          cfg.rotary_dim, cfg.attn_output_gate, eps, self.rope_delta if self.mrope else None)
            self._row_parallel(lw["o_w"], nb.attn_out, nb)
        if cfg.layer_uses_moe(i):
            E, k = cfg.num_experts, cfg.num_experts_per_tok
            J = k + (1 if self.has_shared else 0)
            C.gemv_router(lw["router"], nb.x, nb.rlogits, lw["ln2"], eps, E, k, self.has_shared,
                          cfg.norm_topk_prob, nb.ids, nb.wts, nb.counter)
            Wgu, Wd = lw["w_gu"], lw["w_d"]
            if isinstance(Wgu, QExperts):
                C.gguf_experts(Wgu.raw, Wgu.type, Wgu.K, nb.x, nb.ids.view(-1), nb.act_moe, J, lw["ln2"], eps)
                C.gguf_moe_down(Wd.raw, Wd.type, Wd.K, nb.act_moe, nb.ids.view(-1), nb.wts.view(-1), nb.x, J)
                return
            if self.moe_fused and nb.B <= 8 and not (d.ep and not self.comm.fused):
                try:
                    self._moe_fused_call(lw, nb, E, k, J)
                    return
                except RuntimeError:
                    if self._moe_fused_ok:
                        raise
                    self.moe_fused = False  # refused on this device: three-kernel path
            tma_gu = self._tma(Wgu.shape[1], Wgu.shape[2], nb.B, nb.B * J)
            tma_d = self._tma(Wd.shape[1], Wd.shape[2], nb.B * J, nb.B)
            e_base, e_count = (d.e0, Wgu.shape[0]) if d.ep else (0, 0)
            if tma_gu:
                C.gemv_tma_experts(Wgu, nb.x, nb.ids.view(-1), nb.act_moe, ops.SILU_PAIR, J, lw["ln2"], eps, e_base,
                                   e_count, self._gemm_err())
            elif d.ep:
                C.gemv_experts_ep(Wgu, nb.x, nb.ids.view(-1), nb.act_moe, ops.SILU_PAIR, J, lw["ln2"], eps, d.e0)
            else:
                C.gemv_experts(Wgu, nb.x, nb.ids.view(-1), nb.act_moe, ops.SILU_PAIR, J, lw["ln2"], eps)
            if d.ep:
                # expert parallel: this rank runs the routes to its own experts; the fused
                # cross-rank sum in the down kernel combines every rank's experts
                if not self.comm.fused:
                    raise RuntimeError("expert parallelism needs the fused p2p reduction (HELEXA_TP_MODE=p2p)")
                if tma_d:
                    bases, rank, slots_, ctr, err, tmo = self.comm.fused_args()
                    C.moe_down_tma(Wd, nb.act_moe, nb.ids, nb.wts, nb.x, None, e_base, e_count, err, bases, rank,
                                   slots_, ctr, tmo)
                else:
                    C.moe_down_ar_ep(Wd, nb.act_moe, nb.ids, nb.wts, nb.x, *self.comm.fused_args(), d.e0)
                return
            if tma_d and (self.comm is None or d.ws == 1):
                C.moe_down_tma(Wd, nb.act_moe, nb.ids, nb.wts, nb.x, None, 0, 0, self._gemm_err())
                return
            if tma_d and self.comm.fused:
                bases, rank, slots_, ctr, err, tmo = self.comm.fused_args()
                C.moe_down_tma(Wd, nb.act_moe, nb.ids, nb.wts, nb.x, None, 0, 0, err, bases, rank, slots_, ctr, tmo)
                return
            if self.comm is None or d.ws == 1:
                C.moe_down(lw["w_d"], nb.act_moe, nb.ids, nb.wts, nb.x, None)
            elif self.comm.fused:
                C.moe_down_ar(lw["w_d"], nb.act_moe, nb.ids, nb.wts, nb.x, *self.comm.fused_args())
            else:
                C.moe_down(lw["w_d"], nb.act_moe, nb.ids, nb.wts, nb.x, nb.partial)
                self.comm.reduce_residual(nb.partial, nb.x)
        else:
            self._gemv(lw["w_gu"], nb.x, nb.act_mlp, ops.SILU_PAIR, None, lw["ln2"], eps)
            self._row_parallel(lw["w_d"], nb.act_mlp, nb)

    def decode_step_launch(self, nb: DecodeBuffers, sampled: bool = False):
        """Enqueue one decode step for the nb.B slots in nb.slots (graph-capturable).
        sampled: the lm_head writes f32 logits and the on-device sampler picks the token
        with each slot's temperature / top-k / top-p / repeat penalty."""
        self.C.embed(self.embed_w, nb.tok, nb.x)
        for i in range(self.cfg.num_hidden_layers):
            self._decode_layer(i, nb)
        if sampled:
            self.C.gemv(self.lm_head, nb.x, nb.logits, ops.STORE_F32, None, self.final_norm, self.cfg.rms_norm_eps)
            full = nb.logits
            if self.vocab_parallel:
                if nb.logits_full is None:
                    nb.logits_full = torch.zeros(nb.B, self.cfg.vocab_size, dtype=torch.float32, device=self.device)
                self._gather_logits(nb)
                full = nb.logits_full
            st = self.sampler
            self.C.sample_step(full, self.cfg.vocab_size, nb.slots, *st.tensors(), nb.tok, self.pos, nb.out_tokens,
                               nb.step)
            return
        if self._tma(self.lm_head.shape[0], self.lm_head.shape[1], nb.B):
            tp = {}
            if self.vocab_parallel:
                bases, rank, slots_, ctr, _, tmo = self.comm.fused_args()
                tp = dict(bases=bases, rank=rank, slot_elems=slots_, ctr=ctr, timeout_s=tmo)
            self.C.gemv_tma_argmax(self.lm_head, nb.x, nb.logits, self.final_norm, self.cfg.rms_norm_eps, nb.best,
                                   nb.counter, nb.tok, nb.slots, self.pos, nb.out_tokens, nb.step, self.v_off,
                                   self.comm.err if self.vocab_parallel else self._gemm_err(), **tp)
        elif self.vocab_parallel:
            self.C.gemv_argmax_tp(self.lm_head, nb.x, nb.logits, self.final_norm, self.cfg.rms_norm_eps, nb.best,
                                  nb.counter, nb.tok, nb.slots, self.pos, nb.out_tokens, nb.step, self.v_off,
                                  *self.comm.fused_args())
        else:
            self.C.gemv_argmax(self.lm_head, nb.x, nb.logits, self.final_norm, self.cfg.rms_norm_eps, nb.best,
                               nb.counter, nb.tok, nb.slots, self.pos, nb.out_tokens, nb.step)

    def _gather_logits(self, nb: DecodeBuffers):
        """logits_full[b] = the concatenation over ranks of each rank's vocabulary slice
        (NCCL all-gather; capturable in the decode graph)."""
        import torch.distributed as dist
        ws = self.dims.ws
        if nb._gather_buf is None:
            nb._gather_buf = torch.empty(ws, nb.B, self.v_local, dtype=torch.float32, device=self.device)
        dist.all_gather_into_tensor(nb._gather_buf, nb.logits, group=self.comm.group)
        nb.logits_full.view(nb.B, ws, self.v_local).copy_(nb._gather_buf.transpose(0, 1))

    def launches_per_step(self) -> int:
        cfg = self.cfg
        n = 2  # embed, lm_head(+arg-max)
        for i in range(cfg.num_hidden_layers):
            n += 3 + ((1 if self.moe_fused else 3) if cfg.layer_uses_moe(i) else 2)
            if self.comm is not None and self.dims.ws > 1:
                n += self.comm.launches_per_reduce * 2
            n += sum(_extra_launches(w) for w in self.layers[i].values())
        return n

    def quantize_(self, scheme: str, experts: bool = True) -> None:
        """In-situ quantization (the reference's ISQ, tp/isq.rs:252-326) of the linear
        projections into GGUF k-quant blocks on the device: GDN in/out, attention
        qkv/o, dense-MLP gate-up/down and (`experts`, single rank, k-quant schemes) the
        stacked MoE experts. Router, embedding and lm_head stay bf16. Weights whose
        input width is not a multiple of the block size stay bf16 too (a
        tensor-parallel shard must hold whole superblocks)."""
        if scheme not in QUANT_SCHEMES:
            raise ValueError(f"unknown quantization {scheme!r}; one of {sorted(QUANT_SCHEMES)}")
        if self.C is None:
            raise RuntimeError("quantized serving needs the CUDA extension")
        rule = QUANT_SCHEMES[scheme]
        for i, lw in enumerate(self.layers):
            keys = ["w_in", "out_w", "w_qkv", "o_w"]
            if not self.cfg.layer_uses_moe(i):
                keys += ["w_gu", "w_d"]
            elif experts and self.dims.ws == 1:
                # stacked experts: every expert's rows quantized in one pass (whole rows on
                # one rank; sharded-intermediate experts would split down_proj superblocks)
                gts = {k: rule.get(k, rule["*"]) for k in ("w_gu", "w_d")}
                ok = not any(isinstance(lw[k], QExperts) or lw[k].shape[2] % 256 or
                             gts[k] not in (GGUF_Q4_K, GGUF_Q6_K) for k in gts)
                for k, gt in (gts.items() if ok else ()):  # both stacks quantized or neither
                    w = lw[k]
                    G, R, K = w.shape
                    lw[k] = QExperts(self.C.gguf_quant(w.reshape(G * R, K).contiguous(), gt), gt, G, R, K)
                    del w
                if ok:
                    self.moe_fused = False
            for k in keys:
                w = lw.get(k)
                if w is None or isinstance(w, (QWeight, QWeightCat)) or w.dim() != 2:
                    continue
                gt = rule.get(k, rule["*"])
                if w.shape[1] % _GGUF_BLOCK[gt][1]:
                    continue
                lw[k] = QWeight(self.C.gguf_quant(w.contiguous(), gt), gt, w.shape[1])
                del w
        self.quant = scheme
        for nb in self._bufs.values():  # captured graphs refer to the old weights
            nb.graph = nb.sgraph = None
        torch.cuda.empty_cache()

    def _gemv(self, W, x, y, mode: int, resid=None, norm=None, eps: float = 0.0):
        if isinstance(W, QWeightCat):
            if mode != ops.STORE_BF16:
                raise ValueError("segmented quantized weights support the plain store epilogue only")
            off = 0
            for p in W.parts:
                n = p.shape[0]
                self._gemv(p, x, y[:, off:off + n], mode, None, norm, eps)
                off += n
            return
        if isinstance(W, QWeight):
            self.C.gguf_gemv(W.raw, W.type, W.K, x, y, mode, resid, norm, eps)
        elif x.shape[0] <= 8 and self._tma(W.shape[0], W.shape[1], x.shape[0]):
            self.C.gemv_tma(W, x, y, mode, resid, norm, eps, self._gemm_err())
        else:
            self.C.gemv(W, x, y, mode, resid, norm, eps)

    def prefill_launches(self) -> int:
        """Kernels of this package one prefill chunk launches (the MoE combine's output
        memset and the vocab-parallel logits gather are library calls, not counted)."""
        cfg = self.cfg
        n = 3  # embedding, first norm, lm_head GEMM of the last token
        for i in range(cfg.num_hidden_layers):
            # in_proj, prep, chunk, scan, onorm, out, conv ring | qkv, q/k-norm+rope+KV, attn, o
            n += 5 + 3 if cfg.is_linear(i) else 4
            n += 7 if cfg.layer_uses_moe(i) else 2          # router, topk, plan, place, 2 grouped, combine | 2 GEMMs
            n += 2                                          # two fused (reduce +) residual + norm kernels
        return n

    def capture(self, B: int, steps: int = 1, sampled: bool = False) -> DecodeBuffers:
        """Capture `steps` consecutive decode steps for batch B into one CUDA graph
        (`sampled`: the on-device sampler instead of the fused arg-max).

        Capture runs one eager warm-up step first; pool state it touches (positions,
        KV at the current position, GDN state, sampler counters and history) is saved
        and restored around it.
        """
        nb = self.buffers(B)
        if sampled and nb.sgraph is not None and nb.sgraph_steps == steps:
            return nb
        if not sampled and nb.graph is not None and nb.graph_steps == steps:
            return nb
        if sampled and self.vocab_parallel and nb.logits_full is None:
            nb.logits_full = torch.zeros(B, self.cfg.vocab_size, dtype=torch.float32, device=self.device)
        saved = self._save_slots(nb.slots.tolist())
        samp = self.sampler.snapshot() if sampled else None
        step_saved, tok_saved = nb.step.clone(), nb.tok.clone()
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.decode_step_launch(nb, sampled)
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self._restore_slots(saved)
        if samp is not None:
            self.sampler.restore(samp)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            for _ in range(steps):
                self.decode_step_launch(nb, sampled)
        torch.cuda.synchronize(self.device)
        nb.step.copy_(step_saved)
        nb.tok.copy_(tok_saved)
        if sampled:
            nb.sgraph, nb.sgraph_steps = g, steps
        else:
            nb.graph, nb.graph_steps = g, steps
        return nb

    def _save_slots(self, slots: list[int]):
        return {"pos": self.pos.clone(),
                "conv": {i: t[slots].clone() for i, t in self.conv.items()},
                "rec": {i: t[slots].clone() for i, t in self.rec.items()}, "slots": slots}

    def _restore_slots(self, saved):
        sl = saved["slots"]
        self.pos.copy_(saved["pos"])
        for i, t in saved["conv"].items():
            self.conv[i][sl] = t
        for i, t in saved["rec"].items():
            self.rec[i][sl] = t

    def replay(self, nb: DecodeBuffers, sampled: bool = False):
        (nb.sgraph if sampled else nb.graph).replay()

    # ------------------------------------------------------------------
    # prefill
    # ------------------------------------------------------------------
    def _rms(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.cfg.rms_norm_eps) * w).to(torch.bfloat16)

    def _linear(self, x: torch.Tensor, W: torch.Tensor, epi: int = 0, out: torch.Tensor | None = None) -> torch.Tensor:
        """x [T, K] @ W[N, K]^T on the tcgen05 GEMM (epi 1: SwiGLU on interleaved rows;
        epi 2: f32 output). `out`: a caller-provided contiguous [T, N] destination."""
        x = x.contiguous()
        if self.C is None:  # CPU layout tests only
            y = x @ W.t()
            if epi == 1:
                y = (torch.nn.functional.silu(y[:, 0::2].float()).to(torch.bfloat16).float()
                     * y[:, 1::2].float()).to(torch.bfloat16)
            if out is not None:
                out.copy_(y)
                return out
            return y
        if isinstance(W, QWeight) and self._fused_dequant(W):
            # dequantization inside the GEMM's producer: no bf16 copy of the weight
            N = W.shape[0] // 2 if epi == 1 else W.shape[0]
            dst = out if (out is not None and N % 8 == 0) else \
                torch.empty(x.shape[0], (N + 7) // 8 * 8, dtype=torch.float32 if epi == 2 else torch.bfloat16,
                            device=x.device)
            self.C.gemm_q(x, W.raw, W.type, W.K, dst, epi, self._gemm_err())
            y = dst if dst.shape[1] == N else dst[:, :N]
            if out is not None and y is not out:
                out.copy_(y)
                return out
            return y
        if isinstance(W, (QWeight, QWeightCat)):
            W = W.dequant(self.C)
        N = W.shape[0] // 2 if epi == 1 else W.shape[0]
        if out is not None and N % 8 == 0:
            self.C.gemm(x, W, out, epi, self._gemm_err())
            return out
        Np = (N + 7) // 8 * 8  # keep output rows 16-byte aligned for the vector epilogue
        y = torch.empty(x.shape[0], Np, dtype=torch.float32 if epi == 2 else torch.bfloat16, device=x.device)
        self.C.gemm(x, W, y, epi, self._gemm_err())
        y = y if Np == N else y[:, :N]
        if out is not None:
            out.copy_(y)
            return out
        return y

    def _fused_dequant(self, W: "QWeight") -> bool:
        """HELEXA_GEMM_DEQUANT=fused: quantized prefill GEMMs dequantize in the GEMM's
        producer warps (Q8_0, Q4_K, padded Q6_K; K a multiple of 256). The default
        dequantizes the whole weight to bf16 scratch first: measured faster at every M
        (`gemm_bench.quant_main`: 10240 x 5120 Q4_K at M = 16, 0.41 ms fused vs 0.087 ms
        for dequantize + GEMM; the fused producer runs on N / 256 CTAs only and
        re-decodes each weight tile once per 128-row block).""" 
        return (self.gemm_dequant == "fused" and W.raw.is_cuda and W.K % 256 == 0
                and W.type in (GGUF_Q8_0, GGUF_Q4_K, GGUF_Q6_K_PADDED))

    def _gemm_err(self) -> torch.Tensor:
        if not hasattr(self, "_gerr"):
            self._gerr = torch.zeros(1, dtype=torch.int32, device=self.device)
        return self._gerr

    def device_error(self) -> int:
        """First nonzero device error word (GEMM bounded waits, TP exchange), else 0.
        Reading it synchronizes the device."""
        words = [self._gemm_err()]
        if self.comm is not None and getattr(self.comm, "err", None) is not None:
            words.append(self.comm.err)
        for v in torch.cat([w.view(-1)[:1] for w in words]).tolist():
            if v:
                return int(v)
        return 0

    def check_errors(self):
        """Raise DeviceError if a device-side bounded wait gave up since the model was
        built: the kernels return instead of hanging, so their outputs after that point
        are not valid and must not be served."""
        code = self.device_error()
        if code:
            raise DeviceError(code)

    # ------------------------------------------------------------------
    # prefill plumbing: residual + norm, reductions, buffers
    # ------------------------------------------------------------------
    def _tp(self) -> bool:
        return self.comm is not None and self.dims.ws > 1

    def _fused_prefill_tp(self) -> bool:
        return self._tp() and self.C is not None and getattr(self.comm, "fused", False)

    def _add_norm(self, x: torch.Tensor, o: torch.Tensor | None, w: torch.Tensor, h: torch.Tensor):
        """x += o (o already summed over ranks, or None), h = RMSNorm(x) * w."""
        if self.C is None:
            if o is not None:
                x.copy_(x + o)
            h.copy_(self._rms(x, w))
            return
        self.C.add_rmsnorm(x, o, w, h, self.cfg.rms_norm_eps)

    def _reduce_add_norm(self, x: torch.Tensor, o: torch.Tensor, w: torch.Tensor, h: torch.Tensor):
        """x += sum over ranks of the row-parallel partial o; h = RMSNorm(x) * w.

        Fused TP (p2p): o lives in this rank's exported staging buffer and one kernel
        reduce-scatters it, adds the residual, normalises and all-gathers h over peer
        memory. Other modes: all-reduce (NCCL or the one-shot kernel), then the fused
        add + norm kernel."""
        if self._fused_prefill_tp():
            self.comm.rs_norm_ag(x, w, self.cfg.rms_norm_eps)
            return
        if self._tp():
            self.comm.all_reduce_(o)
        self._add_norm(x, o, w, h)

    def _prefill_bufs(self, T: int):
        """(row-parallel output destination or None, h) for a chunk of T tokens."""
        H = self.cfg.hidden_size
        if self._fused_prefill_tp():
            stage, h = self.comm.prefill_region(self.prefill_cap, H)
            return stage[:T * H].view(T, H), h[:T * H].view(T, H)
        return None, torch.empty(T, H, dtype=torch.bfloat16, device=self.device)

    @property
    def prefill_cap(self) -> int:
        """Largest prefill chunk (tokens) one pass handles; longer prompts are chunked."""
        return min(8192, self.max_len)

    def _gdn_prefill(self, i: int, h: torch.Tensor, slot: int, p0: int, out=None) -> torch.Tensor:
        from .reference import causal_conv1d, delta_rule_chunked, delta_rule_recurrent, gdn_gating, l2norm
        d, lw, cfg = self.dims, self.layers[i], self.cfg
        T = h.shape[0]
        kd, vd, K = d.gdn_kd, d.gdn_vd, cfg.linear_conv_kernel_dim
        self._mark("gdn.in_proj")
        proj = self._linear(h, lw["w_in"])
        if self.C is not None:
            ring = self.conv[i][slot]
            o = torch.empty(T, vd, dtype=torch.bfloat16, device=h.device)
            self._mark("gdn.core")
            self.C.gdn_prefill(proj, lw["conv_w"], ring, lw["A_log"], lw["dt_bias"], lw["gnorm"], self.rec[i][slot],
                               o, d.hk, d.hv, d.dk, p0, cfg.rms_norm_eps)
            # the ring keeps the last K conv inputs (slot = position % K) for decode
            self.C.conv_ring_update(proj, ring, p0)
            self._mark("gdn.out_proj")
            return self._linear(o, lw["out_w"], out=out)
        mixed = proj[:, :2 * kd + vd]
        z = proj[:, 2 * kd + vd:2 * kd + 2 * vd]
        bb = proj[:, 2 * kd + 2 * vd:2 * kd + 2 * vd + d.hv]
        aa = proj[:, 2 * kd + 2 * vd + d.hv:]
        ring = self.conv[i][slot]                                   # [C, K]
        prev = [p0 - (K - 1) + j for j in range(K - 1)]
        state = torch.stack([ring[:, p % K] if p >= 0 else torch.zeros_like(ring[:, 0]) for p in prev], 1)
        y, _ = causal_conv1d(mixed, lw["conv_w"], state)
        y = y.to(torch.bfloat16)
        for p in range(max(p0, p0 + T - K), p0 + T):
            ring[:, p % K] = mixed[p - p0]
        r = d.hv // d.hk
        q = y[:, :kd].float().view(T, d.hk, d.dk).repeat_interleave(r, 1)
        k = y[:, kd:2 * kd].float().view(T, d.hk, d.dk).repeat_interleave(r, 1)
        v = y[:, 2 * kd:].float().view(T, d.hv, d.dv)
        g, beta = gdn_gating(aa, bb, lw["A_log"], lw["dt_bias"])
        q = l2norm(q) * (d.dk ** -0.5)
        k = l2norm(k)
        fn = delta_rule_chunked if T >= 64 else delta_rule_recurrent
        o, S = fn(q, k, v, g, beta, self.rec[i][slot])
        self.rec[i][slot] = S
        o = o.to(torch.bfloat16).float()
        o = o * torch.rsqrt(o.pow(2).mean(-1, keepdim=True) + cfg.rms_norm_eps)
        o = o.to(torch.bfloat16).float() * lw["gnorm"]
        o = (o * torch.nn.functional.silu(z.float().view(T, d.hv, d.dv))).to(torch.bfloat16)
        return self._linear(o.reshape(T, vd), lw["out_w"], out=out)

    def _attn_prefill(self, i: int, h: torch.Tensor, slot: int, p0: int, out=None) -> torch.Tensor:
        d, lw, cfg = self.dims, self.layers[i], self.cfg
        T, D = h.shape[0], d.D
        self._mark("attn.qkv")
        qkv = self._linear(h, lw["w_qkv"])
        if self.C is not None:
            self._mark("attn.rope_kv")
            # q/k-norm + partial RoPE + KV-cache append in one kernel; the sigmoid output
            # gate is applied in the attention kernel's epilogue
            q = torch.empty(T, d.hq * D, dtype=torch.bfloat16, device=h.device)
            pos3 = self._pos3
            self.C.qk_rope_kv(qkv, d.hq, d.hkv, D, d.qw, lw.get("q_norm"), lw.get("k_norm"), self.inv_freq,
                              cfg.rotary_dim, self.kc[i][slot], self.vc[i][slot], p0, q, cfg.rms_norm_eps,
                              pos3, self.mrope_axes if pos3 is not None else None, self._rope_delta_host[slot])
            o = torch.empty(T, d.hq * D, dtype=torch.bfloat16, device=h.device)
            gate = qkv[:, D:] if cfg.attn_output_gate else None
            self._mark("attn.core")
            if self.attn_engine == "tc":
                self.C.attn_prefill_tc(q, self.kc[i][slot], self.vc[i][slot], o, d.hq, p0, D ** -0.5, gate, d.qw,
                                       self._gemm_err())
            else:
                self.C.attn_prefill(q, self.kc[i][slot], self.vc[i][slot], o, d.hq, p0, D ** -0.5, gate, d.qw)
            self._mark("attn.o_proj")
            return self._linear(o, lw["o_w"], out=out)
        from .reference import apply_rope, rope_cos_sin
        qp = qkv[:, :d.hq * d.qw].view(T, d.hq, d.qw)
        q, gate = qp[..., :D], (qp[..., D:] if cfg.attn_output_gate else None)
        k = qkv[:, d.hq * d.qw:d.hq * d.qw + d.hkv * D].view(T, d.hkv, D)
        v = qkv[:, d.hq * d.qw + d.hkv * D:].view(T, d.hkv, D)
        if "q_norm" in lw:
            q, k = self._rms(q, lw["q_norm"]), self._rms(k, lw["k_norm"])
        cos, sin = rope_cos_sin(torch.arange(p0, p0 + T, device=h.device), cfg.rotary_dim, cfg.rope_theta,
                                self.inv_freq)
        q = apply_rope(q.float(), cos, sin).to(torch.bfloat16)
        k = apply_rope(k.float(), cos, sin).to(torch.bfloat16)
        self.kc[i][slot, :, p0:p0 + T] = k.transpose(0, 1)
        self.vc[i][slot, :, p0:p0 + T] = v.transpose(0, 1)
        L = p0 + T
        Kc, Vc = self.kc[i][slot, :, :L], self.vc[i][slot, :, :L]
        if p0 == 0:
            o = torch.nn.functional.scaled_dot_product_attention(
                q.transpose(0, 1)[None], Kc[None], Vc[None], is_causal=True, enable_gqa=True)[0]
        else:
            mask = torch.arange(L, device=h.device)[None, :] <= torch.arange(p0, L, device=h.device)[:, None]
            o = torch.nn.functional.scaled_dot_product_attention(
                q.transpose(0, 1)[None], Kc[None], Vc[None], attn_mask=mask, enable_gqa=True)[0]
        o = o.transpose(0, 1).reshape(T, d.hq * D)
        if gate is not None:
            o = (o.float() * torch.sigmoid(gate.reshape(T, d.hq * D).float())).to(torch.bfloat16)
        return self._linear(o, lw["o_w"], out=out)

    def _ffn_prefill(self, i: int, hn: torch.Tensor, out=None) -> torch.Tensor:
        cfg, lw = self.cfg, self.layers[i]
        if not cfg.layer_uses_moe(i):
            return self._linear(self._linear(hn, lw["w_gu"], 1), lw["w_d"], out=out)
        E, k = cfg.num_experts, cfg.num_experts_per_tok
        T = hn.shape[0]
        self._mark("moe.router")
        logits = self._linear(hn, lw["router"], 2)
        if self.C is not None:
            return self._moe_prefill_device(lw, hn, logits, E, k, out)
        # CPU path (tests without the extension): per-expert loops over sorted routes
        probs = torch.softmax(logits[:, :E].float(), -1)
        topv, topi = torch.topk(probs, k, -1)
        if cfg.norm_topk_prob:
            topv = topv / topv.sum(-1, keepdim=True)
        acc = torch.zeros(T, cfg.hidden_size, dtype=torch.float32, device=hn.device)
        flat = topi.view(-1)
        order = torch.argsort(flat, stable=True)
        tok_of, w_of = order // k, topv.view(-1)[order]
        counts = torch.bincount(flat, minlength=E).tolist()
        d = self.dims
        start = 0
        for e, c in enumerate(counts):
            le = e - d.e0 if d.ep else e  # expert parallel: only this rank's experts
            if c and 0 <= le < lw["w_gu"].shape[0]:
                t = tok_of[start:start + c]
                y = self._linear(self._linear(hn[t], lw["w_gu"][le], 1), lw["w_d"][le])
                acc.index_add_(0, t, y.float() * w_of[start:start + c, None])
            start += c
        if self.has_shared:
            y = self._linear(self._linear(hn, lw["w_gu"][E], 1), lw["w_d"][E])
            acc += y.float() * torch.sigmoid(logits[:, E:E + 1].float())
        if out is not None:
            out.copy_(acc)
            return out
        return acc.to(torch.bfloat16)

    def _moe_prefill_device(self, lw, hn, logits, E: int, k: int, out=None) -> torch.Tensor:
        """Routing, grouped expert GEMMs and combine with no host synchronisation."""
        cfg, dev = self.cfg, hn.device
        T, H = hn.shape
        shared = self.has_shared
        d = self.dims
        J, G = k + int(shared), (d.e_local if d.ep else E + int(shared))
        i32 = torch.int32
        ids = torch.empty(T, J, dtype=i32, device=dev)
        wts = torch.empty(T, J, dtype=torch.float32, device=dev)
        rows = torch.empty(T, J, dtype=i32, device=dev)
        counts = torch.zeros(G, dtype=i32, device=dev)
        offsets = torch.empty(G, dtype=i32, device=dev)
        cursor = torch.empty(G, dtype=i32, device=dev)
        tiles = torch.empty((T * J + 127) // 128 + G, 4, dtype=i32, device=dev)
        ntiles = torch.empty(1, dtype=i32, device=dev)
        A = torch.empty(T * J, H, dtype=torch.bfloat16, device=dev)
        self._mark("moe.route")
        self.C.moe_route_prefill(logits, E, k, shared, cfg.norm_topk_prob, hn.contiguous(), ids, wts, rows, counts,
                                 offsets, cursor, tiles, ntiles, A, d.e0 if d.ep else 0, d.e_local if d.ep else 0)
        Wgu, Wd = lw["w_gu"], lw["w_d"]
        if isinstance(Wgu, QExperts):
            # quantized experts: dequantize the stacks into the shared bf16 scratch
            need = max(Wgu.G * Wgu.R * Wgu.K, Wd.G * Wd.R * Wd.K)
            if self._xscratch is None or self._xscratch[0].numel() < need:
                self._xscratch = [torch.empty(need, dtype=torch.bfloat16, device=dev) for _ in range(2)]
            Wgu, Wd = Wgu.dequant(self.C, self._xscratch[0]), Wd.dequant(self.C, self._xscratch[1])
        I2 = Wgu.shape[1]
        act = torch.empty(T * J, I2 // 2, dtype=torch.bfloat16, device=dev)
        self._mark("moe.gemm_gate_up")
        self.C.gemm_grouped_dev(A, Wgu.reshape(-1, H), act, tiles, ntiles, I2, 1, self._gemm_err())
        y = torch.empty(T * J, H, dtype=torch.bfloat16, device=dev)
        self._mark("moe.gemm_down")
        self.C.gemm_grouped_dev(act, Wd.reshape(-1, Wd.shape[-1]), y, tiles, ntiles, H, 0,
                                self._gemm_err())
        if out is None:
            out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        self._mark("moe.combine")
        self.C.moe_combine(y, rows, wts, out, accumulate=False)  # writes every row of out
        return out

    _pos3 = None

    @torch.no_grad()
    def prefill(self, slot: int, tokens: torch.Tensor | None, p0: int, embeds: torch.Tensor | None = None,
                pos3: torch.Tensor | None = None, next_pos: int | None = None) -> torch.Tensor:
        """Run `tokens` (device int tensor [T]) for `slot` starting at position p0.

        Updates the slot's KV / GDN state and position; returns the last token's
        f32 logits [V]. Prompts longer than `prefill_cap` run as consecutive chunks.
        Vision-language prompts pass `embeds` [T, H] (image tokens spliced in) instead of
        token ids, their M-RoPE positions `pos3` [3, T] and `next_pos`, the rotary
        position of the token after the prompt (models/mrope.py).
        """
        T = tokens.shape[0] if tokens is not None else embeds.shape[0]
        if p0 + T > self.max_len:
            raise ValueError(f"sequence of {p0 + T} tokens exceeds max_len {self.max_len}")
        if pos3 is not None and not self.mrope:
            raise ValueError("multimodal positions need a config with mrope_section")
        cap = self.prefill_cap
        logits = None
        for s in range(0, T, cap):
            self._pos3 = pos3[:, s:s + cap].to(self.device, torch.int32).contiguous() if pos3 is not None else None
            logits = self._prefill_chunk(slot, tokens[s:s + cap] if tokens is not None else None, p0 + s,
                                         embeds[s:s + cap] if embeds is not None else None)
        self._pos3 = None
        if next_pos is not None:
            self.set_rope_delta(slot, next_pos - (p0 + T))
        return logits

    def set_rope_delta(self, slot: int, delta: int):
        self._rope_delta_host[slot] = int(delta)
        self.rope_delta[slot] = int(delta)

    def _prefill_chunk(self, slot: int, tokens: torch.Tensor | None, p0: int,
                       embeds: torch.Tensor | None = None) -> torch.Tensor:
        cfg = self.cfg
        T = tokens.shape[0] if tokens is not None else embeds.shape[0]
        H = cfg.hidden_size
        L = cfg.num_hidden_layers
        if embeds is not None:
            x = embeds.to(device=self.device, dtype=torch.bfloat16).contiguous().clone()
        elif self.C is not None:
            x = torch.empty(T, H, dtype=torch.bfloat16, device=self.device)
            self.C.embed(self.embed_w, tokens.to(torch.int32).contiguous(), x)
        else:
            x = self.embed_w[tokens.long()].clone()
        out, h = self._prefill_bufs(T)
        # every rank computes all rows of the first norm itself (the embedding is replicated)
        self._add_norm(x, None, self.layers[0]["ln1"], h)
        tm = self.prefill_timer
        for i in range(L):
            lw = self.layers[i]
            if tm is not None:
                tm.mark("gdn" if cfg.is_linear(i) else "attn")
            o = self._gdn_prefill(i, h, slot, p0, out) if cfg.is_linear(i) else \
                self._attn_prefill(i, h, slot, p0, out)
            self._mark("norm")
            self._reduce_add_norm(x, o, lw["ln2"], h)
            if tm is not None:
                tm.mark("moe" if cfg.layer_uses_moe(i) else "mlp")
            o = self._ffn_prefill(i, h, out)
            nxt = self.layers[i + 1]["ln1"] if i + 1 < L else self.final_norm
            self._mark("norm")
            self._reduce_add_norm(x, o, nxt, h)
        if tm is not None:
            tm.mark("head")
        self.pos[slot] = p0 + T
        # h holds the final-normed rows (all-gathered under TP): the lm_head reads the last
        return self.full_logits(self._linear(h[-1:], self.lm_head, 2))[0]

    def _mark(self, name: str):
        """Start a named prefill sub-phase on the optional PhaseTimer (profiling)."""
        if self.prefill_timer is not None:
            self.prefill_timer.mark(name)

    def full_logits(self, local: torch.Tensor) -> torch.Tensor:
        """[n, V_local] logits of this rank's vocabulary slice -> [n, V] on every rank."""
        if not self.vocab_parallel:
            return local
        return self.comm.all_gather_rows(local)
