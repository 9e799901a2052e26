"""Plain-PyTorch reference implementation of the served architectures.

This module is the numerical oracle for every CUDA kernel in the package and the
model the runtime uses when it runs on the CPU (tests, plumbing). It restates the
math of the reference's model files in torch, with every reduction in fp32:

  * `(1+w)` RMSNorm, gated RMSNorm and L2-norm:      arch/qwen3_5/rmsnorm.rs:31-137
  * gated full attention with partial RoPE:          arch/qwen3_5/full_attn.rs:112-260, rope.rs:29-263
  * Gated DeltaNet (conv1d+SiLU, gating, delta rule): arch/qwen3_5/linear_attn.rs:260-646
  * MoE block (softmax over all experts -> top-k -> optional renorm, shared expert
    scaled by sigmoid(shared_expert_gate(x))):       arch/qwen3_5/moe.rs:39-199

Unlike the reference's CUDA path (linear_attn.rs:815-823), a multi-token conv1d
forward here always prepends the carried conv state, so chunked prefill keeps its
left context.

Weights are taken from an HF-layout state dict (`model.layers.{i}....`), so the
same tensors drive this module, the fast CUDA model and HF transformers.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

from ..config import ModelConfig

# --------------------------------------------------------------------------
# elementary ops (fp32)
# --------------------------------------------------------------------------


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float, offset: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return y * (offset + w.float())


def gated_rms_norm(x: torch.Tensor, z: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    y = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return (w.float() * y) * F.silu(z.float())


def l2norm(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    return x * torch.rsqrt((x * x).sum(-1, keepdim=True) + eps)


def rope_cos_sin(positions: torch.Tensor, rotary_dim: int, theta: float, inv: torch.Tensor | None = None):
    if inv is None:
        inv = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.int64).float() / rotary_dim))
    freqs = positions.float()[:, None] * inv[None, :].to(positions.device)
    emb = torch.cat([freqs, freqs], -1)
    return emb.cos(), emb.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x: [T, H, D]; cos/sin: [T, rotary_dim]. Rotate-half on the first rotary_dim dims."""
    rd = cos.shape[-1]
    xr, xp = x[..., :rd], x[..., rd:]
    x1, x2 = xr[..., : rd // 2], xr[..., rd // 2:]
    rot = torch.cat([-x2, x1], -1)
    out = xr * cos[:, None, :] + rot * sin[:, None, :]
    return torch.cat([out, xp], -1)


def causal_conv1d(x: torch.Tensor, w: torch.Tensor, state: torch.Tensor):
    """Depthwise causal conv + SiLU over a token block with carried state.

    x: [T, C]; w: [C, K]; state: [C, K-1] (the previous K-1 inputs, oldest first).
    Returns (y [T, C], new_state [C, K-1]).
    """
    K = w.shape[1]
    full = torch.cat([state.to(x.dtype), x.t()], dim=1)         # [C, K-1+T]
    y = F.conv1d(full[None].float(), w.float()[:, None, :], groups=w.shape[0])[0]  # [C, T]
    new_state = full[:, -(K - 1):].clone()
    return F.silu(y).t(), new_state


def gdn_gating(a: torch.Tensor, b: torch.Tensor, A_log: torch.Tensor, dt_bias: torch.Tensor):
    beta = torch.sigmoid(b.float())
    g = -torch.exp(A_log.float()) * F.softplus(a.float() + dt_bias.float())
    return g, beta


def delta_rule_recurrent(q, k, v, g, beta, state):
    """Token-by-token gated delta rule. q,k: [T,H,Dk] (already l2-normed and scaled);
    v: [T,H,Dv]; g,beta: [T,H]; state: [H,Dk,Dv] f32. Returns (o [T,H,Dv], state)."""
    S = state.clone().float()
    outs = []
    for t in range(q.shape[0]):
        S = S * torch.exp(g[t])[:, None, None]
        kv = torch.einsum("hk,hkv->hv", k[t], S)
        delta = (v[t] - kv) * beta[t][:, None]
        S = S + k[t][:, :, None] * delta[:, None, :]
        outs.append(torch.einsum("hk,hkv->hv", q[t], S))
    return torch.stack(outs, 0), S


def delta_rule_chunked(q, k, v, g, beta, state, chunk: int = 64):
    """Chunk-parallel gated delta rule (WY/UT form). Same contract as the recurrent form.

    Within a chunk the unit-lower-triangular system (I + A) is solved by row-wise
    forward substitution (arch/qwen3_5/linear_attn.rs:566-596); the state is carried
    across chunks in fp32.
    """
    T, H, Dk = k.shape
    Dv = v.shape[-1]
    pad = (-T) % chunk
    q, k, v = (F.pad(x.float(), (0, 0, 0, 0, 0, pad)) for x in (q, k, v))
    g = F.pad(g.float(), (0, 0, 0, pad))
    beta = F.pad(beta.float(), (0, 0, 0, pad))
    n = (T + pad) // chunk
    # -> [H, n, C, *]
    q, k, v = (x.view(n, chunk, H, -1).permute(2, 0, 1, 3) for x in (q, k, v))
    g = g.view(n, chunk, H).permute(2, 0, 1)
    beta = beta.view(n, chunk, H).permute(2, 0, 1)
    gc = g.cumsum(-1)                                             # [H, n, C]
    kb = k * beta[..., None]
    vb = v * beta[..., None]
    dev = q.device
    lower = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool, device=dev), -1)
    causal = torch.tril(torch.ones(chunk, chunk, dtype=torch.bool, device=dev))
    decay = torch.exp((gc[..., :, None] - gc[..., None, :]).masked_fill(~causal, float("-inf")))
    A = -(kb @ k.transpose(-1, -2)) * decay
    A = A.masked_fill(~lower, 0.0)
    # forward substitution: T = (I - A)^-1 applied row by row
    Tm = A.clone()
    for i in range(1, chunk):
        row = Tm[..., i, :i].clone()
        Tm[..., i, :i] = row + (row[..., :, None] * Tm[..., :i, :i]).sum(-2)
    Tm = Tm + torch.eye(chunk, device=dev)
    u = Tm @ vb                                                   # [H, n, C, Dv]
    w = Tm @ (kb * torch.exp(gc)[..., None])                      # [H, n, C, Dk]
    S = state.clone().float()
    out = torch.empty(H, n, chunk, Dv, device=dev)
    for c in range(n):
        qi, ki = q[:, c], k[:, c]
        attn = (qi @ ki.transpose(-1, -2)) * decay[:, c]
        attn = attn.masked_fill(~causal, 0.0)
        vnew = u[:, c] - w[:, c] @ S
        out[:, c] = (qi * torch.exp(gc[:, c])[..., None]) @ S + attn @ vnew
        glast = gc[:, c, -1]
        S = S * torch.exp(glast)[:, None, None] + \
            (ki * torch.exp(glast[:, None] - gc[:, c])[..., None]).transpose(-1, -2) @ vnew
    out = out.permute(1, 2, 0, 3).reshape(n * chunk, H, Dv)[:T]
    return out, S


# --------------------------------------------------------------------------
# sequence state
# --------------------------------------------------------------------------


@dataclass
class RefState:
    """Per-sequence cache: K/V per full-attention layer, conv+recurrent per GDN layer."""
    length: int = 0
    rope_delta: int = 0        # rotary position - cache index (negative after an image)
    k: dict[int, torch.Tensor] = field(default_factory=dict)       # [L, Hkv, D]
    v: dict[int, torch.Tensor] = field(default_factory=dict)
    conv: dict[int, torch.Tensor] = field(default_factory=dict)    # [C, K-1]
    rec: dict[int, torch.Tensor] = field(default_factory=dict)     # [Hv, Dk, Dv] f32

    def clone(self) -> "RefState":
        return RefState(self.length, self.rope_delta,
                        {i: t.clone() for i, t in self.k.items()},
                        {i: t.clone() for i, t in self.v.items()},
                        {i: t.clone() for i, t in self.conv.items()},
                        {i: t.clone() for i, t in self.rec.items()})

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for d in (self.k, self.v, self.conv, self.rec)
                   for t in d.values())


# --------------------------------------------------------------------------
# model
# --------------------------------------------------------------------------


class ReferenceModel:
    """fp32 (or any dtype) torch model over an HF-layout state dict."""

    def __init__(self, cfg: ModelConfig, weights: dict[str, torch.Tensor],
                 dtype: torch.dtype = torch.float32, device: str | torch.device = "cpu",
                 gdn_chunk_threshold: int = 64):
        self.cfg = cfg
        self.dtype = dtype
        self.device = torch.device(device)
        self.w = {k: v.to(device=self.device, dtype=dtype) for k, v in weights.items()}
        self.gdn_chunk_threshold = gdn_chunk_threshold
        if cfg.tie_word_embeddings and "lm_head.weight" not in self.w:
            self.w["lm_head.weight"] = self.w["model.embed_tokens.weight"]

    def new_state(self) -> RefState:
        return RefState()

    # ---- blocks ---------------------------------------------------------
    def _attn(self, i: int, x: torch.Tensor, st: RefState, pos0: int, pos3=None) -> torch.Tensor:
        c, p = self.cfg, f"model.layers.{i}.self_attn."
        T = x.shape[0]
        H, Hk, D = c.num_attention_heads, c.num_key_value_heads, c.head_dim
        qg = x @ self.w[p + "q_proj.weight"].t()
        if c.attn_output_gate:
            qg = qg.view(T, H, 2 * D)
            q, gate = qg[..., :D], qg[..., D:].reshape(T, H * D)
        else:
            q, gate = qg.view(T, H, D), None
        k = (x @ self.w[p + "k_proj.weight"].t()).view(T, Hk, D)
        v = (x @ self.w[p + "v_proj.weight"].t()).view(T, Hk, D)
        if c.qk_norm:
            q = rms_norm(q, self.w[p + "q_norm.weight"], c.rms_norm_eps, c.norm_offset).to(x.dtype)
            k = rms_norm(k, self.w[p + "k_norm.weight"], c.rms_norm_eps, c.norm_offset).to(x.dtype)
        if pos3 is not None:  # multimodal rotary: per-token (t, h, w) positions
            from .mrope import mrope_axis_map, mrope_cos_sin
            inv = c.rope_inv_freq()
            axes = mrope_axis_map(inv.numel(), c.mrope_section, c.mrope_interleaved)
            cos, sin = mrope_cos_sin(pos3.to(x.device), inv.to(x.device), axes.to(x.device))
        else:
            pos = torch.arange(pos0, pos0 + T, device=x.device) + st.rope_delta
            cos, sin = rope_cos_sin(pos, c.rotary_dim, c.rope_theta, c.rope_inv_freq())
        q = apply_rope(q.float(), cos, sin).to(x.dtype)
        k = apply_rope(k.float(), cos, sin).to(x.dtype)
        if i in st.k:
            K = torch.cat([st.k[i], k], 0)
            V = torch.cat([st.v[i], v], 0)
        else:
            K, V = k, v
        st.k[i], st.v[i] = K, V
        L = K.shape[0]
        rep = H // Hk
        Kr = K.repeat_interleave(rep, dim=1).float()                # [L, H, D]
        Vr = V.repeat_interleave(rep, dim=1).float()
        s = torch.einsum("thd,lhd->htl", q.float(), Kr) / math.sqrt(D)
        qpos = torch.arange(pos0, pos0 + T, device=x.device)[:, None]
        kpos = torch.arange(L, device=x.device)[None, :]
        s = s.masked_fill((kpos > qpos)[None], float("-inf"))
        pr = torch.softmax(s, -1)
        o = torch.einsum("htl,lhd->thd", pr, Vr).reshape(T, H * D)
        if gate is not None:
            o = o * torch.sigmoid(gate.float())
        return (o.to(x.dtype) @ self.w[p + "o_proj.weight"].t())

    def _gdn(self, i: int, x: torch.Tensor, st: RefState) -> torch.Tensor:
        c, p = self.cfg, f"model.layers.{i}.linear_attn."
        T = x.shape[0]
        Hk, Hv = c.linear_num_key_heads, c.linear_num_value_heads
        Dk, Dv = c.linear_key_head_dim, c.linear_value_head_dim
        r = Hv // Hk
        qkvz = (x @ self.w[p + "in_proj_qkvz.weight"].t()).view(T, Hk, 2 * Dk + 2 * r * Dv)
        ba = (x @ self.w[p + "in_proj_ba.weight"].t()).view(T, Hk, 2 * r)
        q, k, vv, z = torch.split(qkvz, [Dk, Dk, r * Dv, r * Dv], dim=-1)
        b, a = torch.split(ba, [r, r], dim=-1)
        mixed = torch.cat([q.reshape(T, -1), k.reshape(T, -1), vv.reshape(T, -1)], -1)
        convw = self.w[p + "conv1d.weight"].reshape(c.gdn_conv_dim, c.linear_conv_kernel_dim)
        if i not in st.conv:
            st.conv[i] = torch.zeros(c.gdn_conv_dim, c.linear_conv_kernel_dim - 1, dtype=x.dtype,
                                     device=x.device)
            st.rec[i] = torch.zeros(Hv, Dk, Dv, dtype=torch.float32, device=x.device)
        y, st.conv[i] = causal_conv1d(mixed, convw, st.conv[i])
        y = y.to(x.dtype)
        kd = c.gdn_key_dim
        qc = y[:, :kd].reshape(T, Hk, Dk).float()
        kc = y[:, kd:2 * kd].reshape(T, Hk, Dk).float()
        vc = y[:, 2 * kd:].reshape(T, Hv, Dv).float()
        g, beta = gdn_gating(a.reshape(T, Hv), b.reshape(T, Hv), self.w[p + "A_log"], self.w[p + "dt_bias"])
        qc = l2norm(qc.repeat_interleave(r, dim=1)) * (Dk ** -0.5)
        kc = l2norm(kc.repeat_interleave(r, dim=1))
        if T >= self.gdn_chunk_threshold:
            o, st.rec[i] = delta_rule_chunked(qc, kc, vc, g, beta, st.rec[i])
        else:
            o, st.rec[i] = delta_rule_recurrent(qc, kc, vc, g, beta, st.rec[i])
        o = gated_rms_norm(o.to(x.dtype), z.reshape(T, Hv, Dv), self.w[p + "norm.weight"], c.rms_norm_eps)
        return o.reshape(T, Hv * Dv).to(x.dtype) @ self.w[p + "out_proj.weight"].t()

    def _mlp(self, prefix: str, x: torch.Tensor) -> torch.Tensor:
        g = x @ self.w[prefix + "gate_proj.weight"].t()
        u = x @ self.w[prefix + "up_proj.weight"].t()
        return (F.silu(g.float()) * u.float()).to(x.dtype) @ self.w[prefix + "down_proj.weight"].t()

    def route(self, i: int, x: torch.Tensor):
        c = self.cfg
        logits = (x @ self.w[f"model.layers.{i}.mlp.gate.weight"].t()).float()
        probs = torch.softmax(logits, -1)
        topv, topi = torch.topk(probs, c.num_experts_per_tok, dim=-1)
        if c.norm_topk_prob:
            topv = topv / topv.sum(-1, keepdim=True)
        return topv, topi

    def _moe(self, i: int, x: torch.Tensor) -> torch.Tensor:
        c, p = self.cfg, f"model.layers.{i}.mlp."
        topv, topi = self.route(i, x)
        out = torch.zeros(x.shape[0], c.hidden_size, dtype=torch.float32, device=x.device)
        for e in topi.unique().tolist():
            rows, slot = (topi == e).nonzero(as_tuple=True)
            y = self._mlp(p + f"experts.{e}.", x[rows]).float()
            out.index_add_(0, rows, y * topv[rows, slot][:, None])
        if c.shared_expert_intermediate_size:
            sh = self._mlp(p + "shared_expert.", x).float()
            sg = torch.sigmoid((x @ self.w[p + "shared_expert_gate.weight"].t()).float())
            out = out + sg * sh
        return out.to(x.dtype)

    # ---- forward ----------------------------------------------------------
    @torch.no_grad()
    def forward(self, tokens: torch.Tensor, st: RefState, all_logits: bool = False, embeds=None, pos3=None,
                next_pos: int | None = None) -> torch.Tensor:
        """Run `tokens` ([T] int64) after the state's current length. Returns fp32 logits
        of the last token ([V]) or of every token ([T, V]). Vision-language prompts pass
        `embeds` [T, H] (image tokens spliced in), their M-RoPE positions `pos3` [3, T]
        and `next_pos`, the rotary position of the token after the prompt."""
        c = self.cfg
        pos0 = st.length
        if embeds is not None:
            x = embeds.to(device=self.device, dtype=self.dtype)
        else:
            tokens = tokens.to(self.device)
            x = self.w["model.embed_tokens.weight"][tokens]
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}."
            h = rms_norm(x, self.w[p + "input_layernorm.weight"], c.rms_norm_eps, c.norm_offset).to(x.dtype)
            h = self._gdn(i, h, st) if c.is_linear(i) else self._attn(i, h, st, pos0, pos3)
            x = x + h
            h = rms_norm(x, self.w[p + "post_attention_layernorm.weight"], c.rms_norm_eps,
                         c.norm_offset).to(x.dtype)
            h = self._moe(i, h) if c.layer_uses_moe(i) else self._mlp(p + "mlp.", h)
            x = x + h
        T = x.shape[0]
        st.length += T
        if next_pos is not None:
            st.rope_delta = next_pos - st.length
        if not all_logits:
            x = x[-1:]
        x = rms_norm(x, self.w["model.norm.weight"], c.rms_norm_eps, c.norm_offset).to(x.dtype)
        logits = (x @ self.w["lm_head.weight"].t()).float()
        return logits if all_logits else logits[0]

    @torch.no_grad()
    def hidden(self, tokens: torch.Tensor, n_layers: int) -> torch.Tensor:
        """Hidden states [T, H] after the first `n_layers` decoder layers (no final norm)
        of a fresh sequence -- the caption features a diffusion text encoder takes."""
        c = self.cfg
        st = self.new_state()
        x = self.w["model.embed_tokens.weight"][tokens.to(self.device)]
        for i in range(n_layers):
            p = f"model.layers.{i}."
            h = rms_norm(x, self.w[p + "input_layernorm.weight"], c.rms_norm_eps, c.norm_offset).to(x.dtype)
            h = self._gdn(i, h, st) if c.is_linear(i) else self._attn(i, h, st, 0)
            x = x + h
            h = rms_norm(x, self.w[p + "post_attention_layernorm.weight"], c.rms_norm_eps,
                         c.norm_offset).to(x.dtype)
            h = self._moe(i, h) if c.layer_uses_moe(i) else self._mlp(p + "mlp.", h)
            x = x + h
        return x

    # ---- snapshots --------------------------------------------------------
    def snapshot(self, st: RefState) -> RefState:
        return st.clone()

    def restore(self, snap: RefState) -> RefState:
        return snap.clone()
