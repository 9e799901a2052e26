"""Model configuration for the served families: Qwen3 dense, Qwen3-MoE and Qwen3-Next.

One dataclass describes all three. A model is a stack of decoder layers whose token
mixer is either full attention or Gated DeltaNet (linear attention), and whose FFN is
either a dense SwiGLU MLP or a sparse MoE block.

Parity notes (reference behaviour this mirrors):
  * nested `text_config` (Qwen3.5/3.6) or flat `qwen3_next` config.json parsing, with
    `layer_types` derived from `full_attention_interval` when absent:
    crates/neuron/src/harness/arch/qwen3_5/mod.rs:104-365
  * Qwen3-Next forces the attention output gate and uses `(1+w)` RMSNorm weights:
    crates/neuron/src/harness/arch/qwen3_5/full_attn.rs:112-160,
    crates/neuron/src/harness/arch/qwen3_5/rmsnorm.rs:31-80
  * MoE-layer selection (`decoder_sparse_step`, `mlp_only_layers`):
    crates/neuron/src/harness/arch/qwen3_5/mod.rs (layer_uses_moe)
"""
from __future__ import annotations

import dataclasses
import json
import os
from dataclasses import dataclass, field
from typing import Any

FULL = "full_attention"
LINEAR = "linear_attention"


@dataclass
class ModelConfig:
    family: str                     # "qwen3" | "qwen3_moe" | "qwen3_next" | "llama"
    vocab_size: int
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int = 0      # dense MLP width (0 when every layer is MoE)
    rms_norm_eps: float = 1e-6
    rope_theta: float = 1e6
    partial_rotary_factor: float = 1.0
    max_position_embeddings: int = 32768
    tie_word_embeddings: bool = False
    # attention flavour
    attn_output_gate: bool = False  # Qwen3-Next: q_proj emits [q | gate] per head
    norm_offset: float = 0.0        # 1.0 for "(1+w)" RMSNorm (Qwen3-Next), 0.0 for plain w
    qk_norm: bool = True
    # MoE
    num_experts: int = 0
    num_experts_per_tok: int = 0
    moe_intermediate_size: int = 0
    shared_expert_intermediate_size: int = 0
    norm_topk_prob: bool = True
    decoder_sparse_step: int = 1
    mlp_only_layers: list[int] = field(default_factory=list)
    # Gated DeltaNet
    layer_types: list[str] = field(default_factory=list)
    linear_num_key_heads: int = 0
    linear_num_value_heads: int = 0
    linear_key_head_dim: int = 0
    linear_value_head_dim: int = 0
    linear_conv_kernel_dim: int = 4
    rope_scaling: dict | None = None  # e.g. {"rope_type": "llama3", "factor": 8, ...}
    # multimodal rotary (vision-language checkpoints): [temporal, height, width] split of
    # the rotary half-dim, interleaved per frequency (Qwen3-VL) or in blocks (Qwen2-VL)
    mrope_section: list[int] = field(default_factory=list)
    mrope_interleaved: bool = True
    vision: dict | None = None         # the checkpoint's vision_config, when present
    # bookkeeping
    name: str = ""
    eos_token_ids: list[int] = field(default_factory=list)
    bos_token_id: int | None = None

    def __post_init__(self) -> None:
        if not self.layer_types:
            self.layer_types = [FULL] * self.num_hidden_layers
        if len(self.layer_types) != self.num_hidden_layers:
            raise ValueError("layer_types length must equal num_hidden_layers")

    # ---- derived shapes -------------------------------------------------
    @property
    def rotary_dim(self) -> int:
        return int(self.head_dim * self.partial_rotary_factor)

    @property
    def q_proj_width(self) -> int:
        return self.num_attention_heads * self.head_dim * (2 if self.attn_output_gate else 1)

    @property
    def kv_width(self) -> int:
        return self.num_key_value_heads * self.head_dim

    @property
    def gdn_key_dim(self) -> int:
        return self.linear_num_key_heads * self.linear_key_head_dim

    @property
    def gdn_value_dim(self) -> int:
        return self.linear_num_value_heads * self.linear_value_head_dim

    @property
    def gdn_conv_dim(self) -> int:
        return 2 * self.gdn_key_dim + self.gdn_value_dim

    def is_linear(self, i: int) -> bool:
        return self.layer_types[i] == LINEAR

    def layer_uses_moe(self, i: int) -> bool:
        return (self.num_experts > 0 and i not in self.mlp_only_layers
                and (i + 1) % self.decoder_sparse_step == 0)

    @property
    def num_full_layers(self) -> int:
        return sum(1 for t in self.layer_types if t == FULL)

    @property
    def num_linear_layers(self) -> int:
        return sum(1 for t in self.layer_types if t == LINEAR)

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        """K+V bytes per token over every full-attention layer (GDN layers hold O(1) state)."""
        return 2 * self.num_full_layers * self.kv_width * dtype_bytes

    def gdn_state_bytes(self) -> int:
        """Per-sequence recurrent (f32) + conv (bf16) state bytes across every GDN layer."""
        rec = self.linear_num_value_heads * self.linear_key_head_dim * self.linear_value_head_dim * 4
        conv = self.gdn_conv_dim * self.linear_conv_kernel_dim * 2
        return self.num_linear_layers * (rec + conv)

    def param_count(self) -> int:
        h = self.hidden_size
        n = self.vocab_size * h * (1 if self.tie_word_embeddings else 2) + h
        for i in range(self.num_hidden_layers):
            n += 2 * h
            if self.is_linear(i):
                n += h * (2 * self.gdn_key_dim + 2 * self.gdn_value_dim)
                n += h * 2 * self.linear_num_value_heads
                n += self.gdn_conv_dim * self.linear_conv_kernel_dim
                n += self.gdn_value_dim * h + 2 * self.linear_num_value_heads + self.linear_value_head_dim
            else:
                n += h * self.q_proj_width + 2 * h * self.kv_width + self.num_attention_heads * self.head_dim * h
                n += 2 * self.head_dim
            if self.layer_uses_moe(i):
                n += self.num_experts * 3 * h * self.moe_intermediate_size + self.num_experts * h
                if self.shared_expert_intermediate_size:
                    n += 3 * h * self.shared_expert_intermediate_size + h
            else:
                n += 3 * h * self.intermediate_size
        return n

    def rope_inv_freq(self):
        """Inverse RoPE frequencies [rotary_dim/2] (f32), with llama3-style scaling when configured."""
        import math

        import torch
        rd = self.rotary_dim
        inv = 1.0 / (self.rope_theta ** (torch.arange(0, rd, 2, dtype=torch.int64).float() / rd))
        rs = self.rope_scaling or {}
        if rs.get("rope_type", rs.get("type")) == "llama3":
            factor = float(rs.get("factor", 8.0))
            lo, hi = float(rs.get("low_freq_factor", 1.0)), float(rs.get("high_freq_factor", 4.0))
            old = float(rs.get("original_max_position_embeddings", 8192))
            lo_wl, hi_wl = old / lo, old / hi
            wl = 2 * math.pi / inv
            smooth = (old / wl - lo) / (hi - lo)
            scaled = torch.where(wl > lo_wl, inv / factor, inv)
            mid = (wl <= lo_wl) & (wl >= hi_wl)
            scaled = torch.where(mid, (1 - smooth) * inv / factor + smooth * inv, scaled)
            inv = scaled
        return inv

    def to_dict(self) -> dict[str, Any]:
        return dataclasses.asdict(self)

    # ---- HF config.json -------------------------------------------------
    def to_hf_config(self) -> dict[str, Any]:
        """Emit an HF-style config.json dict that `from_hf_config` (and transformers) parse."""
        arch = {"qwen3": "Qwen3ForCausalLM", "qwen3_moe": "Qwen3MoeForCausalLM",
                "qwen3_next": "Qwen3NextForCausalLM", "llama": "LlamaForCausalLM"}[self.family]
        d: dict[str, Any] = {
            "architectures": [arch], "model_type": self.family,
            "vocab_size": self.vocab_size, "hidden_size": self.hidden_size,
            "num_hidden_layers": self.num_hidden_layers,
            "num_attention_heads": self.num_attention_heads,
            "num_key_value_heads": self.num_key_value_heads, "head_dim": self.head_dim,
            "intermediate_size": self.intermediate_size, "rms_norm_eps": self.rms_norm_eps,
            "rope_theta": self.rope_theta, "max_position_embeddings": self.max_position_embeddings,
            "tie_word_embeddings": self.tie_word_embeddings, "hidden_act": "silu",
            "attention_bias": False, "torch_dtype": "bfloat16",
            "rope_parameters": dict(self.rope_scaling or {"rope_type": "default"}, rope_theta=self.rope_theta,
                                    partial_rotary_factor=self.partial_rotary_factor),
        }
        if self.eos_token_ids:
            d["eos_token_id"] = self.eos_token_ids if len(self.eos_token_ids) > 1 else self.eos_token_ids[0]
        if self.family in ("qwen3_moe", "qwen3_next"):
            d.update(num_experts=self.num_experts, num_experts_per_tok=self.num_experts_per_tok,
                     moe_intermediate_size=self.moe_intermediate_size,
                     norm_topk_prob=self.norm_topk_prob, decoder_sparse_step=self.decoder_sparse_step,
                     mlp_only_layers=list(self.mlp_only_layers))
        if self.family == "qwen3_next":
            d.update(shared_expert_intermediate_size=self.shared_expert_intermediate_size,
                     layer_types=list(self.layer_types),
                     linear_num_key_heads=self.linear_num_key_heads,
                     linear_num_value_heads=self.linear_num_value_heads,
                     linear_key_head_dim=self.linear_key_head_dim,
                     linear_value_head_dim=self.linear_value_head_dim,
                     linear_conv_kernel_dim=self.linear_conv_kernel_dim,
                     partial_rotary_factor=self.partial_rotary_factor)
        return d

    @classmethod
    def from_hf_config(cls, raw: dict[str, Any], name: str = "") -> "ModelConfig":
        # Qwen3.5/3.6 nest the language model under text_config.
        if "text_config" in raw and isinstance(raw["text_config"], dict):
            merged = dict(raw["text_config"])
            merged.setdefault("model_type", raw.get("model_type", "qwen3_next"))
            raw = merged
        mt = raw.get("model_type", "qwen3")
        archs = raw.get("architectures") or []
        if mt in ("qwen3_next", "qwen3_5", "qwen3_5_text", "qwen3_5_moe", "qwen3_5_moe_text") or \
                any("Next" in a or "Qwen3_5" in a for a in archs):
            family = "qwen3_next"
        elif mt == "qwen3_moe" or any("Moe" in a for a in archs):
            family = "qwen3_moe"
        elif mt == "qwen3":
            family = "qwen3"
        elif mt == "llama" or any("Llama" in a for a in archs):
            family = "llama"
        else:
            raise ValueError(f"unsupported model_type {mt!r} (architectures {archs})")
        vision = raw.get("vision_config")
        if "text_config" in raw:  # vision-language checkpoints nest the LM config
            outer = raw
            raw = dict(raw["text_config"])
            raw.setdefault("vocab_size", outer.get("vocab_size"))
        rope = raw.get("rope_parameters") or raw.get("rope_scaling") or {}
        theta = float(rope.get("rope_theta", raw.get("rope_theta", 1e6)))
        prf = float(raw.get("partial_rotary_factor", rope.get("partial_rotary_factor",
                    0.25 if family == "qwen3_next" else 1.0)))
        nl = int(raw["num_hidden_layers"])
        layer_types = list(raw.get("layer_types") or [])
        if family == "qwen3_next" and not layer_types:
            interval = int(raw.get("full_attention_interval", 4))
            layer_types = [LINEAR if (i + 1) % interval else FULL for i in range(nl)]
        eos = raw.get("eos_token_id")
        eos_ids = [] if eos is None else ([eos] if isinstance(eos, int) else list(eos))
        heads = int(raw["num_attention_heads"])
        return cls(
            family=family, name=name,
            vocab_size=int(raw["vocab_size"]), hidden_size=int(raw["hidden_size"]),
            num_hidden_layers=nl, num_attention_heads=heads,
            num_key_value_heads=int(raw.get("num_key_value_heads", heads)),
            head_dim=int(raw.get("head_dim") or raw["hidden_size"] // heads),
            intermediate_size=int(raw.get("intermediate_size", 0) or 0),
            rms_norm_eps=float(raw.get("rms_norm_eps", 1e-6)), rope_theta=theta,
            partial_rotary_factor=prf,
            max_position_embeddings=int(raw.get("max_position_embeddings", 32768)),
            tie_word_embeddings=bool(raw.get("tie_word_embeddings", False)),
            attn_output_gate=(family == "qwen3_next"), qk_norm=(family != "llama"),
            rope_scaling=(rope if rope.get("rope_type", rope.get("type", "default")) not in (None, "default")
                          else None),
            norm_offset=1.0 if family == "qwen3_next" else 0.0,
            num_experts=int(raw.get("num_experts", 0) or 0),
            num_experts_per_tok=int(raw.get("num_experts_per_tok", 0) or 0),
            moe_intermediate_size=int(raw.get("moe_intermediate_size", 0) or 0),
            shared_expert_intermediate_size=int(raw.get("shared_expert_intermediate_size", 0) or 0),
            norm_topk_prob=bool(raw.get("norm_topk_prob", True)),
            decoder_sparse_step=int(raw.get("decoder_sparse_step", 1) or 1),
            mlp_only_layers=list(raw.get("mlp_only_layers") or []),
            layer_types=layer_types,
            linear_num_key_heads=int(raw.get("linear_num_key_heads", 0) or 0),
            linear_num_value_heads=int(raw.get("linear_num_value_heads", 0) or 0),
            linear_key_head_dim=int(raw.get("linear_key_head_dim", 0) or 0),
            linear_value_head_dim=int(raw.get("linear_value_head_dim", 0) or 0),
            linear_conv_kernel_dim=int(raw.get("linear_conv_kernel_dim", 4) or 4),
            eos_token_ids=eos_ids, bos_token_id=raw.get("bos_token_id"),
            mrope_section=list(rope.get("mrope_section") or []),
            mrope_interleaved=bool(rope.get("mrope_interleaved", True)),
            vision=vision,
        )

    @classmethod
    def from_json_file(cls, path: str) -> "ModelConfig":
        with open(path) as f:
            raw = json.load(f)
        return cls.from_hf_config(raw, name=os.path.basename(os.path.dirname(os.path.abspath(path))))
