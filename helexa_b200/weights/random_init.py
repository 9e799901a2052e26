"""Random-init weights for a named architecture, in HF checkpoint layout.

Every tensor is drawn from N(0, 0.02) with a single torch.Generator seeded once,
visiting tensor names in sorted order, so the same seed always yields the same
model (the tiny Qwen3-Next parity config uses seed 0). Large models are initialised
directly on the target device in bf16 with `normal_` per tensor.
"""
from __future__ import annotations

from typing import Iterator

import torch

from ..config import ModelConfig


def weight_shapes(cfg: ModelConfig) -> dict[str, tuple[int, ...]]:
    """HF-layout tensor names and shapes (per-expert keys, like the published checkpoints)."""
    h = cfg.hidden_size
    s: dict[str, tuple[int, ...]] = {"model.embed_tokens.weight": (cfg.vocab_size, h),
                                     "model.norm.weight": (h,)}
    if not cfg.tie_word_embeddings:
        s["lm_head.weight"] = (cfg.vocab_size, h)
    for i in range(cfg.num_hidden_layers):
        p = f"model.layers.{i}."
        s[p + "input_layernorm.weight"] = (h,)
        s[p + "post_attention_layernorm.weight"] = (h,)
        if cfg.is_linear(i):
            q = p + "linear_attn."
            s[q + "in_proj_qkvz.weight"] = (2 * cfg.gdn_key_dim + 2 * cfg.gdn_value_dim, h)
            s[q + "in_proj_ba.weight"] = (2 * cfg.linear_num_value_heads, h)
            s[q + "conv1d.weight"] = (cfg.gdn_conv_dim, 1, cfg.linear_conv_kernel_dim)
            s[q + "dt_bias"] = (cfg.linear_num_value_heads,)
            s[q + "A_log"] = (cfg.linear_num_value_heads,)
            s[q + "norm.weight"] = (cfg.linear_value_head_dim,)
            s[q + "out_proj.weight"] = (h, cfg.gdn_value_dim)
        else:
            q = p + "self_attn."
            s[q + "q_proj.weight"] = (cfg.q_proj_width, h)
            s[q + "k_proj.weight"] = (cfg.kv_width, h)
            s[q + "v_proj.weight"] = (cfg.kv_width, h)
            s[q + "o_proj.weight"] = (h, cfg.num_attention_heads * cfg.head_dim)
            if cfg.qk_norm:
                s[q + "q_norm.weight"] = (cfg.head_dim,)
                s[q + "k_norm.weight"] = (cfg.head_dim,)
        m = p + "mlp."
        if cfg.layer_uses_moe(i):
            s[m + "gate.weight"] = (cfg.num_experts, h)
            for e in range(cfg.num_experts):
                s[m + f"experts.{e}.gate_proj.weight"] = (cfg.moe_intermediate_size, h)
                s[m + f"experts.{e}.up_proj.weight"] = (cfg.moe_intermediate_size, h)
                s[m + f"experts.{e}.down_proj.weight"] = (h, cfg.moe_intermediate_size)
            if cfg.shared_expert_intermediate_size:
                si = cfg.shared_expert_intermediate_size
                s[m + "shared_expert.gate_proj.weight"] = (si, h)
                s[m + "shared_expert.up_proj.weight"] = (si, h)
                s[m + "shared_expert.down_proj.weight"] = (h, si)
                s[m + "shared_expert_gate.weight"] = (1, h)
        else:
            s[m + "gate_proj.weight"] = (cfg.intermediate_size, h)
            s[m + "up_proj.weight"] = (cfg.intermediate_size, h)
            s[m + "down_proj.weight"] = (h, cfg.intermediate_size)
    if cfg.vision:
        from ..models.vision import VisionConfig, vision_weight_shapes
        s.update(vision_weight_shapes(VisionConfig.from_dict(cfg.vision)))
    return s


def random_weights(cfg: ModelConfig, seed: int = 0, std: float = 0.02,
                   dtype: torch.dtype = torch.float32) -> dict[str, torch.Tensor]:
    """Deterministic CPU init (small models): one generator, sorted-name order."""
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, shape in sorted(weight_shapes(cfg).items()):
        out[name] = (torch.randn(shape, generator=g, dtype=torch.float32) * std).to(dtype)
    return out


def iter_device_init(shapes: dict[str, tuple[int, ...]], device, dtype=torch.bfloat16,
                     seed: int = 0, std: float = 0.02) -> Iterator[tuple[str, torch.Tensor]]:
    """Device-side init for large models: one CUDA generator, sorted-name order."""
    g = torch.Generator(device=device).manual_seed(seed)
    for name, shape in sorted(shapes.items()):
        t = torch.empty(shape, dtype=dtype, device=device)
        t.normal_(0.0, std, generator=g)
        yield name, t


def save_safetensors(weights: dict[str, torch.Tensor], cfg: ModelConfig, out_dir: str,
                     shard_bytes: int = 4 << 30) -> list[str]:
    """Write an HF-style checkpoint directory (config.json + sharded safetensors + index)."""
    import json
    import os

    from safetensors.torch import save_file

    os.makedirs(out_dir, exist_ok=True)
    with open(os.path.join(out_dir, "config.json"), "w") as f:
        json.dump(cfg.to_hf_config(), f, indent=1)
    shards: list[dict[str, torch.Tensor]] = [{}]
    size = 0
    for name in sorted(weights):
        t = weights[name].contiguous()
        nb = t.numel() * t.element_size()
        if size and size + nb > shard_bytes:
            shards.append({})
            size = 0
        shards[-1][name] = t
        size += nb
    files, index = [], {}
    for j, sh in enumerate(shards):
        fn = f"model-{j + 1:05d}-of-{len(shards):05d}.safetensors" if len(shards) > 1 else "model.safetensors"
        save_file(sh, os.path.join(out_dir, fn), metadata={"format": "pt"})
        files.append(fn)
        for k in sh:
            index[k] = fn
    if len(shards) > 1:
        with open(os.path.join(out_dir, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {}, "weight_map": index}, f)
    return files
