"""Named architectures from the benchmark configs (random-init weights of these shapes).

Shapes follow the public HF configs of the named checkpoints.
"""
from __future__ import annotations

from .model_config import FULL, LINEAR, ModelConfig


def _next_layers(n: int, interval: int = 4) -> list[str]:
    return [LINEAR if (i + 1) % interval else FULL for i in range(n)]


def tiny_qwen3_next() -> ModelConfig:
    """Tiny Qwen3-Next used for CPU fp32 token-exact parity against HF transformers."""
    return ModelConfig(
        family="qwen3_next", name="tiny-qwen3-next", vocab_size=1024, hidden_size=256,
        num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
        intermediate_size=512, rms_norm_eps=1e-6, rope_theta=1e7, partial_rotary_factor=0.25,
        attn_output_gate=True, norm_offset=1.0,
        num_experts=8, num_experts_per_tok=2, moe_intermediate_size=128,
        shared_expert_intermediate_size=128, norm_topk_prob=True,
        layer_types=_next_layers(4), linear_num_key_heads=4, linear_num_value_heads=8,
        linear_key_head_dim=32, linear_value_head_dim=32, linear_conv_kernel_dim=4,
    )


def qwen3_next_80b_a3b() -> ModelConfig:
    return ModelConfig(
        family="qwen3_next", name="Qwen3-Next-80B-A3B", vocab_size=151936, hidden_size=2048,
        num_hidden_layers=48, num_attention_heads=16, num_key_value_heads=2, head_dim=256,
        intermediate_size=5120, rms_norm_eps=1e-6, rope_theta=1e7, partial_rotary_factor=0.25,
        max_position_embeddings=262144, attn_output_gate=True, norm_offset=1.0,
        num_experts=512, num_experts_per_tok=10, moe_intermediate_size=512,
        shared_expert_intermediate_size=512, norm_topk_prob=True,
        layer_types=_next_layers(48), linear_num_key_heads=16, linear_num_value_heads=32,
        linear_key_head_dim=128, linear_value_head_dim=128, linear_conv_kernel_dim=4,
        eos_token_ids=[151645, 151643],
    )


def qwen3_8b() -> ModelConfig:
    return ModelConfig(
        family="qwen3", name="Qwen3-8B", vocab_size=151936, hidden_size=4096,
        num_hidden_layers=36, num_attention_heads=32, num_key_value_heads=8, head_dim=128,
        intermediate_size=12288, rms_norm_eps=1e-6, rope_theta=1e6, max_position_embeddings=40960,
        eos_token_ids=[151645, 151643],
    )


def qwen3_32b() -> ModelConfig:
    return ModelConfig(
        family="qwen3", name="Qwen3-32B", vocab_size=151936, hidden_size=5120,
        num_hidden_layers=64, num_attention_heads=64, num_key_value_heads=8, head_dim=128,
        intermediate_size=25600, rms_norm_eps=1e-6, rope_theta=1e6, max_position_embeddings=40960,
        eos_token_ids=[151645, 151643],
    )


def qwen3_235b_a22b() -> ModelConfig:
    return ModelConfig(
        family="qwen3_moe", name="Qwen3-235B-A22B", vocab_size=151936, hidden_size=4096,
        num_hidden_layers=94, num_attention_heads=64, num_key_value_heads=4, head_dim=128,
        intermediate_size=12288, rms_norm_eps=1e-6, rope_theta=1e6, max_position_embeddings=40960,
        num_experts=128, num_experts_per_tok=8, moe_intermediate_size=1536, norm_topk_prob=True,
        eos_token_ids=[151645, 151643],
    )


def tiny_qwen3() -> ModelConfig:
    return ModelConfig(
        family="qwen3", name="tiny-qwen3", vocab_size=1024, hidden_size=256, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=64, intermediate_size=512,
        rope_theta=1e6,
    )


def tiny_qwen3_vl() -> ModelConfig:
    """Tiny vision-language model: the tiny Qwen3 LM with interleaved M-RoPE and a
    2-block vision tower (patch 4, 2 x 2 merge) whose merger emits the LM width."""
    import dataclasses
    return dataclasses.replace(
        tiny_qwen3(), name="tiny-qwen3-vl", mrope_section=[11, 11, 10], mrope_interleaved=True,
        vision={"depth": 2, "hidden_size": 64, "intermediate_size": 128, "num_heads": 4,
                "num_position_embeddings": 64, "out_hidden_size": 256, "patch_size": 4,
                "temporal_patch_size": 2, "spatial_merge_size": 2, "in_channels": 3})


def tiny_qwen3_moe() -> ModelConfig:
    return ModelConfig(
        family="qwen3_moe", name="tiny-qwen3-moe", vocab_size=1024, hidden_size=256,
        num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
        intermediate_size=512, rope_theta=1e6, num_experts=8, num_experts_per_tok=2,
        moe_intermediate_size=128, norm_topk_prob=True,
    )


def tiny_qwen3_moe_wide() -> ModelConfig:
    """Tiny MoE with the 235B-A22B head layout scaled down (16 query / 4 KV heads, top-8
    of 16 experts), so 8-way tensor / expert parallelism replicates KV heads as the
    large model does."""
    return ModelConfig(
        family="qwen3_moe", name="tiny-qwen3-moe-wide", vocab_size=1024, hidden_size=256,
        num_hidden_layers=2, num_attention_heads=16, num_key_value_heads=4, head_dim=64,
        intermediate_size=512, rope_theta=1e6, num_experts=16, num_experts_per_tok=8,
        moe_intermediate_size=128, norm_topk_prob=True,
    )


def tiny_llama() -> ModelConfig:
    return ModelConfig(
        family="llama", name="tiny-llama", vocab_size=1024, hidden_size=256, num_hidden_layers=2,
        num_attention_heads=4, num_key_value_heads=2, head_dim=64, intermediate_size=512, rope_theta=5e5,
        qk_norm=False, rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                                     "high_freq_factor": 4.0, "original_max_position_embeddings": 64},
    )


def llama3_8b() -> ModelConfig:
    return ModelConfig(
        family="llama", name="Llama-3.1-8B", vocab_size=128256, hidden_size=4096, num_hidden_layers=32,
        num_attention_heads=32, num_key_value_heads=8, head_dim=128, intermediate_size=14336, rope_theta=5e5,
        rms_norm_eps=1e-5, qk_norm=False, max_position_embeddings=131072,
        rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                      "original_max_position_embeddings": 8192}, eos_token_ids=[128001, 128008, 128009],
    )


PRESETS = {
    "tiny-llama": tiny_llama,
    "llama-3.1-8b": llama3_8b,
    "tiny-qwen3-next": tiny_qwen3_next,
    "tiny-qwen3": tiny_qwen3,
    "tiny-qwen3-vl": tiny_qwen3_vl,
    "tiny-qwen3-moe": tiny_qwen3_moe,
    "tiny-qwen3-moe-wide": tiny_qwen3_moe_wide,
    "qwen3-next-80b-a3b": qwen3_next_80b_a3b,
    "qwen3-8b": qwen3_8b,
    "qwen3-32b": qwen3_32b,
    "qwen3-235b-a22b": qwen3_235b_a22b,
}


def get_preset(name: str) -> ModelConfig:
    key = name.lower()
    if key not in PRESETS:
        raise KeyError(f"unknown preset {name!r}; known: {sorted(PRESETS)}")
    return PRESETS[key]()
