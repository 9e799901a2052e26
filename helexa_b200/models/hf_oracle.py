"""Bridge to HF transformers' Qwen3-Next / Qwen3 / Qwen3-MoE as an external oracle.

The reference validates its in-tree Qwen3-Next against HF `Qwen3NextForCausalLM`
(crates/neuron/tests/qwen3_next_parity.rs:1-121); this module builds that HF model
from our config and loads an HF-layout state dict into it, mapping per-expert keys
onto transformers' fused expert tensors where the installed version uses them.
"""
from __future__ import annotations

import torch

from ..config import ModelConfig


def build_hf_model(cfg: ModelConfig, weights: dict[str, torch.Tensor], dtype=torch.float32):
    import transformers

    hf_cfg_dict = cfg.to_hf_config()
    if cfg.family == "qwen3_next":
        hc = transformers.Qwen3NextConfig(**{k: v for k, v in hf_cfg_dict.items()
                                             if k not in ("architectures", "model_type", "torch_dtype")})
        model = transformers.Qwen3NextForCausalLM(hc)
    elif cfg.family == "llama":
        hc = transformers.LlamaConfig(**{k: v for k, v in hf_cfg_dict.items()
                                         if k not in ("architectures", "model_type", "torch_dtype")})
        model = transformers.LlamaForCausalLM(hc)
    elif cfg.family == "qwen3_moe":
        hc = transformers.Qwen3MoeConfig(**{k: v for k, v in hf_cfg_dict.items()
                                            if k not in ("architectures", "model_type", "torch_dtype")})
        model = transformers.Qwen3MoeForCausalLM(hc)
    else:
        hc = transformers.Qwen3Config(**{k: v for k, v in hf_cfg_dict.items()
                                         if k not in ("architectures", "model_type", "torch_dtype")})
        model = transformers.Qwen3ForCausalLM(hc)
    model = model.to(dtype).eval()
    sd = model.state_dict()
    mapped: dict[str, torch.Tensor] = {}
    for k in sd:
        if k in weights:
            mapped[k] = weights[k]
        elif k.endswith("mlp.experts.gate_up_proj"):
            pre = k[: -len("gate_up_proj")]
            E = cfg.num_experts
            mapped[k] = torch.stack([torch.cat([weights[f"{pre}{e}.gate_proj.weight"],
                                                weights[f"{pre}{e}.up_proj.weight"]], 0) for e in range(E)])
        elif k.endswith("mlp.experts.down_proj"):
            pre = k[: -len("down_proj")]
            mapped[k] = torch.stack([weights[f"{pre}{e}.down_proj.weight"] for e in range(cfg.num_experts)])
        elif k == "lm_head.weight" and cfg.tie_word_embeddings:
            mapped[k] = weights["model.embed_tokens.weight"]
        else:
            raise KeyError(f"HF parameter {k} has no source tensor")
    model.load_state_dict({k: v.to(dtype) for k, v in mapped.items()}, strict=True)
    return model


@torch.no_grad()
def hf_greedy(model, prompt: list[int], n_new: int) -> tuple[list[int], list[float]]:
    """Greedy decode with HF's cache; returns new tokens and each step's top1-top2 margin."""
    ids = torch.tensor([prompt])
    out = model(input_ids=ids, use_cache=True)
    past = out.past_key_values
    logits = out.logits[0, -1].double()
    toks, margins = [], []
    for _ in range(n_new):
        top = torch.topk(logits, 2)
        margins.append(float(top.values[0] - top.values[1]))
        t = int(top.indices[0])
        toks.append(t)
        out = model(input_ids=torch.tensor([[t]]), past_key_values=past, use_cache=True)
        past = out.past_key_values
        logits = out.logits[0, -1].double()
    return toks, margins
