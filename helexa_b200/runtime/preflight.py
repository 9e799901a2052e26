"""Load preflight: classify the source and check that the requested placement can work
before any device work (harness/preflight.rs:32-808). Failures carry a reason code
and a hint, returned to the client as a structured 422.

Checks: source kind (dense safetensors / GGUF / mixed / diffusers / empty); supported
architecture; tensor-parallel divisibility per family (query heads, GDN key heads,
expert intermediate size; KV heads replicate when ranks exceed them, which the
reference refuses, tp/tp_qwen3_5.rs:564-569); GGUF under TP needs superblock-aligned
row-parallel shards; weights must fit the devices.
"""
from __future__ import annotations

from dataclasses import dataclass

from ..config import ModelConfig


@dataclass
class PreflightError(Exception):
    code: str
    message: str
    hint: str = ""

    def to_json(self) -> dict:
        return {"error": {"code": self.code, "message": self.message, "hint": self.hint, "type": "preflight"}}


def check_tp(cfg: ModelConfig, tp: int, quant: str | None = None) -> None:
    if tp < 1 or tp & (tp - 1):
        raise PreflightError("bad_tensor_parallel", f"tensor_parallel={tp} must be a power of two")
    if cfg.num_full_layers:
        if cfg.num_attention_heads % tp:
            raise PreflightError("tp_indivisible", f"{cfg.num_attention_heads} attention heads over {tp} ranks",
                                 "choose a tensor_parallel that divides the head count")
        if cfg.num_key_value_heads < tp and tp % cfg.num_key_value_heads:
            raise PreflightError("tp_indivisible", f"{cfg.num_key_value_heads} KV heads cannot be replicated "
                                 f"evenly over {tp} ranks")
    if cfg.num_linear_layers and cfg.linear_num_key_heads % tp:
        raise PreflightError("tp_indivisible", f"{cfg.linear_num_key_heads} GDN key heads over {tp} ranks")
    if cfg.num_experts and cfg.moe_intermediate_size % tp:
        raise PreflightError("tp_indivisible", f"expert intermediate {cfg.moe_intermediate_size} over {tp} ranks")
    if quant and "_K" in quant.upper():
        # row-parallel shards must hold whole 256-value superblocks: down_proj splits
        # unevenly on superblock boundaries (Qwen3-32B: 12 or 13 of 100 per rank at TP8),
        # so only a too-narrow intermediate or o_proj head slice refuses
        if cfg.intermediate_size and (cfg.intermediate_size % 256 or cfg.intermediate_size // 256 < tp):
            raise PreflightError("quant_shard_misaligned",
                                 f"{quant} down_proj ({cfg.intermediate_size} columns) cannot give each of {tp} "
                                 "ranks whole 256-value superblocks", "use a smaller tensor_parallel")
        if cfg.num_full_layers and (cfg.num_attention_heads // tp * cfg.head_dim) % 256:
            raise PreflightError("quant_shard_misaligned",
                                 f"{quant} o_proj shard of {cfg.num_attention_heads // tp} heads is not a whole "
                                 "number of superblocks", "use a smaller tensor_parallel")


def check_memory(cfg: ModelConfig, tp: int, free_bytes_per_device: list[int], bytes_per_param: float = 2.0,
                 headroom: float = 0.9) -> None:
    need = cfg.param_count() * bytes_per_param / tp
    if not free_bytes_per_device:
        return
    tight = min(free_bytes_per_device[:tp] if len(free_bytes_per_device) >= tp else free_bytes_per_device)
    if need > tight * headroom:
        raise PreflightError("insufficient_memory",
                             f"needs {need / 2**30:.1f} GiB per rank, tightest device has {tight / 2**30:.1f} GiB free",
                             "increase tensor_parallel or choose a quantized variant")


def preflight(kind: str, cfg: ModelConfig | None, tp: int = 1, quant: str | None = None,
              free_bytes_per_device: list[int] | None = None) -> None:
    if kind in ("empty",):
        raise PreflightError("no_weights", "the source has no weight files")
    if kind == "diffusers":
        raise PreflightError("wrong_modality", "diffusers pipelines are image models; this node serves text models")
    if kind == "mixed":
        raise PreflightError("ambiguous_source", "both GGUF and safetensors files found",
                             "point the source at one format")
    if cfg is None:
        raise PreflightError("no_config", "missing config.json / GGUF metadata")
    if cfg.family not in ("qwen3", "qwen3_moe", "qwen3_next", "llama"):
        raise PreflightError("unsupported_arch", f"unsupported architecture {cfg.family}")
    check_tp(cfg, tp, quant)
    if free_bytes_per_device is not None:
        bpp = {"Q4_K": 0.5625, "Q4_K_M": 0.6, "Q6_K": 0.82, "Q8_0": 1.0625}.get((quant or "").upper(), 2.0)
        check_memory(cfg, tp, free_bytes_per_device, bpp)
