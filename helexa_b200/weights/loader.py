"""Checkpoint sources: HF safetensors directories (sharded, memory-mapped), the local HF
cache, random-init presets, and GGUF files.

Loading never materialises a full fused tensor on the device: `get(name)` maps the
tensor from the mmap'd file and the per-rank layout builder slices rows/columns on
the host before the device copy (the reference's fused-region slicer,
tp/fused_load.rs:33-213, reads per-rank byte ranges for the same reason).

Source strings (the reference's source schemes, cortex-core/src/source.rs):
  preset:<name>        random-init N(0, 0.02) weights of a named architecture
  dir:<path> / <path>  HF directory with config.json + *.safetensors
  hf:<org>/<repo>      resolved in HF_HUB_CACHE / HF_HOME (no network)
  gguf:<path>          GGUF file (Q4_K / Q6_K / Q8_0 / F16 / BF16 / F32 tensors)
"""
from __future__ import annotations

import glob
import json
import os
from dataclasses import dataclass

import torch

from ..config import ModelConfig, get_preset


class SafetensorsDir:
    def __init__(self, path: str):
        from safetensors import safe_open

        self.path = path
        index = os.path.join(path, "model.safetensors.index.json")
        if os.path.exists(index):
            with open(index) as f:
                wm = json.load(f)["weight_map"]
            files = sorted(set(wm.values()))
        else:
            files = sorted(os.path.basename(p) for p in glob.glob(os.path.join(path, "*.safetensors")))
            wm = None
        if not files:
            raise FileNotFoundError(f"no safetensors files in {path}")
        self._handles = {fn: safe_open(os.path.join(path, fn), framework="pt") for fn in files}
        self.weight_map: dict[str, str] = {}
        for fn, h in self._handles.items():
            for k in h.keys():
                self.weight_map[k] = fn
        if wm:
            self.weight_map.update({k: v for k, v in wm.items() if v in self._handles})
        # Qwen3.5/3.6 multimodal checkpoints nest the language model
        self.prefix_map = {}
        if any(k.startswith("model.language_model.") for k in self.weight_map):
            for k in list(self.weight_map):
                if k.startswith("model.language_model."):
                    self.prefix_map["model." + k[len("model.language_model."):]] = k

    def keys(self):
        return list(self.weight_map)

    def __contains__(self, name: str) -> bool:
        return name in self.weight_map or name in self.prefix_map

    def get(self, name: str) -> torch.Tensor:
        real = self.prefix_map.get(name, name)
        if real not in self.weight_map:
            real = self._fallback(name)
        return self._handles[self.weight_map[real]].get_tensor(real)

    def _fallback(self, name: str) -> str:
        # transformers >= 5 fused expert tensors are unpacked by the caller; here only
        # name aliases are resolved
        raise KeyError(f"tensor {name} not found in {self.path}")


def resolve_hf_cache(repo: str) -> str | None:
    roots = []
    if os.environ.get("HF_HUB_CACHE"):
        roots.append(os.environ["HF_HUB_CACHE"])
    if os.environ.get("HF_HOME"):
        roots.append(os.path.join(os.environ["HF_HOME"], "hub"))
    roots.append(os.path.expanduser("~/.cache/huggingface/hub"))
    d = "models--" + repo.replace("/", "--")
    for r in roots:
        snaps = os.path.join(r, d, "snapshots")
        if os.path.isdir(snaps):
            cands = sorted(glob.glob(os.path.join(snaps, "*")), key=os.path.getmtime)
            if cands:
                return cands[-1]
    return None


@dataclass
class ResolvedSource:
    kind: str            # "preset" | "dir" | "gguf"
    config: ModelConfig
    path: str | None = None
    preset: str | None = None


def resolve_source(source: str) -> ResolvedSource:
    if source.startswith("preset:"):
        name = source.split(":", 1)[1]
        return ResolvedSource("preset", get_preset(name), preset=name)
    if source.startswith("gguf:") or source.endswith(".gguf"):
        from .gguf import GGUFFile
        path = source.split(":", 1)[1] if source.startswith("gguf:") else source
        g = GGUFFile(path)
        return ResolvedSource("gguf", g.model_config(), path=path)
    if source.startswith("hf:"):
        repo = source.split(":", 1)[1]
        path = resolve_hf_cache(repo)
        if path is None:
            raise FileNotFoundError(f"{repo} is not in the local HF cache (no network access)")
    else:
        path = source.split(":", 1)[1] if source.startswith("dir:") else source
    cfgp = os.path.join(path, "config.json")
    if not os.path.exists(cfgp):
        raise FileNotFoundError(f"{path} has no config.json")
    return ResolvedSource("dir", ModelConfig.from_json_file(cfgp), path=path)


def classify_dir(path: str) -> str:
    """Preflight classification of a model directory (harness/preflight.rs:32-808):
    'gguf', 'dense', 'mixed', 'diffusers' or 'empty'."""
    files = os.listdir(path) if os.path.isdir(path) else []
    has_gguf = any(f.endswith(".gguf") for f in files)
    has_st = any(f.endswith(".safetensors") for f in files)
    if "model_index.json" in files:
        return "diffusers"
    if has_gguf and has_st:
        return "mixed"
    if has_gguf:
        return "gguf"
    if has_st:
        return "dense"
    return "empty"


def discover_capabilities(path: str) -> list[str]:
    """Capabilities of a model directory from its files alone, without loading it (the
    reference derives image / vision capability from the local HF cache the same way):
    a diffusers pipeline -> ["image"]; a config with a vision tower or vision token ids ->
    chat + completion + vision; otherwise chat + completion."""
    import json
    kind = classify_dir(path)
    if kind == "diffusers":
        return ["image"]
    caps = ["chat", "completion"]
    cfgp = os.path.join(path, "config.json")
    if os.path.exists(cfgp):
        with open(cfgp) as f:
            raw = json.load(f)
        if "vision_config" in raw or "image_token_id" in raw or "vision_start_token_id" in raw:
            caps.append("vision")
    return caps
