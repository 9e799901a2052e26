"""Image models on the node: load a Z-Image pipeline and serve
`POST /v1/images/generations` (api.rs:519-613 and harness/candle.rs
`image_generation` in the reference).

A served image model owns one `ZImagePipeline`; generations run one at a time on a
worker thread (the DiT and VAE are resident, the text encoder runs on the CPU like the
reference's default `te_on_cpu`). The request surface matches the reference: n = 1,
`response_format` b64_json, `output_format` png, `size` "WxH" (default 1024x1024),
`num_steps`, `guidance_scale` (with `negative_prompt`: classifier-free guidance), `seed`;
the response carries `usage.helexa_image_units` (megapixel-steps) and
`usage.helexa_timing`.
"""
from __future__ import annotations

import asyncio
import base64
import json
import os
import threading
import time
from dataclasses import dataclass, field

import torch

from ..models import zimage as zi

IMAGE_PRESETS = ("tiny-z-image", "z-image-turbo")


class ImageRequestError(ValueError):
    def __init__(self, message: str, code: str = "invalid_request_error", status: int = 400):
        super().__init__(message)
        self.code, self.status = code, status


def is_image_source(source: str) -> bool:
    if source.startswith("preset:"):
        return source.split(":", 1)[1] in IMAGE_PRESETS
    path = source.split(":", 1)[1] if source.startswith("dir:") else source
    return os.path.isdir(path) and os.path.exists(os.path.join(path, "model_index.json"))


def _preset_pipeline(name: str, device) -> zi.ZImagePipeline:
    from ..config import get_preset
    from ..models.reference import ReferenceModel
    from ..weights.random_init import random_weights as lm_weights
    if name == "tiny-z-image":
        lm_cfg = get_preset("tiny-qwen3")
        dcfg, vcfg = zi.tiny_dit_config(lm_cfg.hidden_size), zi.tiny_vae_config()
        tile = 8
    else:  # full-size architecture, random-init weights (no checkpoint download here)
        import dataclasses
        lm_cfg = dataclasses.replace(get_preset("qwen3-8b"), name="Qwen3-4B", hidden_size=2560, num_hidden_layers=36,
                                     num_attention_heads=32, num_key_value_heads=8, intermediate_size=9728,
                                     tie_word_embeddings=True)
        dcfg, vcfg = zi.DiTConfig(), zi.VaeConfig()
        tile = 64
    te = zi.TextEncoder(ReferenceModel(lm_cfg, lm_weights(lm_cfg, seed=1)))
    dw = zi.random_weights(zi.dit_weight_shapes(dcfg), seed=2, device=device if device.type == "cuda" else "cpu",
                           dtype=torch.bfloat16 if device.type == "cuda" else torch.float32)
    vw = zi.random_weights(zi.vae_decoder_shapes(vcfg), seed=3)
    dit = zi.ZImageDiT(dcfg, dw, device)
    vae = zi.VaeDecoder(vcfg, vw, device, torch.bfloat16 if device.type == "cuda" else torch.float32)
    return zi.ZImagePipeline(dit, vae, te, tokenizer=None, tile=tile, overlap=tile // 4)


def load_pipeline_dir(path: str, device, te_device: str = "cpu") -> zi.ZImagePipeline:
    """A diffusers-layout Z-Image directory: transformer/, vae/, text_encoder/,
    tokenizer/ (each with its config and safetensors)."""
    from ..config.model_config import ModelConfig
    from ..models.reference import ReferenceModel
    from ..weights.loader import SafetensorsDir
    from .tokenizer import load_tokenizer
    with open(os.path.join(path, "model_index.json")) as f:
        if not zi.is_supported_pipeline_class(f.read()):
            raise ValueError(f"{path}: model_index.json does not declare a ZImagePipeline")

    def cfg_of(sub):
        with open(os.path.join(path, sub, "config.json")) as f:
            return json.load(f)

    dcfg = zi.DiTConfig.from_json(cfg_of("transformer"))
    vcfg = zi.VaeConfig.from_json(cfg_of("vae"))
    st = SafetensorsDir(os.path.join(path, "transformer"))
    dit = zi.ZImageDiT(dcfg, {k: st.get(k) for k in st.keys()}, device)
    vs = SafetensorsDir(os.path.join(path, "vae"))
    vae = zi.VaeDecoder(vcfg, {k: vs.get(k) for k in vs.keys() if k.startswith("decoder.")}, device,
                        torch.bfloat16 if torch.device(device).type == "cuda" else torch.float32)
    lm_cfg = ModelConfig.from_json_file(os.path.join(path, "text_encoder", "config.json"))
    ts = SafetensorsDir(os.path.join(path, "text_encoder"))
    te = zi.TextEncoder(ReferenceModel(lm_cfg, {k: ts.get(k) for k in ts.keys()}, device=te_device))
    tok = load_tokenizer(os.path.join(path, "tokenizer"), lm_cfg.vocab_size)
    return zi.ZImagePipeline(dit, vae, te, tokenizer=tok)


@dataclass
class ServedImageModel:
    model_id: str
    pipeline: zi.ZImagePipeline
    devices: list = field(default_factory=list)
    spec: dict = field(default_factory=dict)
    status: str = "loaded"
    capabilities: list = field(default_factory=lambda: ["image"])
    max_dim: int = zi.DEFAULT_MAX_DIM
    generations: int = 0

    def __post_init__(self):
        self._lock = threading.Lock()

    def _tokens(self, prompt):
        tok = self.pipeline.tok
        if tok is None:  # random-init presets: bytes of the wrapped prompt, folded into the vocab
            vocab = self.pipeline.te.m.cfg.vocab_size
            return [b % vocab for b in zi.format_prompt(prompt).encode()]
        return tok.encode(zi.format_prompt(prompt))

    def validate(self, body: dict) -> dict:
        """Request body -> generation arguments (400-class errors raise ImageRequestError)."""
        n = body.get("n", 1)
        if n != 1:
            raise ImageRequestError(f"n={n} is not supported; this endpoint serves n=1", "unsupported_parameter")
        rf = body.get("response_format")
        if rf is not None and rf != "b64_json":
            raise ImageRequestError(f"response_format '{rf}' is not supported; use b64_json", "unsupported_parameter")
        of = body.get("output_format")
        if of is not None and of != "png":
            raise ImageRequestError(f"output_format '{of}' is not supported; use png", "unsupported_parameter")
        try:
            width, height = zi.parse_size(body.get("size"))
            zi.validate_dims(width, height, self.max_dim)
        except ValueError as e:
            raise ImageRequestError(str(e), "invalid_size") from None
        steps = body.get("num_steps", zi.DEFAULT_STEPS)
        try:
            zi.validate_steps(int(steps))
        except ValueError as e:
            raise ImageRequestError(str(e)) from None
        prompt = body.get("prompt")
        if not isinstance(prompt, str) or not prompt:
            raise ImageRequestError("prompt must be a non-empty string")
        neg = body.get("negative_prompt")
        return dict(prompt=self._tokens(prompt), negative_prompt=self._tokens(neg) if neg else None,
                    width=width, height=height, steps=int(steps),
                    guidance_scale=float(body.get("guidance_scale", zi.DEFAULT_GUIDANCE_SCALE)),
                    seed=body.get("seed"))

    def generate_sync(self, args: dict) -> dict:
        with self._lock:
            r = self.pipeline.generate(**args)
        self.generations += 1
        png = zi.encode_png(r.rgb, r.width, r.height)
        t = r.timing
        return {"created": int(time.time()), "data": [{"b64_json": base64.b64encode(png).decode()}],
                "usage": {"helexa_image_units": zi.megapixel_steps(r.width, r.height, t.steps, t.cfg),
                          "helexa_timing": {"encode_ms": round(t.encode_ms, 1), "denoise_ms": round(t.denoise_ms, 1),
                                            "decode_ms": round(t.decode_ms, 1), "steps": t.steps, "cfg": t.cfg}}}

    async def generate(self, body: dict) -> dict:
        args = self.validate(body)
        return await asyncio.to_thread(self.generate_sync, args)

    def describe(self) -> dict:
        return {"id": self.model_id, "status": self.status, "devices": self.devices, "tensor_parallel": 1,
                "capabilities": self.capabilities, "limit": None, "servable": self.status == "loaded"}


def build_image_model(spec) -> ServedImageModel:
    use_cuda = (spec.device or ("cuda" if torch.cuda.is_available() else "cpu")) == "cuda"
    dev = torch.device("cuda", (spec.devices or [0])[0]) if use_cuda else torch.device("cpu")
    src = spec.source
    if src.startswith("preset:"):
        pipe = _preset_pipeline(src.split(":", 1)[1], dev)
    else:
        pipe = load_pipeline_dir(src.split(":", 1)[1] if src.startswith("dir:") else src, dev)
    if spec.quant:
        zi.parse_image_quant(spec.quant)  # reject anything but q8_0 before any work
        pipe.dit.quantize_(spec.quant)
    return ServedImageModel(model_id=spec.model_id, pipeline=pipe, devices=[dev.index] if use_cuda else [],
                            spec={"source": spec.source})
