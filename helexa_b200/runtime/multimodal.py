"""Images in chat requests -> one multimodal prefill (the reference's vision path:
preprocess, vision tower, splice at the `<|image_pad|>` run, M-RoPE positions;
harness/preprocess.rs, arch/qwen3_5/mod.rs:740-1050, arch/qwen3_5/vision.rs).

The chat template renders every image content part as
`<|vision_start|><|image_pad|><|vision_end|>`. `VisionFrontend.build` decodes and
resizes the images in message order, runs the tower, and expands each single pad
token to the image's rows x cols LM tokens, returning the prompt's input embeddings,
its [3, T] rotary positions and the position after it. The engine prefills such a
prompt in one pass with no prefix-cache lookup (the cache is keyed by token ids,
which do not identify an image).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from ..models.vision import VisionConfig, VisionTower
from ..models.vlm import VisionLanguage
from .preprocess import PreprocessProfile, decode_image, preprocess

IMAGE_PART_TYPES = ("image_url", "input_image", "image")
VISION_START, IMAGE_PAD, VISION_END = "<|vision_start|>", "<|image_pad|>", "<|vision_end|>"


def image_placeholder() -> str:
    return VISION_START + IMAGE_PAD + VISION_END


def _part_uri(p: dict) -> str | None:
    v = p.get("image_url", p.get("image"))
    if isinstance(v, dict):
        v = v.get("url")
    return v if isinstance(v, str) else None


def request_images(messages) -> list[str]:
    """Image URIs of the request's content parts, in prompt order."""
    out = []
    for m in messages or []:
        content = m.get("content") if isinstance(m, dict) else None
        if isinstance(content, list):
            for p in content:
                if isinstance(p, dict) and p.get("type") in IMAGE_PART_TYPES:
                    uri = _part_uri(p)
                    if uri is None:
                        raise ValueError("image content part without a URL")
                    out.append(uri)
    return out


@dataclass
class MultimodalPrompt:
    tokens: list[int]          # prompt ids with each image's pad expanded to its token count
    embeds: torch.Tensor       # [T, H] LM input rows (image tokens spliced in)
    pos3: torch.Tensor         # int32 [3, T] rotary (t, h, w) positions
    next_pos: int              # rotary position of the first generated token


class VisionFrontend:
    def __init__(self, embed_table: torch.Tensor, tower: VisionTower, pad_id: int,
                 profile: PreprocessProfile | None = None, max_images: int = 8):
        self.vl = VisionLanguage(embed_table, tower)
        self.tower = tower
        self.pad_id = pad_id
        f = tower.vc.factor
        # the reference's pixel budget (64 to 576 LM tokens per image) at this tower's factor
        self.profile = profile or PreprocessProfile(factor=f, min_pixels=64 * f * f, max_pixels=576 * f * f)
        self.max_images = max_images

    @classmethod
    def from_weights(cls, cfg, get, embed_table, tokenizer, device="cpu", prefix: str = "model.visual."):
        pad = tokenizer.token_id(IMAGE_PAD)
        if pad is None:
            raise ValueError(f"tokenizer has no {IMAGE_PAD} token")
        tower = VisionTower(VisionConfig.from_dict(cfg.vision), get, device=device, prefix=prefix)
        return cls(embed_table, tower, pad)

    @torch.no_grad()
    def build(self, ids: list[int], uris: list[str]) -> MultimodalPrompt:
        pads = [i for i, t in enumerate(ids) if t == self.pad_id]
        if len(pads) != len(uris):
            raise ValueError(f"{len(uris)} images but {len(pads)} image placeholders in the rendered prompt")
        if len(uris) > self.max_images:
            raise ValueError(f"at most {self.max_images} images per request")
        segments, tokens, prev = [], [], 0
        for at, uri in zip(pads, uris):
            img = preprocess(decode_image(uri), self.profile)
            if at > prev:
                segments.append(("text", ids[prev:at]))
            segments.append(("image", img))
            rows, cols = self.tower.lm_grid(img.shape[1], img.shape[2])
            tokens += ids[prev:at] + [self.pad_id] * (rows * cols)
            prev = at + 1
        if prev < len(ids):
            segments.append(("text", ids[prev:]))
            tokens += ids[prev:]
        embeds, pos3, nxt = self.vl.build(segments)
        assert embeds.shape[0] == len(tokens)
        return MultimodalPrompt(tokens=tokens, embeds=embeds, pos3=pos3, next_pos=nxt)
