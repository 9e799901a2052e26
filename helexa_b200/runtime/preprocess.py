"""Image preprocessing for vision-language requests (harness/preprocess.rs).

`data:image/...;base64,...` URIs from OpenAI `image_url` content parts are decoded,
resized to the native aspect with `smart_resize` (both sides multiples of
patch_size x merge_size, pixel count inside [min_pixels, max_pixels]) and normalised
per channel to the (C, H, W) f32 tensor the vision tower takes. Only data URIs are
accepted: the node does not fetch remote URLs.
"""
from __future__ import annotations

import base64
import io
import math
from dataclasses import dataclass

import torch


@dataclass
class PreprocessProfile:
    factor: int = 32
    min_pixels: int = 64 * 32 * 32
    max_pixels: int = 2304 * 16 * 16
    image_mean: tuple = (0.5, 0.5, 0.5)
    image_std: tuple = (0.5, 0.5, 0.5)


def smart_resize(h: int, w: int, factor: int, min_pixels: int, max_pixels: int) -> tuple[int, int]:
    """Factor-aligned (h, w) near the original aspect whose area lies in the budget."""
    if max(h, w) / max(1, min(h, w)) > 200:
        raise ValueError(f"aspect ratio of {h}x{w} is too extreme")
    hb = max(factor, round(h / factor) * factor)
    wb = max(factor, round(w / factor) * factor)
    if hb * wb > max_pixels:
        beta = math.sqrt(h * w / max_pixels)
        hb = max(factor, math.floor(h / beta / factor) * factor)
        wb = max(factor, math.floor(w / beta / factor) * factor)
    elif hb * wb < min_pixels:
        beta = math.sqrt(min_pixels / (h * w))
        hb = math.ceil(h * beta / factor) * factor
        wb = math.ceil(w * beta / factor) * factor
    return hb, wb


def decode_image(uri: str):
    """A `data:image/<fmt>;base64,<payload>` URI -> RGB PIL image."""
    from PIL import Image
    if not uri.startswith("data:image/") or ";base64," not in uri:
        raise ValueError("only data:image/...;base64 URIs are accepted (no remote fetches)")
    raw = base64.b64decode(uri.split(";base64,", 1)[1], validate=False)
    img = Image.open(io.BytesIO(raw))
    return img.convert("RGB")


def preprocess(img, prof: PreprocessProfile) -> torch.Tensor:
    """PIL image -> normalised f32 [3, H, W] with H, W multiples of prof.factor."""
    from PIL import Image
    w, h = img.size
    hb, wb = smart_resize(h, w, prof.factor, prof.min_pixels, prof.max_pixels)
    if (hb, wb) != (h, w):
        img = img.resize((wb, hb), Image.BICUBIC)
    x = torch.frombuffer(bytearray(img.tobytes()), dtype=torch.uint8).view(hb, wb, 3).permute(2, 0, 1).float() / 255.0
    mean = torch.tensor(prof.image_mean)[:, None, None]
    std = torch.tensor(prof.image_std)[:, None, None]
    return ((x - mean) / std).contiguous()
