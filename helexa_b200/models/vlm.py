"""Vision-language prompt assembly: text runs and images -> LM input embeddings plus
multimodal rotary positions (the reference splices vision tokens into the input
embeddings at the `<|image_pad|>` run, arch/qwen3_5/mod.rs:740-1050).

A prompt is a list of segments, ("text", token ids) or ("image", [3, H, W] normalised
image). Each image becomes rows x cols LM tokens from the vision tower (rows, cols =
H, W over patch size x merge size); text tokens come from the embedding table. The
result feeds `FastModel.prefill(None, p0, embeds=..., pos3=..., next_pos=...)` or
`ReferenceModel.forward(None, state, embeds=..., pos3=..., next_pos=...)`.
"""
from __future__ import annotations

import torch

from .mrope import mrope_positions


class VisionLanguage:
    def __init__(self, embed_table: torch.Tensor, tower):
        self.embed = embed_table
        self.tower = tower

    @torch.no_grad()
    def build(self, segments: list[tuple], start: int = 0) -> tuple[torch.Tensor, torch.Tensor, int]:
        """(embeds [T, H], pos3 int32 [3, T], rotary position after the prompt)."""
        parts, spans = [], []
        for kind, val in segments:
            if kind == "text":
                ids = torch.as_tensor(val, dtype=torch.long, device=self.embed.device)
                parts.append(self.embed[ids].float())
                spans.append(("text", len(val)))
            elif kind == "image":
                toks = self.tower.forward(val).float().to(self.embed.device)
                rows, cols = self.tower.lm_grid(val.shape[1], val.shape[2])
                parts.append(toks)
                spans.append(("image", rows, cols))
            else:
                raise ValueError(f"unknown segment {kind!r}")
        pos3, nxt = mrope_positions(spans, start)
        return torch.cat(parts, 0), pos3, nxt
