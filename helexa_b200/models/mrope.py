"""Multimodal rotary position embedding (M-RoPE) for vision-language prompts.

The rotary half-dimension is split over three position axes -- temporal, height,
width -- by `mrope_section` (`[11, 11, 10]` for Qwen3.6), either interleaved per
frequency (Qwen3-VL: height on columns 1, 4, 7, ..., width on 2, 5, 8, ...) or in
contiguous blocks (Qwen2-VL). Text tokens carry the same position on all three axes,
which reduces to plain RoPE; image tokens carry their patch row / column
(arch/qwen3_5/rope.rs in the reference; HF `get_rope_index`):

  text  of length n      positions st .. st+n-1 on every axis
  image of rows x cols   t = st, h = st + row, w = st + col
  the next span starts at 1 + the largest position used so far.

Because an image's tokens share positions, the rotary position of later tokens lags
their KV-cache index; `mrope_positions` returns the position the next token takes, and
the model keeps `next - cache length` per sequence as its rotary offset for decode.
"""
from __future__ import annotations

import torch


def mrope_axis_map(half: int, section: list[int], interleaved: bool = True) -> torch.Tensor:
    """int8 [half]: the axis (0 t, 1 h, 2 w) each rotary frequency column reads."""
    ax = torch.zeros(half, dtype=torch.int8)
    if len(section) != 3:
        return ax
    if interleaved:
        for n, i in enumerate(range(1, half, 3)):
            if n < section[1]:
                ax[i] = 1
        for n, i in enumerate(range(2, half, 3)):
            if n < section[2]:
                ax[i] = 2
    else:
        h0 = min(section[0], half)
        h1 = min(section[0] + section[1], half)
        ax[h0:h1] = 1
        ax[h1:] = 2
    return ax


def mrope_positions(spans: list[tuple], start: int = 0) -> tuple[torch.Tensor, int]:
    """spans: ("text", n) or ("image", rows, cols) in prompt order. Returns int32 [3, T]
    positions and the position of the token after the prompt."""
    cols_t: list[torch.Tensor] = []
    st = start
    for sp in spans:
        if sp[0] == "text":
            n = sp[1]
            p = torch.arange(st, st + n, dtype=torch.int32)
            cols_t.append(torch.stack([p, p, p]))
            st += n
        elif sp[0] == "image":
            r, c = sp[1], sp[2]
            hh = torch.arange(r, dtype=torch.int32)[:, None].expand(r, c).reshape(-1)
            ww = torch.arange(c, dtype=torch.int32)[None, :].expand(r, c).reshape(-1)
            tt = torch.zeros(r * c, dtype=torch.int32)
            cols_t.append(torch.stack([tt + st, hh + st, ww + st]))
            st += max(r, c)
        else:
            raise ValueError(f"unknown span {sp[0]!r}")
    pos = torch.cat(cols_t, 1) if cols_t else torch.zeros(3, 0, dtype=torch.int32)
    return pos, st


def mrope_cos_sin(pos: torch.Tensor, inv_freq: torch.Tensor, axes: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """cos / sin [T, 2 * half] (rotate-half layout) for positions [3, T]."""
    p = pos.to(torch.float32)                                  # [3, T]
    sel = p[axes.long()]                                       # [half, T]: each column's axis
    freqs = sel.t() * inv_freq.float()[None, :]                # [T, half]
    emb = torch.cat([freqs, freqs], -1)
    return emb.cos(), emb.sin()
