"""Qwen3-VL / Qwen3.6 vision tower: image -> LM-side tokens.

Architecture (arch/qwen3_5/vision.rs in the reference; HF `Qwen3VLVisionModel`):

  patch embed   Conv3d with kernel = stride = (temporal 2, 16, 16) over the image
                repeated along time, i.e. one linear map of each flattened
                (C, T, P, P) patch -- run as a GEMM here;
  position      learned `pos_embed` grid (48 x 48 for Qwen3.6) bilinearly
                interpolated onto the patch grid, plus a 2D rotary embedding
                (row frequencies, then column frequencies) on q and k;
  blocks        pre-LayerNorm ViT blocks: fused qkv, full (non-causal) attention,
                projection, LayerNorm, MLP (gelu-tanh), residuals;
  merger        LayerNorm, 2 x 2 spatial merge of neighbouring patches into one vector,
                fc1, GELU, fc2 -> the LM hidden size.

Patches are kept in merge-block order (each 2 x 2 group of neighbouring patches is
contiguous), so the merger is a plain reshape. On CUDA the linear layers run on the
repository's tcgen05 GEMM; LayerNorm, GELU, the rotary and attention (head dim 72 for
Qwen3.6, outside the prefill attention kernel's 64/128/256) use PyTorch ops.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F


@dataclass
class VisionConfig:
    depth: int
    hidden_size: int
    intermediate_size: int
    num_heads: int
    num_position_embeddings: int
    out_hidden_size: int
    patch_size: int = 16
    temporal_patch_size: int = 2
    spatial_merge_size: int = 2
    in_channels: int = 3
    hidden_act: str = "gelu_pytorch_tanh"

    @classmethod
    def from_dict(cls, d: dict) -> "VisionConfig":
        keys = cls.__dataclass_fields__
        return cls(**{k: v for k, v in d.items() if k in keys})

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def factor(self) -> int:
        """Image sides are multiples of this (patch size x merge size)."""
        return self.patch_size * self.spatial_merge_size


def tiny_vision_config(out_hidden: int = 256) -> VisionConfig:
    return VisionConfig(depth=2, hidden_size=64, intermediate_size=128, num_heads=4, num_position_embeddings=64,
                        out_hidden_size=out_hidden, patch_size=4)


def vision_weight_shapes(vc: VisionConfig, prefix: str = "model.visual.") -> dict[str, tuple[int, ...]]:
    h, mh = vc.hidden_size, vc.hidden_size * vc.spatial_merge_size ** 2
    s = {f"{prefix}patch_embed.proj.weight": (h, vc.in_channels, vc.temporal_patch_size, vc.patch_size,
                                              vc.patch_size),
         f"{prefix}patch_embed.proj.bias": (h,),
         f"{prefix}pos_embed.weight": (vc.num_position_embeddings, h),
         f"{prefix}merger.norm.weight": (h,), f"{prefix}merger.norm.bias": (h,),
         f"{prefix}merger.linear_fc1.weight": (mh, mh), f"{prefix}merger.linear_fc1.bias": (mh,),
         f"{prefix}merger.linear_fc2.weight": (vc.out_hidden_size, mh),
         f"{prefix}merger.linear_fc2.bias": (vc.out_hidden_size,)}
    for i in range(vc.depth):
        b = f"{prefix}blocks.{i}."
        s.update({b + "norm1.weight": (h,), b + "norm1.bias": (h,), b + "norm2.weight": (h,), b + "norm2.bias": (h,),
                  b + "attn.qkv.weight": (3 * h, h), b + "attn.qkv.bias": (3 * h,),
                  b + "attn.proj.weight": (h, h), b + "attn.proj.bias": (h,),
                  b + "mlp.linear_fc1.weight": (vc.intermediate_size, h),
                  b + "mlp.linear_fc1.bias": (vc.intermediate_size,),
                  b + "mlp.linear_fc2.weight": (h, vc.intermediate_size), b + "mlp.linear_fc2.bias": (h,)})
    return s


def random_vision_weights(vc: VisionConfig, seed: int = 0, std: float = 0.02,
                          prefix: str = "model.visual.") -> dict[str, torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    out = {}
    for name, shape in vision_weight_shapes(vc, prefix).items():
        if "norm" in name and name.endswith("weight"):
            out[name] = 1.0 + 0.1 * torch.randn(shape, generator=g)
        else:
            out[name] = torch.randn(shape, generator=g) * std
    return out


def patchify(image: torch.Tensor, vc: VisionConfig) -> tuple[torch.Tensor, tuple[int, int, int]]:
    """[C, H, W] -> flattened (C, T, P, P) patches [N, C*T*P*P] in merge-block order
    (grid_h/m, grid_w/m, m, m), the still image repeated over the temporal patch."""
    C, H, W = image.shape
    P, T, m = vc.patch_size, vc.temporal_patch_size, vc.spatial_merge_size
    if H % (P * m) or W % (P * m):
        raise ValueError(f"image {H}x{W} is not a multiple of {P * m}")
    gh, gw = H // P, W // P
    x = image.unsqueeze(0).expand(T, C, H, W)                          # [T, C, H, W]
    x = x.reshape(T, C, gh // m, m, P, gw // m, m, P)
    x = x.permute(2, 5, 3, 6, 1, 0, 4, 7)                              # [gh/m, gw/m, m, m, C, T, P, P]
    return x.reshape(gh * gw, C * T * P * P).contiguous(), (1, gh, gw)


def _merge_order(gh: int, gw: int, m: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(row, col) of every patch in merge-block order."""
    br = torch.arange(gh // m)[:, None, None, None] * m + torch.arange(m)[None, None, :, None]
    bc = torch.arange(gw // m)[None, :, None, None] * m + torch.arange(m)[None, None, None, :]
    rows = br.expand(gh // m, gw // m, m, m).reshape(-1)
    cols = bc.expand(gh // m, gw // m, m, m).reshape(-1)
    return rows, cols


class VisionTower:
    def __init__(self, vc: VisionConfig, get, device="cpu", prefix: str = "model.visual."):
        if isinstance(get, dict):
            get = get.__getitem__
        self.vc = vc
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.dtype = torch.bfloat16 if self.cuda else torch.float32
        p = prefix
        dev, dt = self.device, self.dtype

        def w(name):
            return get(p + name).to(device=dev, dtype=dt).contiguous()

        def f32(name):
            return get(p + name).to(device=dev, dtype=torch.float32).contiguous()
        self.patch_w = w("patch_embed.proj.weight").reshape(vc.hidden_size, -1).contiguous()
        self.patch_b = f32("patch_embed.proj.bias")
        self.pos_embed = f32("pos_embed.weight")
        self.blocks = []
        for i in range(vc.depth):
            b = f"blocks.{i}."
            self.blocks.append({k: (w(b + k + ".weight") if "norm" not in k else f32(b + k + ".weight"),
                                    f32(b + k + ".bias"))
                                for k in ("norm1", "attn.qkv", "attn.proj", "norm2", "mlp.linear_fc1",
                                          "mlp.linear_fc2")})
        self.merger = {k: (w("merger." + k + ".weight") if k != "norm" else f32("merger.norm.weight"),
                           f32("merger." + k + ".bias")) for k in ("norm", "linear_fc1", "linear_fc2")}
        half = vc.head_dim // 2
        self.rot_inv = 1.0 / (10000.0 ** (torch.arange(0, half, 2, dtype=torch.float32) / half))
        self.C = None
        if self.cuda:
            from .. import ops
            self.C = ops.C
            self._err = torch.zeros(1, dtype=torch.int32, device=dev)

    # ---- pieces -----------------------------------------------------------------------
    def _linear(self, x: torch.Tensor, wb) -> torch.Tensor:
        W, b = wb
        if self.C is not None and x.shape[1] % 8 == 0 and W.shape[0] % 8 == 0:
            y = torch.empty(x.shape[0], W.shape[0], dtype=torch.float32, device=x.device)
            self.C.gemm(x.to(torch.bfloat16).contiguous(), W, y, 2, self._err)
        else:
            y = x.to(W.dtype) @ W.t()
        return (y.float() + b).to(self.dtype)

    @staticmethod
    def _ln(x: torch.Tensor, wb, eps: float = 1e-6) -> torch.Tensor:
        return F.layer_norm(x.float(), (x.shape[-1],), wb[0], wb[1], eps).to(x.dtype)

    def _act(self, x: torch.Tensor) -> torch.Tensor:
        approx = "tanh" if self.vc.hidden_act in ("gelu_pytorch_tanh", "gelu_new", "gelu_tanh") else "none"
        return F.gelu(x.float(), approximate=approx).to(x.dtype)

    def pos_embed_interp(self, gh: int, gw: int) -> torch.Tensor:
        """Bilinear interpolation of the learned grid onto gh x gw patches (row-major)."""
        n = int(round(math.sqrt(self.vc.num_position_embeddings)))
        hs = torch.linspace(0, n - 1, gh)
        ws = torch.linspace(0, n - 1, gw)
        hf, wf = hs.int(), ws.int()
        hc, wc = (hf + 1).clamp(max=n - 1), (wf + 1).clamp(max=n - 1)
        dh, dw = (hs - hf)[:, None], (ws - wf)[None, :]
        tab = self.pos_embed.cpu()

        def at(r, c):
            return tab[(r[:, None] * n + c[None, :]).reshape(-1)].reshape(gh, gw, -1)
        out = (at(hf, wf) * ((1 - dh) * (1 - dw))[..., None] + at(hf, wc) * ((1 - dh) * dw)[..., None]
               + at(hc, wf) * (dh * (1 - dw))[..., None] + at(hc, wc) * (dh * dw)[..., None])
        return out.reshape(gh * gw, -1)

    def rotary(self, gh: int, gw: int) -> tuple[torch.Tensor, torch.Tensor]:
        rows, cols = _merge_order(gh, gw, self.vc.spatial_merge_size)
        fr = torch.cat([rows[:, None].float() * self.rot_inv[None], cols[:, None].float() * self.rot_inv[None]], 1)
        emb = torch.cat([fr, fr], 1)
        return emb.cos().to(self.device), emb.sin().to(self.device)

    @staticmethod
    def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        x1, x2 = x[..., : x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
        return x * cos + torch.cat([-x2, x1], -1) * sin

    # ---- forward ------------------------------------------------------------------------
    @torch.no_grad()
    def forward_patches(self, patches: torch.Tensor, grid: tuple[int, int, int]) -> torch.Tensor:
        vc = self.vc
        _, gh, gw = grid
        m = vc.spatial_merge_size
        x = self._linear(patches.to(self.device), (self.patch_w, self.patch_b))
        pos = self.pos_embed_interp(gh, gw)
        rows, cols = _merge_order(gh, gw, m)
        x = (x.float() + pos[rows * gw + cols].to(self.device)).to(self.dtype)
        cos, sin = self.rotary(gh, gw)
        N, h, nh, hd = x.shape[0], vc.hidden_size, vc.num_heads, vc.head_dim
        for blk in self.blocks:
            a = self._ln(x, blk["norm1"])
            qkv = self._linear(a, blk["attn.qkv"]).view(N, 3, nh, hd).float()
            q = self._rope(qkv[:, 0], cos[:, None], sin[:, None])
            k = self._rope(qkv[:, 1], cos[:, None], sin[:, None])
            v = qkv[:, 2]
            o = F.scaled_dot_product_attention(q.transpose(0, 1)[None].to(self.dtype),
                                               k.transpose(0, 1)[None].to(self.dtype),
                                               v.transpose(0, 1)[None].to(self.dtype))[0]
            x = (x.float() + self._linear(o.transpose(0, 1).reshape(N, h), blk["attn.proj"]).float()).to(self.dtype)
            a = self._ln(x, blk["norm2"])
            mlp = self._linear(self._act(self._linear(a, blk["mlp.linear_fc1"])), blk["mlp.linear_fc2"])
            x = (x.float() + mlp.float()).to(self.dtype)
        x = self._ln(x, self.merger["norm"]).reshape(N // (m * m), h * m * m)
        x = self._linear(x, self.merger["linear_fc1"])
        x = F.gelu(x.float()).to(self.dtype)
        return self._linear(x, self.merger["linear_fc2"])

    def forward(self, image: torch.Tensor) -> torch.Tensor:
        """[C, H, W] normalised image -> [N_lm, out_hidden] LM-side tokens."""
        patches, grid = patchify(image.float(), self.vc)
        return self.forward_patches(patches, grid)

    def lm_grid(self, H: int, W: int) -> tuple[int, int]:
        """(rows, cols) of LM tokens an H x W image becomes."""
        f = self.vc.factor
        return H // f, W // f
