"""Z-Image text-to-image: single-stream diffusion transformer (S3-DiT), 16-channel VAE
decoder, flow-matching Euler sampler and the pipeline around them.

The reference wraps candle-transformers' `z_image` family behind its device worker
(harness/image.rs:1-19, generate at :413-524): a Qwen3-4B text encoder (the hidden
states one layer below the top), a 6B DiT run for `steps` flow-matching steps with
optional classifier-free guidance, and a tiled VAE decode. This module is written for
one B200:

* the DiT runs in bf16 on the device: every projection on the tcgen05 GEMM
  (`csrc/gemm_tcgen05.cu`; the FFN's gate / up rows are interleaved so the SwiGLU is the
  GEMM's epilogue), attention on the tcgen05 flash-attention kernel in bidirectional
  mode (`csrc/attn_prefill_tc.cu`), the modulated norms, gated residuals and the
  q/k-norm + 3-axis RoPE in `csrc/dit_ops.cu`. A plain-torch path of the same math
  (fp32 on the CPU) is the oracle the GPU path is tested against;
* batch-1 sequences carry no padding tokens: the reference pads the caption and image
  token runs to a multiple of 32 and masks the pads out of attention, which changes no
  valid token's output; only the caption's padded length enters the image tokens'
  rotary positions, and that is kept;
* the VAE decoder's convolutions go to cuDNN through torch (the reference uses cuDNN
  for the same convolutions, `crates/neuron/Cargo.toml:30-36`).

Checkpoint tensor names follow the diffusers layout (`transformer/`, `vae/`) so the
same safetensors load.
"""
from __future__ import annotations

import json
import math
import struct
import time
import zlib
from dataclasses import dataclass, field

import torch
import torch.nn.functional as F

# Scheduler shift interpolation and request bounds (harness/image.rs:34-53).
BASE_IMAGE_SEQ_LEN = 256
MAX_IMAGE_SEQ_LEN = 4096
BASE_SHIFT = 0.5
MAX_SHIFT = 1.15
DIM_ALIGN = 16
DEFAULT_STEPS = 9
MAX_STEPS = 50
DEFAULT_MAX_DIM = 2048
DEFAULT_GUIDANCE_SCALE = 5.0
SEQ_MULTIPLE = 32


@dataclass
class DiTConfig:
    in_channels: int = 16
    dim: int = 3840
    n_layers: int = 30
    n_refiner_layers: int = 2
    n_heads: int = 30
    norm_eps: float = 1e-5
    qk_norm: bool = True
    cap_feat_dim: int = 2560
    patch: int = 2
    f_patch: int = 1
    rope_theta: float = 256.0
    t_scale: float = 1000.0
    axes_dims: tuple = (32, 48, 48)
    axes_lens: tuple = (1024, 512, 512)
    adaln_dim: int = 256
    t_mid: int = 1024

    @property
    def head_dim(self) -> int:
        return self.dim // self.n_heads

    @property
    def ffn_dim(self) -> int:
        return int(self.dim / 3 * 8)

    @classmethod
    def from_json(cls, d: dict) -> "DiTConfig":
        ps = d.get("all_patch_size", [2])
        fps = d.get("all_f_patch_size", [1])
        return cls(in_channels=d.get("in_channels", 16), dim=d.get("dim", 3840), n_layers=d.get("n_layers", 30),
                   n_refiner_layers=d.get("n_refiner_layers", 2), n_heads=d.get("n_heads", 30),
                   norm_eps=d.get("norm_eps", 1e-5), qk_norm=d.get("qk_norm", True),
                   cap_feat_dim=d.get("cap_feat_dim", 2560), patch=ps[0], f_patch=fps[0],
                   rope_theta=float(d.get("rope_theta", 256.0)), t_scale=float(d.get("t_scale", 1000.0)),
                   axes_dims=tuple(d.get("axes_dims", (32, 48, 48))), axes_lens=tuple(d.get("axes_lens", (1024, 512, 512))),
                   adaln_dim=min(d.get("dim", 3840), 256), t_mid=d.get("t_embed_mid", 1024))

    def to_json(self) -> dict:
        """diffusers transformer/config.json keys of this configuration (plus
        `t_embed_mid`, this repository's key for a non-default timestep-MLP width)."""
        return {"in_channels": self.in_channels, "dim": self.dim, "n_layers": self.n_layers,
                "n_refiner_layers": self.n_refiner_layers, "n_heads": self.n_heads, "n_kv_heads": self.n_heads,
                "norm_eps": self.norm_eps, "qk_norm": self.qk_norm, "cap_feat_dim": self.cap_feat_dim,
                "all_patch_size": [self.patch], "all_f_patch_size": [self.f_patch], "rope_theta": self.rope_theta,
                "t_scale": self.t_scale, "axes_dims": list(self.axes_dims), "axes_lens": list(self.axes_lens),
                "t_embed_mid": self.t_mid}


@dataclass
class VaeConfig:
    latent_channels: int = 16
    out_channels: int = 3
    block_out_channels: tuple = (128, 256, 512, 512)
    layers_per_block: int = 2
    norm_groups: int = 32
    scaling_factor: float = 0.3611
    shift_factor: float = 0.1159
    mid_attention: bool = True

    @classmethod
    def from_json(cls, d: dict) -> "VaeConfig":
        return cls(latent_channels=d.get("latent_channels", 16), out_channels=d.get("out_channels", 3),
                   block_out_channels=tuple(d.get("block_out_channels", (128, 256, 512, 512))),
                   layers_per_block=d.get("layers_per_block", 2), norm_groups=d.get("norm_num_groups", 32),
                   scaling_factor=d.get("scaling_factor", 0.3611), shift_factor=d.get("shift_factor", 0.1159) or 0.0,
                   mid_attention=d.get("mid_block_add_attention", True))

    def to_json(self) -> dict:
        return {"latent_channels": self.latent_channels, "out_channels": self.out_channels,
                "block_out_channels": list(self.block_out_channels), "layers_per_block": self.layers_per_block,
                "norm_num_groups": self.norm_groups, "scaling_factor": self.scaling_factor,
                "shift_factor": self.shift_factor, "mid_block_add_attention": self.mid_attention}


def tiny_dit_config(cap_feat_dim: int = 256) -> DiTConfig:
    """Small DiT with the production structure (head dim 64, so the GPU kernels run it)."""
    return DiTConfig(dim=192, n_layers=2, n_refiner_layers=1, n_heads=3, cap_feat_dim=cap_feat_dim,
                     axes_dims=(16, 24, 24), axes_lens=(256, 64, 64), adaln_dim=192, t_mid=256)


def tiny_vae_config() -> VaeConfig:
    return VaeConfig(block_out_channels=(16, 16, 32, 32), layers_per_block=1, norm_groups=8)


# ----------------------------------------------------------------------------------
# request-side helpers (pure CPU)
# ----------------------------------------------------------------------------------
def validate_dims(width: int, height: int, max_dim: int = DEFAULT_MAX_DIM) -> tuple[int, int]:
    """(latent_h, latent_w) for a request; dims must be non-zero multiples of 16 (VAE 8x
    times patch 2) within the ceiling (harness/image.rs:109-124)."""
    if width <= 0 or height <= 0:
        raise ValueError(f"image dimensions must be non-zero, got {width}x{height}")
    if width % DIM_ALIGN or height % DIM_ALIGN:
        raise ValueError(f"image dimensions must be divisible by {DIM_ALIGN}, got {width}x{height}")
    if width > max_dim or height > max_dim:
        raise ValueError(f"image dimensions {width}x{height} exceed the configured ceiling {max_dim}x{max_dim}")
    return 2 * (height // DIM_ALIGN), 2 * (width // DIM_ALIGN)


def validate_steps(steps: int) -> int:
    if steps <= 0 or steps > MAX_STEPS:
        raise ValueError(f"num_steps must be in 1..={MAX_STEPS}, got {steps}")
    return steps


def format_prompt(prompt: str) -> str:
    """Qwen3 chat wrapping the text encoder was trained with (generation prompt on)."""
    return f"<|im_start|>user\n{prompt}<|im_end|>\n<|im_start|>assistant\n"


def megapixel_steps(width: int, height: int, steps: int, cfg: bool) -> float:
    """Metered image work: megapixels x denoise steps, doubled under guidance."""
    return width * height / 1e6 * steps * (2.0 if cfg else 1.0)


def parse_size(size: str | None) -> tuple[int, int]:
    """OpenAI `size` ("WIDTHxHEIGHT", default 1024x1024) -> (width, height)."""
    raw = size or "1024x1024"
    sep = "x" if "x" in raw else ("X" if "X" in raw else None)
    if sep is None:
        raise ValueError(f"size '{raw}' is not of the form WIDTHxHEIGHT")
    w, h = raw.split(sep, 1)
    try:
        width = int(w.strip())
    except ValueError:
        raise ValueError(f"size '{raw}': width is not a number") from None
    try:
        height = int(h.strip())
    except ValueError:
        raise ValueError(f"size '{raw}': height is not a number") from None
    return width, height


def parse_image_quant(quant: str) -> str:
    """The image path serves q8_0 (bf16 when no quant is given); anything else is an
    error rather than an untested precision."""
    if quant.lower() in ("q8_0", "q8"):
        return "Q8_0"
    raise ValueError(f"unsupported image quant '{quant}'; the image path serves q8_0 (bf16 when quant is omitted)")


def is_diffusers_layout(filenames) -> bool:
    return "model_index.json" in set(filenames)


def is_supported_pipeline_class(model_index_json: str) -> bool:
    try:
        return json.loads(model_index_json).get("_class_name") == "ZImagePipeline"
    except (ValueError, AttributeError):
        return False


def encode_png(rgb: bytes | torch.Tensor, width: int, height: int) -> bytes:
    """8-bit RGB rows -> PNG (one IDAT, filter 0 per scanline, zlib level 6)."""
    if isinstance(rgb, torch.Tensor):
        rgb = rgb.to(torch.uint8).contiguous().numpy().tobytes()
    if len(rgb) != width * height * 3:
        raise ValueError(f"rgb buffer is {len(rgb)} bytes, expected {width * height * 3}")
    stride = width * 3
    raw = b"".join(b"\x00" + rgb[y * stride:(y + 1) * stride] for y in range(height))

    def chunk(tag: bytes, data: bytes) -> bytes:
        return struct.pack(">I", len(data)) + tag + data + struct.pack(">I", zlib.crc32(tag + data) & 0xFFFFFFFF)

    ihdr = struct.pack(">IIBBBBB", width, height, 8, 2, 0, 0, 0)
    return b"\x89PNG\r\n\x1a\n" + chunk(b"IHDR", ihdr) + chunk(b"IDAT", zlib.compress(raw, 6)) + chunk(b"IEND", b"")


def decode_png(data: bytes) -> tuple[int, int, bytes]:
    """Inverse of encode_png for its own output (filter 0 rows); tests and tooling."""
    assert data[:8] == b"\x89PNG\r\n\x1a\n"
    pos, idat = 8, b""
    w = h = 0
    while pos < len(data):
        n = struct.unpack(">I", data[pos:pos + 4])[0]
        tag = data[pos + 4:pos + 8]
        body = data[pos + 8:pos + 8 + n]
        if tag == b"IHDR":
            w, h = struct.unpack(">II", body[:8])
        elif tag == b"IDAT":
            idat += body
        pos += 12 + n
    raw = zlib.decompress(idat)
    stride = w * 3
    rows = [raw[y * (stride + 1) + 1:(y + 1) * (stride + 1)] for y in range(h)]
    return w, h, b"".join(rows)


# ----------------------------------------------------------------------------------
# flow-matching Euler sampler
# ----------------------------------------------------------------------------------
def calculate_shift(image_seq_len: int, base_len: int = BASE_IMAGE_SEQ_LEN, max_len: int = MAX_IMAGE_SEQ_LEN,
                    base_shift: float = BASE_SHIFT, max_shift: float = MAX_SHIFT) -> float:
    """mu, linear in the image token count between (base_len, base_shift) and
    (max_len, max_shift)."""
    m = (max_shift - base_shift) / (max_len - base_len)
    return image_seq_len * m + (base_shift - m * base_len)


class FlowMatchEuler:
    """Euler steps of the rectified-flow ODE on a time-shifted sigma grid: sigmas run
    from 1 to 0 in `steps` evenly spaced values, each mapped by
    s -> e^mu / (e^mu + 1/s - 1) (resolution-dependent shift), then a terminal 0. A step
    moves x by (sigma_next - sigma) * velocity; the model is conditioned on
    t = 1 - sigma."""

    def __init__(self, steps: int, mu: float):
        base = torch.linspace(1.0, 0.0, steps, dtype=torch.float64)
        em = math.exp(mu)
        shifted = [0.0 if s <= 0 else em / (em + (1.0 / s - 1.0)) for s in base.tolist()]
        self.sigmas = shifted + [0.0]
        self.i = 0

    def __len__(self):
        return len(self.sigmas) - 1

    @property
    def sigma(self) -> float:
        return self.sigmas[self.i]

    def t_normalized(self) -> float:
        return 1.0 - self.sigmas[self.i]

    def step(self, velocity: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
        dt = self.sigmas[self.i + 1] - self.sigmas[self.i]
        self.i += 1
        return (x.float() + dt * velocity.float()).to(x.dtype)


# ----------------------------------------------------------------------------------
# rotary tables, patchify
# ----------------------------------------------------------------------------------
def rope_angles(pos: torch.Tensor, cfg: DiTConfig) -> torch.Tensor:
    """pos int [T, 3] -> f32 angles [T, head_dim/2]: per axis i, pos_i * theta^(-2j/d_i)."""
    parts = []
    for ax, d in enumerate(cfg.axes_dims):
        inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.float64) / d))
        parts.append(pos[:, ax:ax + 1].double() * inv[None, :].to(pos.device))
    return torch.cat(parts, -1).float()


def patchify(lat: torch.Tensor, p: int) -> tuple[torch.Tensor, tuple]:
    """lat [C, H, W] -> tokens [(H/p)(W/p), p*p*C] (row-major over the token grid; each
    token's features ordered (py, px, c)), and the grid."""
    C, H, W = lat.shape
    ht, wt = H // p, W // p
    x = lat.view(C, ht, p, wt, p).permute(1, 3, 2, 4, 0).reshape(ht * wt, p * p * C)
    return x, (ht, wt)


def unpatchify(x: torch.Tensor, grid: tuple, p: int, C: int) -> torch.Tensor:
    ht, wt = grid
    return x.view(ht, wt, p, p, C).permute(4, 0, 2, 1, 3).reshape(C, ht * p, wt * p)


def positions(cap_len: int, grid: tuple, device) -> tuple[torch.Tensor, torch.Tensor]:
    """3-axis positions: caption tokens (1 + i, 0, 0); image tokens
    (padded caption length + 1, row, col)."""
    pad = (cap_len + SEQ_MULTIPLE - 1) // SEQ_MULTIPLE * SEQ_MULTIPLE
    cap = torch.zeros(cap_len, 3, dtype=torch.int64, device=device)
    cap[:, 0] = torch.arange(1, cap_len + 1, device=device)
    ht, wt = grid
    img = torch.zeros(ht * wt, 3, dtype=torch.int64, device=device)
    img[:, 0] = pad + 1
    img[:, 1] = torch.arange(ht, device=device).repeat_interleave(wt)
    img[:, 2] = torch.arange(wt, device=device).repeat(ht)
    return img, cap


def timestep_embedding(t: torch.Tensor, dim: int = 256, max_period: float = 10000.0) -> torch.Tensor:
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    args = t.float()[:, None] * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], -1)


# ----------------------------------------------------------------------------------
# weights
# ----------------------------------------------------------------------------------
def dit_weight_shapes(cfg: DiTConfig) -> dict[str, tuple]:
    D, Fh, Dh, A = cfg.dim, cfg.ffn_dim, cfg.head_dim, cfg.adaln_dim
    pin = cfg.f_patch * cfg.patch * cfg.patch * cfg.in_channels
    key = f"{cfg.patch}-{cfg.f_patch}"
    s = {
        f"all_x_embedder.{key}.weight": (D, pin), f"all_x_embedder.{key}.bias": (D,),
        f"all_final_layer.{key}.linear.weight": (pin, D), f"all_final_layer.{key}.linear.bias": (pin,),
        f"all_final_layer.{key}.adaLN_modulation.1.weight": (D, A),
        f"all_final_layer.{key}.adaLN_modulation.1.bias": (D,),
        "t_embedder.mlp.0.weight": (cfg.t_mid, 256), "t_embedder.mlp.0.bias": (cfg.t_mid,),
        "t_embedder.mlp.2.weight": (A, cfg.t_mid), "t_embedder.mlp.2.bias": (A,),
        "cap_embedder.0.weight": (cfg.cap_feat_dim,),
        "cap_embedder.1.weight": (D, cfg.cap_feat_dim), "cap_embedder.1.bias": (D,),
        "x_pad_token": (1, D), "cap_pad_token": (1, D),
    }

    def block(pre: str, modulation: bool):
        s.update({pre + "attention.to_q.weight": (D, D), pre + "attention.to_k.weight": (D, D),
                  pre + "attention.to_v.weight": (D, D), pre + "attention.to_out.0.weight": (D, D),
                  pre + "feed_forward.w1.weight": (Fh, D), pre + "feed_forward.w3.weight": (Fh, D),
                  pre + "feed_forward.w2.weight": (D, Fh),
                  pre + "attention_norm1.weight": (D,), pre + "attention_norm2.weight": (D,),
                  pre + "ffn_norm1.weight": (D,), pre + "ffn_norm2.weight": (D,)})
        if cfg.qk_norm:
            s.update({pre + "attention.norm_q.weight": (Dh,), pre + "attention.norm_k.weight": (Dh,)})
        if modulation:
            s.update({pre + "adaLN_modulation.0.weight": (4 * D, A), pre + "adaLN_modulation.0.bias": (4 * D,)})

    for i in range(cfg.n_refiner_layers):
        block(f"noise_refiner.{i}.", True)
        block(f"context_refiner.{i}.", False)
    for i in range(cfg.n_layers):
        block(f"layers.{i}.", True)
    return s


def vae_decoder_shapes(cfg: VaeConfig) -> dict[str, tuple]:
    ch = list(reversed(cfg.block_out_channels))
    s = {}

    def resnet(pre, cin, cout):
        s.update({pre + "norm1.weight": (cin,), pre + "norm1.bias": (cin,), pre + "conv1.weight": (cout, cin, 3, 3),
                  pre + "conv1.bias": (cout,), pre + "norm2.weight": (cout,), pre + "norm2.bias": (cout,),
                  pre + "conv2.weight": (cout, cout, 3, 3), pre + "conv2.bias": (cout,)})
        if cin != cout:
            s.update({pre + "conv_shortcut.weight": (cout, cin, 1, 1), pre + "conv_shortcut.bias": (cout,)})

    c0 = ch[0]
    s.update({"decoder.conv_in.weight": (c0, cfg.latent_channels, 3, 3), "decoder.conv_in.bias": (c0,)})
    resnet("decoder.mid_block.resnets.0.", c0, c0)
    resnet("decoder.mid_block.resnets.1.", c0, c0)
    if cfg.mid_attention:
        a = "decoder.mid_block.attentions.0."
        s.update({a + "group_norm.weight": (c0,), a + "group_norm.bias": (c0,)})
        for n in ("to_q", "to_k", "to_v", "to_out.0"):
            s.update({a + n + ".weight": (c0, c0), a + n + ".bias": (c0,)})
    cin = c0
    for bi, cout in enumerate(ch):
        for j in range(cfg.layers_per_block + 1):
            resnet(f"decoder.up_blocks.{bi}.resnets.{j}.", cin if j == 0 else cout, cout)
        cin = cout
        if bi < len(ch) - 1:
            s.update({f"decoder.up_blocks.{bi}.upsamplers.0.conv.weight": (cout, cout, 3, 3),
                      f"decoder.up_blocks.{bi}.upsamplers.0.conv.bias": (cout,)})
    s.update({"decoder.conv_norm_out.weight": (ch[-1],), "decoder.conv_norm_out.bias": (ch[-1],),
              "decoder.conv_out.weight": (cfg.out_channels, ch[-1], 3, 3), "decoder.conv_out.bias": (cfg.out_channels,)})
    return s


def random_weights(shapes: dict, seed: int = 0, std: float = 0.02, device="cpu",
                   dtype=torch.float32) -> dict[str, torch.Tensor]:
    """N(0, std) weights; norm scales start at 1 (GroupNorm / RMSNorm weights)."""
    g = torch.Generator(device=device).manual_seed(seed)
    out = {}
    for name, shp in sorted(shapes.items()):
        t = torch.empty(shp, dtype=dtype, device=device)
        if "norm" in name and name.endswith("weight") and len(shp) == 1:
            t.fill_(1.0)
        elif "norm" in name and name.endswith("bias"):
            t.zero_()
        else:
            t.normal_(0.0, std, generator=g)
        out[name] = t
    return out


# ----------------------------------------------------------------------------------
# the transformer
# ----------------------------------------------------------------------------------
def _rms(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps) * w.float()).to(x.dtype)


def _rope_torch(x: torch.Tensor, ang: torch.Tensor) -> torch.Tensor:
    """x [T, H, Dh], rotation of interleaved pairs by ang [T, Dh/2]."""
    xf = x.float().view(*x.shape[:-1], -1, 2)
    c, s = torch.cos(ang)[:, None], torch.sin(ang)[:, None]
    a, b = xf[..., 0], xf[..., 1]
    return torch.stack([a * c - b * s, a * s + b * c], -1).flatten(-2).to(x.dtype)


class ZImageDiT:
    """Z-Image single-stream DiT. device cpu: plain torch in `dtype` (the oracle);
    device cuda: bf16 on this repository's kernels."""

    def __init__(self, cfg: DiTConfig, weights: dict[str, torch.Tensor], device="cpu",
                 dtype: torch.dtype = torch.float32):
        self.cfg = cfg
        self.device = torch.device(device)
        self.cuda = self.device.type == "cuda"
        self.dtype = torch.bfloat16 if self.cuda else dtype
        self.key = f"{cfg.patch}-{cfg.f_patch}"
        small = ("bias", "norm", "adaLN", "t_embedder", "pad_token")
        self.w = {}
        for k, v in weights.items():
            keep_f32 = any(s in k for s in small) or v.dim() == 1
            self.w[k] = v.to(self.device, torch.float32 if (keep_f32 and self.cuda) else self.dtype).contiguous()
        if self.cuda:
            from .. import ops
            self.C = ops.C
            self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
            self._fuse()

    def _fuse(self):
        """GPU layouts: q|k|v rows stacked into one projection; FFN gate / up rows
        interleaved (g0, u0, g1, u1, ...) for the GEMM's SwiGLU epilogue."""
        pres = [f"noise_refiner.{i}." for i in range(self.cfg.n_refiner_layers)]
        pres += [f"context_refiner.{i}." for i in range(self.cfg.n_refiner_layers)]
        pres += [f"layers.{i}." for i in range(self.cfg.n_layers)]
        for p in pres:
            w = self.w
            w[p + "qkv"] = torch.cat([w.pop(p + "attention.to_q.weight"), w.pop(p + "attention.to_k.weight"),
                                      w.pop(p + "attention.to_v.weight")], 0).contiguous()
            g, u = w.pop(p + "feed_forward.w1.weight"), w.pop(p + "feed_forward.w3.weight")
            w[p + "gu"] = torch.stack([g, u], 1).reshape(-1, g.shape[1]).contiguous()

    # ---- shared small math (f32, M = 1) ----
    def _adaln_input(self, t_norm: float) -> torch.Tensor:
        w = self.w
        t = torch.tensor([t_norm * self.cfg.t_scale], device=self.device)
        e = timestep_embedding(t, 256)
        h = F.silu(e @ w["t_embedder.mlp.0.weight"].float().t() + w["t_embedder.mlp.0.bias"].float())
        return (h @ w["t_embedder.mlp.2.weight"].float().t() + w["t_embedder.mlp.2.bias"].float())[0]

    def _mods(self, pre: str, c: torch.Tensor):
        m = c @ self.w[pre + "adaLN_modulation.0.weight"].float().t() + self.w[pre + "adaLN_modulation.0.bias"].float()
        sm, gm, sf, gf = m.chunk(4)
        return sm, torch.tanh(gm), sf, torch.tanh(gf)

    # ---- one block ----
    def _block(self, pre: str, x: torch.Tensor, ang: torch.Tensor, c: torch.Tensor | None) -> torch.Tensor:
        return self._block_cuda(pre, x, ang, c) if self.cuda else self._block_torch(pre, x, ang, c)

    def _block_torch(self, pre, x, ang, c):
        cfg, w = self.cfg, self.w
        eps, H, Dh = cfg.norm_eps, cfg.n_heads, cfg.head_dim
        T = x.shape[0]
        if c is not None:
            sm, gm, sf, gf = self._mods(pre, c)
        h = _rms(x, w[pre + "attention_norm1.weight"], eps)
        if c is not None:
            h = (h.float() * (1 + sm)).to(x.dtype)
        q = (h @ w[pre + "attention.to_q.weight"].t()).view(T, H, Dh)
        k = (h @ w[pre + "attention.to_k.weight"].t()).view(T, H, Dh)
        v = (h @ w[pre + "attention.to_v.weight"].t()).view(T, H, Dh)
        if cfg.qk_norm:
            q = _rms(q, w[pre + "attention.norm_q.weight"], eps)
            k = _rms(k, w[pre + "attention.norm_k.weight"], eps)
        q, k = _rope_torch(q, ang), _rope_torch(k, ang)
        o = F.scaled_dot_product_attention(q.transpose(0, 1).float(), k.transpose(0, 1).float(),
                                           v.transpose(0, 1).float()).transpose(0, 1).reshape(T, H * Dh).to(x.dtype)
        o = o @ w[pre + "attention.to_out.0.weight"].t()
        o = _rms(o, w[pre + "attention_norm2.weight"], eps)
        x = x + ((o.float() * gm).to(x.dtype) if c is not None else o)
        h = _rms(x, w[pre + "ffn_norm1.weight"], eps)
        if c is not None:
            h = (h.float() * (1 + sf)).to(x.dtype)
        f = F.silu(h @ w[pre + "feed_forward.w1.weight"].t()) * (h @ w[pre + "feed_forward.w3.weight"].t())
        f = f @ w[pre + "feed_forward.w2.weight"].t()
        f = _rms(f, w[pre + "ffn_norm2.weight"], eps)
        return x + ((f.float() * gf).to(x.dtype) if c is not None else f)

    def quantize_(self, scheme: str = "q8_0") -> None:
        """In-situ q8_0 quantization of the transformer blocks' projections (the
        reference's image-path ISQ, harness/image.rs:528-539 accepts q8_0 only): the
        weights live as Q8_0 block rows (about half the bytes of bf16) and each GEMM
        dequantizes its weight to bf16 scratch first."""
        if parse_image_quant(scheme) != "Q8_0":
            raise ValueError(scheme)
        if not self.cuda:
            raise RuntimeError("quantized DiT serving needs the CUDA extension")
        from .fast import GGUF_Q8_0, QWeight
        for k in list(self.w):
            if k.endswith(("qkv", "gu", "attention.to_out.0.weight", "feed_forward.w2.weight")):
                w = self.w[k]
                self.w[k] = QWeight(self.C.gguf_quant(w, GGUF_Q8_0), GGUF_Q8_0, w.shape[1])
                del w
        self.quant = "q8_0"

    def _gemm(self, x: torch.Tensor, W, epi: int = 0) -> torch.Tensor:
        if not isinstance(W, torch.Tensor):
            W = W.dequant(self.C)
        N = W.shape[0] // 2 if epi == 1 else W.shape[0]
        y = torch.empty(x.shape[0], N, dtype=torch.bfloat16, device=self.device)
        self.C.gemm(x, W, y, epi, self.err)
        return y

    def _block_cuda(self, pre, x, ang, c):
        cfg, w, C = self.cfg, self.w, self.C
        eps, H, Dh = cfg.norm_eps, cfg.n_heads, cfg.head_dim
        T, D = x.shape
        mods = self._mods(pre, c) if c is not None else (None, None, None, None)
        sm, gm, sf, gf = (m.contiguous() if m is not None else None for m in mods)
        h = torch.empty_like(x)
        C.dit_norm_mod(x, w[pre + "attention_norm1.weight"], sm, h, eps)
        qkv = self._gemm(h, w[pre + "qkv"])
        q = torch.empty(T, H * Dh, dtype=torch.bfloat16, device=self.device)
        k = torch.empty(H, T, Dh, dtype=torch.bfloat16, device=self.device)
        v = torch.empty_like(k)
        C.dit_qk_rope(qkv, w.get(pre + "attention.norm_q.weight"), w.get(pre + "attention.norm_k.weight"), ang,
                      H, Dh, eps, q, k, v)
        o = torch.empty(T, H * Dh, dtype=torch.bfloat16, device=self.device)
        C.attn_prefill_tc(q, k, v, o, H, 0, Dh ** -0.5, None, 0, self.err, causal=False)
        o = self._gemm(o, w[pre + "attention.to_out.0.weight"])
        C.dit_gate_res(x, o, w[pre + "attention_norm2.weight"], gm, eps)
        C.dit_norm_mod(x, w[pre + "ffn_norm1.weight"], sf, h, eps)
        f = self._gemm(h, w[pre + "gu"], epi=1)
        f = self._gemm(f, w[pre + "feed_forward.w2.weight"])
        C.dit_gate_res(x, f, w[pre + "ffn_norm2.weight"], gf, eps)
        return x

    # ---- forward ----
    @torch.no_grad()
    def forward(self, latent: torch.Tensor, t_norm: float, cap_feats: torch.Tensor) -> torch.Tensor:
        """latent [C, H, W], t_norm = 1 - sigma, cap_feats [Lc, cap_feat_dim] ->
        the model output [C, H, W] (the negated flow velocity)."""
        cfg, w, dt = self.cfg, self.w, self.dtype
        p = cfg.patch
        c = self._adaln_input(t_norm)
        img, grid = patchify(latent.to(self.device, dt), p)
        Ti, Lc = img.shape[0], cap_feats.shape[0]
        pos_img, pos_cap = positions(Lc, grid, self.device)
        ang_img, ang_cap = rope_angles(pos_img, cfg), rope_angles(pos_cap, cfg)
        x = (img.float() @ w[f"all_x_embedder.{self.key}.weight"].float().t()
             + w[f"all_x_embedder.{self.key}.bias"].float()).to(dt).contiguous()
        for i in range(cfg.n_refiner_layers):
            x = self._block(f"noise_refiner.{i}.", x, ang_img, c)
        cap = _rms(cap_feats.to(self.device, torch.float32), w["cap_embedder.0.weight"].float(), cfg.norm_eps)
        cap = (cap @ w["cap_embedder.1.weight"].float().t() + w["cap_embedder.1.bias"].float()).to(dt).contiguous()
        for i in range(cfg.n_refiner_layers):
            cap = self._block(f"context_refiner.{i}.", cap, ang_cap, None)
        u = torch.cat([x, cap], 0).contiguous()
        ang = torch.cat([ang_img, ang_cap], 0).contiguous()
        for i in range(cfg.n_layers):
            u = self._block(f"layers.{i}.", u, ang, c)
        # final layer: LayerNorm (no affine, eps 1e-6) * (1 + scale(SiLU(c))), linear
        fl = f"all_final_layer.{self.key}."
        scale = 1.0 + (F.silu(c) @ w[fl + "adaLN_modulation.1.weight"].float().t() + w[fl + "adaLN_modulation.1.bias"].float())
        y = F.layer_norm(u[:Ti].float(), (cfg.dim,), eps=1e-6) * scale
        y = y @ w[fl + "linear.weight"].float().t() + w[fl + "linear.bias"].float()
        return unpatchify(y, grid, p, cfg.in_channels)


# ----------------------------------------------------------------------------------
# VAE decoder
# ----------------------------------------------------------------------------------
class VaeDecoder:
    """AutoencoderKL decoder (16 latent channels, 8x upsampling): conv_in, mid block
    (resnet, single-head attention, resnet), up blocks of (layers_per_block + 1) resnets
    with nearest-2x + conv upsampling, GroupNorm + SiLU + conv_out."""

    def __init__(self, cfg: VaeConfig, weights: dict[str, torch.Tensor], device="cpu", dtype=torch.float32):
        self.cfg = cfg
        self.device = torch.device(device)
        self.dtype = dtype
        self.w = {k: v.to(self.device, dtype) for k, v in weights.items() if k.startswith("decoder.")}

    def _gn(self, x, pre):
        return F.group_norm(x, self.cfg.norm_groups, self.w[pre + ".weight"], self.w[pre + ".bias"], eps=1e-6)

    def _conv(self, x, pre, pad=1):
        return F.conv2d(x, self.w[pre + ".weight"], self.w[pre + ".bias"], padding=pad)

    def _resnet(self, x, pre):
        h = self._conv(F.silu(self._gn(x, pre + "norm1")), pre + "conv1")
        h = self._conv(F.silu(self._gn(h, pre + "norm2")), pre + "conv2")
        if pre + "conv_shortcut.weight" in self.w:
            x = self._conv(x, pre + "conv_shortcut", pad=0)
        return x + h

    def _attn(self, x, pre):
        B, C, H, W = x.shape
        h = self._gn(x, pre + "group_norm").view(B, C, H * W).transpose(1, 2)
        q = F.linear(h, self.w[pre + "to_q.weight"], self.w[pre + "to_q.bias"])
        k = F.linear(h, self.w[pre + "to_k.weight"], self.w[pre + "to_k.bias"])
        v = F.linear(h, self.w[pre + "to_v.weight"], self.w[pre + "to_v.bias"])
        o = F.scaled_dot_product_attention(q[:, None], k[:, None], v[:, None])[:, 0]
        o = F.linear(o, self.w[pre + "to_out.0.weight"], self.w[pre + "to_out.0.bias"])
        return x + o.transpose(1, 2).view(B, C, H, W)

    @torch.no_grad()
    def decode(self, z: torch.Tensor) -> torch.Tensor:
        """z [B, C, h, w] (DiT latents) -> image [B, 3, 8h, 8w] in [-1, 1] (unclamped)."""
        cfg = self.cfg
        x = (z.to(self.device, self.dtype) / cfg.scaling_factor) + cfg.shift_factor
        x = self._conv(x, "decoder.conv_in")
        x = self._resnet(x, "decoder.mid_block.resnets.0.")
        if cfg.mid_attention:
            x = self._attn(x, "decoder.mid_block.attentions.0.")
        x = self._resnet(x, "decoder.mid_block.resnets.1.")
        nblk = len(cfg.block_out_channels)
        for bi in range(nblk):
            for j in range(cfg.layers_per_block + 1):
                x = self._resnet(x, f"decoder.up_blocks.{bi}.resnets.{j}.")
            if bi < nblk - 1:
                x = F.interpolate(x, scale_factor=2.0, mode="nearest")
                x = self._conv(x, f"decoder.up_blocks.{bi}.upsamplers.0.conv")
        x = F.silu(self._gn(x, "decoder.conv_norm_out"))
        return self._conv(x, "decoder.conv_out")

    @property
    def factor(self) -> int:
        return 2 ** (len(self.cfg.block_out_channels) - 1)


def tile_positions(extent: int, tile: int, overlap: int) -> list[int]:
    """Tile origins at stride tile - overlap; the last tile is pulled flush with the edge."""
    if extent <= tile:
        return [0]
    out, pos = [], 0
    while True:
        if pos + tile >= extent:
            out.append(extent - tile)
            return out
        out.append(pos)
        pos += tile - overlap


def _ramp(n: int, ov: int, lead: bool, trail: bool) -> torch.Tensor:
    i = torch.arange(n, dtype=torch.float32)
    w = torch.ones(n)
    if lead:
        w = torch.minimum(w, torch.where(i < ov, (i + 1) / (ov + 1), torch.ones(n)))
    if trail:
        w = torch.minimum(w, torch.where(i >= n - ov, (n - i) / (ov + 1), torch.ones(n)))
    return w


def tiled_decode(vae: VaeDecoder, z: torch.Tensor, tile: int = 64, overlap: int = 16) -> torch.Tensor:
    """Decode overlapping latent tiles and blend the seams with linear ramps over the
    overlap (weights normalised per pixel), so transient memory is bounded by one tile
    (harness/image.rs:159-262 in the reference; same placement and blend rule)."""
    _, _, lh, lw = z.shape
    if lh <= tile and lw <= tile:
        return vae.decode(z).float()
    px = vae.factor
    rows, cols = tile_positions(lh, tile, overlap), tile_positions(lw, tile, overlap)
    acc = wsum = None
    for ri, r in enumerate(rows):
        for ci, c in enumerate(cols):
            t = vae.decode(z[:, :, r:r + min(tile, lh), c:c + min(tile, lw)]).float()
            _, ch, th, tw = t.shape
            if acc is None:
                acc = torch.zeros(1, ch, lh * px, lw * px, device=t.device)
                wsum = torch.zeros(1, 1, lh * px, lw * px, device=t.device)
            wy = _ramp(th, overlap * px, ri > 0, ri + 1 < len(rows)).to(t.device)
            wx = _ramp(tw, overlap * px, ci > 0, ci + 1 < len(cols)).to(t.device)
            w2 = wy[:, None] * wx[None, :]
            y0, x0 = r * px, c * px
            acc[:, :, y0:y0 + th, x0:x0 + tw] += t * w2
            wsum[:, :, y0:y0 + th, x0:x0 + tw] += w2
    return acc / wsum


def postprocess(img: torch.Tensor) -> torch.Tensor:
    """[-1, 1] float [3, H, W] -> uint8 [H, W, 3]."""
    return ((img.float() / 2 + 0.5).clamp(0, 1) * 255).round().to(torch.uint8).permute(1, 2, 0).contiguous()


# ----------------------------------------------------------------------------------
# pipeline
# ----------------------------------------------------------------------------------
@dataclass
class ImageTiming:
    encode_ms: float = 0.0
    denoise_ms: float = 0.0
    decode_ms: float = 0.0
    steps: int = 0
    cfg: bool = False


@dataclass
class ImageResult:
    rgb: torch.Tensor                     # uint8 [H, W, 3] on the CPU
    width: int
    height: int
    timing: ImageTiming = field(default_factory=ImageTiming)


class TextEncoder:
    """Caption features: the hidden states of a Qwen3 model after all but its last layer
    (no final norm), one row per prompt token."""

    def __init__(self, model):
        self.m = model

    @torch.no_grad()
    def encode(self, tokens: list[int]) -> torch.Tensor:
        m = self.m
        return m.hidden(torch.tensor(tokens, dtype=torch.long), m.cfg.num_hidden_layers - 1)


class ZImagePipeline:
    def __init__(self, dit: ZImageDiT, vae: VaeDecoder, text_encoder: TextEncoder, tokenizer=None,
                 max_dim: int = DEFAULT_MAX_DIM, tile: int = 64, overlap: int = 16):
        self.dit, self.vae, self.te, self.tok = dit, vae, text_encoder, tokenizer
        self.max_dim, self.tile, self.overlap = max_dim, tile, overlap

    def _sync(self):
        if self.dit.cuda:
            torch.cuda.synchronize(self.dit.device)

    def encode_prompt(self, prompt: str | list[int]) -> list[int]:
        if isinstance(prompt, list):
            return prompt
        if self.tok is None:
            raise ValueError("no tokenizer: pass prompt token ids")
        return self.tok.encode(format_prompt(prompt))

    @torch.no_grad()
    def generate(self, prompt, width: int = 1024, height: int = 1024, steps: int = DEFAULT_STEPS,
                 negative_prompt=None, guidance_scale: float = DEFAULT_GUIDANCE_SCALE,
                 seed: int | None = None) -> ImageResult:
        lh, lw = validate_dims(width, height, self.max_dim)
        steps = validate_steps(steps)
        toks = self.encode_prompt(prompt)
        if not toks:
            raise ValueError("prompt tokens must be non-empty")
        timing = ImageTiming(steps=steps)
        t0 = time.perf_counter()
        cap = self.te.encode(toks)
        use_cfg = negative_prompt is not None and guidance_scale > 1.0
        neg = self.te.encode(self.encode_prompt(negative_prompt)) if use_cfg else None
        timing.cfg = use_cfg
        timing.encode_ms = (time.perf_counter() - t0) * 1e3
        t0 = time.perf_counter()
        g = torch.Generator().manual_seed(seed if seed is not None else int(time.time_ns() % (2**63)))
        C = self.dit.cfg.in_channels
        lat = torch.randn(C, lh, lw, generator=g, dtype=torch.float32).to(self.dit.device, self.dit.dtype)
        sched = FlowMatchEuler(steps, calculate_shift((lh // 2) * (lw // 2)))
        for _ in range(len(sched)):
            if sched.sigmas[sched.i + 1] == sched.sigma:  # terminal zero step: no model call
                sched.i += 1
                continue
            t = sched.t_normalized()
            pred = self.dit.forward(lat, t, cap).float()
            if neg is not None:
                npred = self.dit.forward(lat, t, neg).float()
                pred = npred + guidance_scale * (pred - npred)
            lat = sched.step(-pred, lat)  # the model predicts the negated velocity
        self._sync()
        timing.denoise_ms = (time.perf_counter() - t0) * 1e3
        t0 = time.perf_counter()
        img = tiled_decode(self.vae, lat[None].to(self.vae.device, self.vae.dtype), self.tile, self.overlap)[0]
        rgb = postprocess(img).cpu()
        timing.decode_ms = (time.perf_counter() - t0) * 1e3
        if rgb.shape[0] != height or rgb.shape[1] != width:
            raise RuntimeError(f"decoded image is {rgb.shape[1]}x{rgb.shape[0]}, expected {width}x{height}")
        return ImageResult(rgb=rgb, width=width, height=height, timing=timing)
