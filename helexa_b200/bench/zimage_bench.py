"""Z-Image-Turbo text-to-image timing on one GPU: the full 6B DiT architecture
(random-init bf16 weights), caption features of a typical prompt length, the default
9-step schedule (8 DiT forwards: the last step has sigma 0) and the VAE decode at
the requested resolution. Device-timed with CUDA events after warm-up.

The reference publishes ~11 s end to end at 1024x1024 (9 steps, bf16, RTX 4090) and a
2.8 s q8_0 denoise on an RTX 5090 (README.md:126-128, CLAUDE.md:1037-1038).

  python -m helexa_b200.bench.zimage_bench --size 1024 --steps 9
"""
from __future__ import annotations

import argparse
import json

import torch

from ..models import zimage as zi


def dit_flops(cfg: zi.DiTConfig, n_img: int, n_cap: int) -> float:
    """Matmul FLOPs of one DiT forward (projections + attention score/value products)."""
    D, Fh = cfg.dim, cfg.ffn_dim
    per_tok = 2 * (4 * D * D + 3 * D * Fh)

    def blocks(n, T):
        return n * (T * per_tok + 4 * T * T * D)

    return (blocks(cfg.n_refiner_layers, n_img) + blocks(cfg.n_refiner_layers, n_cap)
            + blocks(cfg.n_layers, n_img + n_cap))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=zi.DEFAULT_STEPS)
    ap.add_argument("--cap", type=int, default=128, help="caption tokens")
    ap.add_argument("--warmup", type=int, default=1)
    ap.add_argument("--reps", type=int, default=2)
    ap.add_argument("--layers", type=int, default=0, help="truncate the DiT (profiling only)")
    ap.add_argument("--quant", default=None, help="q8_0: in-situ quantized DiT projections")
    args = ap.parse_args()
    dev = torch.device("cuda", 0)
    cfg = zi.DiTConfig()
    if args.layers:
        cfg.n_layers = args.layers
    w = zi.random_weights(zi.dit_weight_shapes(cfg), seed=0, device=dev, dtype=torch.bfloat16)
    dit = zi.ZImageDiT(cfg, w, dev)
    del w
    if args.quant:
        dit.quantize_(args.quant)
    vcfg = zi.VaeConfig()
    vae = zi.VaeDecoder(vcfg, zi.random_weights(zi.vae_decoder_shapes(vcfg), seed=1, device=dev), dev, torch.bfloat16)
    lh, lw = zi.validate_dims(args.size, args.size)
    g = torch.Generator(device=dev).manual_seed(0)
    cap = torch.randn(args.cap, cfg.cap_feat_dim, device=dev, generator=g).bfloat16()
    n_img = (lh // 2) * (lw // 2)

    def run():
        lat = torch.randn(cfg.in_channels, lh, lw, device=dev, generator=g).bfloat16()
        sched = zi.FlowMatchEuler(args.steps, zi.calculate_shift(n_img))
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
        ev[0].record()
        calls = 0
        for _ in range(len(sched)):
            if sched.sigmas[sched.i + 1] == sched.sigma:
                sched.i += 1
                continue
            pred = dit.forward(lat, sched.t_normalized(), cap)
            lat = sched.step(-pred.float(), lat)
            calls += 1
        ev[1].record()
        img = zi.tiled_decode(vae, lat[None], 64, 16)
        zi.postprocess(img[0])
        ev[2].record()
        ev[2].synchronize()
        return ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), calls

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    res = [run() for _ in range(args.reps)]
    den = min(r[0] for r in res)
    dec = min(r[1] for r in res)
    calls = res[0][2]
    fl = dit_flops(cfg, n_img, args.cap) * calls
    assert dit.err.item() == 0, "device error word set"
    print(json.dumps({"model": "Z-Image-Turbo (6B DiT, random-init bf16)", "quant": args.quant, "size": args.size, "steps": args.steps,
                      "dit_forwards": calls, "caption_tokens": args.cap, "image_tokens": n_img,
                      "denoise_ms": round(den, 1), "ms_per_dit_forward": round(den / max(calls, 1), 2),
                      "vae_decode_ms": round(dec, 1), "total_ms": round(den + dec, 1),
                      "dit_tflops": round(fl / (den / 1e3) / 1e12, 1)}))


if __name__ == "__main__":
    main()
