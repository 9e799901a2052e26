"""Decode-step driver for kernel profiling and per-step timing.

Builds a random-init model (optionally truncated to --layers to keep an ncu capture
small), places the sequence at --context tokens (the KV / GDN state contents do not
change the work a decode step does, so no prefill is run), then times --steps
decode steps with CUDA events, eagerly or as one replayed CUDA graph.

  python -m helexa_b200.bench.profile_decode --model qwen3-next-80b-a3b --layers 8 \
      --context 8192 --steps 20 [--eager]
"""
from __future__ import annotations

import argparse
import dataclasses
import json

import torch

from .. import ops
from ..config import get_preset
from ..models.fast import FastModel


class SkippingModel(FastModel):
    """FastModel whose decode layer leaves named components out (single rank), so a
    replayed step measures their share of the step time. Profiling only."""

    skip: frozenset = frozenset()

    def _decode_layer(self, i, nb):
        C, cfg, d, lw, skip = self.C, self.cfg, self.dims, self.layers[i], self.skip
        eps = cfg.rms_norm_eps
        if not skip:
            return super()._decode_layer(i, nb)
        if cfg.is_linear(i) and "gdn" in skip or not cfg.is_linear(i) and "attn" in skip:
            pass
        elif cfg.is_linear(i):
            self._gemv(lw["w_in"], nb.x, nb.proj_gdn, ops.STORE_BF16, None, lw["ln1"], eps)
            if "gdn_core" not in skip:
                C.gdn_decode(nb.proj_gdn, lw["conv_w"], self.conv[i], self.rec[i], lw["A_log"], lw["dt_bias"],
                             lw["gnorm"], nb.slots, self.pos, nb.gdn_out, d.hk, d.hv, d.dk, d.dv, eps)
            self._row_parallel(lw["out_w"], nb.gdn_out, nb)
        else:
            self._gemv(lw["w_qkv"], nb.x, nb.proj_attn, ops.STORE_BF16, None, lw["ln1"], eps)
            if "attn_core" not in skip:
                C.attn_decode(nb.proj_attn, lw.get("q_norm"), lw.get("k_norm"), self.inv_freq, self.kc[i],
                              self.vc[i], nb.slots, self.pos, nb.part_o, nb.part_ml, nb.counters, nb.attn_out,
                              d.hq, d.hkv, d.D, cfg.rotary_dim, cfg.attn_output_gate, eps)
            self._row_parallel(lw["o_w"], nb.attn_out, nb)
        if "ffn" not in skip and cfg.layer_uses_moe(i):
            E, k = cfg.num_experts, cfg.num_experts_per_tok
            J = k + (1 if self.has_shared else 0)
            C.gemv_router(lw["router"], nb.x, nb.rlogits, lw["ln2"], eps, E, k, self.has_shared,
                          cfg.norm_topk_prob, nb.ids, nb.wts, nb.counter)
            if "experts" not in skip:
                C.gemv_experts(lw["w_gu"], nb.x, nb.ids.view(-1), nb.act_moe, ops.SILU_PAIR, J, lw["ln2"], eps)
                if "down" not in skip:
                    C.moe_down(lw["w_d"], nb.act_moe, nb.ids, nb.wts, nb.x, None)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen3-next-80b-a3b")
    ap.add_argument("--layers", type=int, default=0, help="truncate to the first N layers (0 = all)")
    ap.add_argument("--context", type=int, default=8192)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--eager", action="store_true")
    ap.add_argument("--quant", default=None, help="in-situ quantization (Q8_0, Q6_K, Q4_K, Q4_K_M)")
    ap.add_argument("--no-pdl", action="store_true", help="launch without programmatic dependent launch")
    ap.add_argument("--skip", default="", help="profiling only: comma list of gdn,attn,gdn_core,attn_core,ffn,experts,down")
    args = ap.parse_args()
    if args.no_pdl:
        from .. import ops
        ops.C.set_pdl(False)
    cfg = get_preset(args.model)
    if args.layers:
        cfg = dataclasses.replace(cfg, num_hidden_layers=args.layers, layer_types=cfg.layer_types[:args.layers])
    dev = torch.device("cuda", 0)
    fm = FastModel.random(cfg, dev, max_slots=args.batch, max_len=args.context + args.steps * 4 + 64)
    B = args.batch
    if args.quant:
        fm.quantize_(args.quant.upper())
    if args.skip:
        fm.__class__ = SkippingModel
        fm.skip = frozenset(x for x in args.skip.split(",") if x)
    if args.eager:
        nb = fm.buffers(B)
    else:
        nb = fm.capture(B, steps=args.steps)
    nb.slots.copy_(torch.arange(B, dtype=torch.int32, device=dev))

    def run():
        fm.pos.fill_(args.context)
        if args.eager:
            for _ in range(args.steps):
                fm.decode_step_launch(nb)
        else:
            fm.replay(nb)

    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    run()
    e1.record()
    e1.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    gb = fm.decode_bytes_per_token() / 1e9
    print(json.dumps({"model": cfg.name, "layers": cfg.num_hidden_layers, "context": args.context, "batch": B,
                      "graph": not args.eager, "pdl": not args.no_pdl, "skip": args.skip, "ms_per_step": round(ms, 4),
                      "weight_gb_per_step": round(gb, 3), "achieved_gbs": round(gb / (ms / 1e3), 1),
                      "launches_per_step": fm.launches_per_step()}))


if __name__ == "__main__":
    main()
