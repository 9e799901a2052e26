"""GGUF container reader/writer (format v3) for Qwen3-family checkpoints.

The container layout and the k-quant block formats are the published GGUF / ggml
formats (so files interoperate with other runtimes); the code is written from the
format description:

  header: "GGUF", u32 version, u64 n_tensors, u64 n_kv; key/value metadata;
  tensor infos (name, n_dims, dims (innermost first), ggml type, data offset);
  data section aligned to `general.alignment` (default 32).

Block types supported here (bytes per block / values per block):
  F32, F16, BF16, Q8_0 (34 / 32), Q4_K (144 / 256), Q6_K (210 / 256).
Quantize / dequantize on the host run in C++ (csrc/gguf_host.cpp); the decode GEMV
and the prefill path dequantize on the GPU (csrc/gguf.cu).

Qwen3 GGUF tensor names map onto HF names (`blk.{i}.attn_q.weight` ->
`model.layers.{i}.self_attn.q_proj.weight`, ...); the reference loads GGUF only on
a single GPU (harness/candle.rs:887-895) while here GGUF tensors are sliced per rank
on superblock boundaries.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass

import numpy as np
import torch

from ..config import ModelConfig

GGUF_MAGIC = b"GGUF"
F32, F16, Q8_0, Q4_K, Q6_K, BF16 = 0, 1, 8, 12, 14, 30
BLOCK = {F32: (4, 1), F16: (2, 1), BF16: (2, 1), Q8_0: (34, 32), Q4_K: (144, 256), Q6_K: (210, 256)}
TYPE_NAMES = {F32: "F32", F16: "F16", BF16: "BF16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}

# value types
_VT = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}


def _hf_name(gname: str) -> str | None:
    if gname == "token_embd.weight":
        return "model.embed_tokens.weight"
    if gname == "output_norm.weight":
        return "model.norm.weight"
    if gname == "output.weight":
        return "lm_head.weight"
    if not gname.startswith("blk."):
        return None
    _, i, rest = gname.split(".", 2)
    if rest in _EXPS:  # [E, rows, cols] stack: no single HF tensor (hf_get slices it)
        return None
    m = {
        "attn_norm.weight": "input_layernorm.weight", "ffn_norm.weight": "post_attention_layernorm.weight",
        "attn_q.weight": "self_attn.q_proj.weight", "attn_k.weight": "self_attn.k_proj.weight",
        "attn_v.weight": "self_attn.v_proj.weight", "attn_output.weight": "self_attn.o_proj.weight",
        "attn_q_norm.weight": "self_attn.q_norm.weight", "attn_k_norm.weight": "self_attn.k_norm.weight",
        "ffn_gate.weight": "mlp.gate_proj.weight", "ffn_up.weight": "mlp.up_proj.weight",
        "ffn_down.weight": "mlp.down_proj.weight", "ffn_gate_inp.weight": "mlp.gate.weight",
    }.get(rest)
    return None if m is None else f"model.layers.{i}.{m}"


# qwen3moe expert stacks: GGUF keeps every expert of a projection in one 3D tensor
_EXPS = {"ffn_gate_exps.weight": "gate_proj", "ffn_up_exps.weight": "up_proj", "ffn_down_exps.weight": "down_proj"}
_EXP_OF = {v: k for k, v in _EXPS.items()}


def expert_name(hf: str) -> tuple[str, int] | None:
    """`model.layers.{i}.mlp.experts.{e}.{proj}.weight` -> (GGUF stack name, e)."""
    parts = hf.split(".")
    if len(parts) == 8 and parts[3] == "mlp" and parts[4] == "experts" and parts[6] in _EXP_OF:
        return f"blk.{parts[2]}.{_EXP_OF[parts[6]]}", int(parts[5])
    return None


def hf_to_gguf_name(hf: str) -> str:
    rev = {
        "input_layernorm.weight": "attn_norm.weight", "post_attention_layernorm.weight": "ffn_norm.weight",
        "self_attn.q_proj.weight": "attn_q.weight", "self_attn.k_proj.weight": "attn_k.weight",
        "self_attn.v_proj.weight": "attn_v.weight", "self_attn.o_proj.weight": "attn_output.weight",
        "self_attn.q_norm.weight": "attn_q_norm.weight", "self_attn.k_norm.weight": "attn_k_norm.weight",
        "mlp.gate_proj.weight": "ffn_gate.weight", "mlp.up_proj.weight": "ffn_up.weight",
        "mlp.down_proj.weight": "ffn_down.weight", "mlp.gate.weight": "ffn_gate_inp.weight",
    }
    if hf == "model.embed_tokens.weight":
        return "token_embd.weight"
    if hf == "model.norm.weight":
        return "output_norm.weight"
    if hf == "lm_head.weight":
        return "output.weight"
    _, _, i, rest = hf.split(".", 3)
    return f"blk.{i}.{rev[rest]}"


@dataclass
class GGUFTensor:
    name: str
    shape: tuple[int, ...]     # torch order (outermost first)
    gtype: int
    offset: int
    nbytes: int


class GGUFFile:
    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self._pos = 0
        if self._read(4) != GGUF_MAGIC:
            raise ValueError(f"{path} is not a GGUF file")
        self.version = self._u32()
        n_t, n_kv = self._u64(), self._u64()
        self.meta: dict = {}
        for _ in range(n_kv):
            k = self._str()
            self.meta[k] = self._value(self._u32())
        infos = []
        for _ in range(n_t):
            name = self._str()
            nd = self._u32()
            dims = [self._u64() for _ in range(nd)]
            gt = self._u32()
            off = self._u64()
            infos.append((name, tuple(reversed(dims)), gt, off))
        align = int(self.meta.get("general.alignment", 32))
        base = (self._pos + align - 1) // align * align
        self.tensors: dict[str, GGUFTensor] = {}
        for name, shape, gt, off in infos:
            bb, bv = BLOCK[gt]
            n = int(np.prod(shape))
            self.tensors[name] = GGUFTensor(name, shape, gt, base + off, n // bv * bb)

    # ---- primitive reads ---------------------------------------------------
    def _read(self, n):
        b = self._mm[self._pos:self._pos + n]
        self._pos += n
        return b

    def _u32(self):
        return struct.unpack("<I", self._read(4))[0]

    def _u64(self):
        return struct.unpack("<Q", self._read(8))[0]

    def _str(self):
        return self._read(self._u64()).decode("utf-8")

    def _value(self, vt):
        if vt == 8:
            return self._str()
        if vt == 9:
            et, n = self._u32(), self._u64()
            return [self._value(et) for _ in range(n)]
        fmt = _VT[vt]
        return struct.unpack("<" + fmt, self._read(struct.calcsize(fmt)))[0]

    # ---- access --------------------------------------------------------------
    def raw(self, name: str) -> torch.Tensor:
        """Undecoded block bytes as a uint8 tensor (shares the mmap)."""
        t = self.tensors[name]
        return torch.frombuffer(self._mm, dtype=torch.uint8, count=t.nbytes, offset=t.offset)

    def tensor(self, name: str) -> torch.Tensor:
        """Decoded tensor (f32 for quantized types)."""
        from .. import ops
        t = self.tensors[name]
        raw = self.raw(name)
        if t.gtype == F32:
            return raw.view(torch.float32).reshape(t.shape).clone()
        if t.gtype == F16:
            return raw.view(torch.float16).reshape(t.shape).float()
        if t.gtype == BF16:
            return raw.view(torch.bfloat16).reshape(t.shape).float()
        return ops.C.gguf_dequant_host(raw.clone(), t.gtype, int(np.prod(t.shape))).reshape(t.shape)

    def hf_state_dict(self) -> dict[str, torch.Tensor]:
        """Every tensor decoded under its HF name; expert stacks split per expert."""
        out = {}
        for name in self.tensors:
            hf = _hf_name(name)
            if hf is not None:
                out[hf] = self.tensor(name)
                continue
            rest = name.split(".", 2)[2] if name.startswith("blk.") else ""
            if rest in _EXPS:
                i = name.split(".")[1]
                st = self.tensor(name)
                for e in range(st.shape[0]):
                    out[f"model.layers.{i}.mlp.experts.{e}.{_EXPS[rest]}.weight"] = st[e]
        return out

    def hf_get(self, hf_name: str) -> torch.Tensor:
        ex = expert_name(hf_name)
        if ex is not None:
            # one expert of a stack: the stack is decoded once and kept until another is asked for
            name, e = ex
            if getattr(self, "_stack", (None,))[0] != name:
                self._stack = (name, self.tensor(name))
            return self._stack[1][e]
        return self.tensor(hf_to_gguf_name(hf_name))

    def model_config(self) -> ModelConfig:
        m = self.meta
        arch = m.get("general.architecture", "qwen3")
        g = lambda k, d=None: m.get(f"{arch}.{k}", d)  # noqa: E731
        heads = int(g("attention.head_count"))
        hidden = int(g("embedding_length"))
        vocab = len(m.get("tokenizer.ggml.tokens", [])) or int(g("vocab_size", 151936))
        family = "qwen3_moe" if arch == "qwen3moe" else "qwen3"
        return ModelConfig(
            family=family, name=m.get("general.name", "gguf-model"), vocab_size=vocab, hidden_size=hidden,
            num_hidden_layers=int(g("block_count")), num_attention_heads=heads,
            num_key_value_heads=int(g("attention.head_count_kv", heads)),
            head_dim=int(g("attention.key_length", hidden // heads)),
            intermediate_size=int(g("feed_forward_length", 0)),
            rms_norm_eps=float(g("attention.layer_norm_rms_epsilon", 1e-6)),
            rope_theta=float(g("rope.freq_base", 1e6)),
            max_position_embeddings=int(g("context_length", 40960)),
            num_experts=int(g("expert_count", 0) or 0), num_experts_per_tok=int(g("expert_used_count", 0) or 0),
            moe_intermediate_size=int(g("expert_feed_forward_length", 0) or 0),
            tie_word_embeddings="output.weight" not in self.tensors)

    def close(self):
        self._mm.close()
        self._f.close()


# ---------------------------------------------------------------------------
# writer
# ---------------------------------------------------------------------------
def _w_str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _w_value(v) -> bytes:
    if isinstance(v, bool):
        return struct.pack("<I?", 7, v)
    if isinstance(v, int):
        return struct.pack("<Iq", 11, v) if v < 0 else struct.pack("<IQ", 10, v) if v >= 2 ** 32 else \
            struct.pack("<II", 4, v)
    if isinstance(v, float):
        return struct.pack("<If", 6, v)
    if isinstance(v, str):
        return struct.pack("<I", 8) + _w_str(v)
    if isinstance(v, list):
        if all(isinstance(x, str) for x in v):
            return struct.pack("<IIQ", 9, 8, len(v)) + b"".join(_w_str(x) for x in v)
        if all(isinstance(x, int) for x in v):
            return struct.pack("<IIQ", 9, 5, len(v)) + b"".join(struct.pack("<i", x) for x in v)
        return struct.pack("<IIQ", 9, 6, len(v)) + b"".join(struct.pack("<f", float(x)) for x in v)
    raise TypeError(type(v))


def write_gguf(path: str, meta: dict, tensors: list[tuple[str, torch.Tensor, int]], align: int = 32):
    """tensors: (gguf name, f32/bf16 tensor, target ggml type); quantizes on the host."""
    from .. import ops
    blobs = []
    for name, t, gt in tensors:
        t = t.detach().float().contiguous().cpu()
        if gt == F32:
            data = t.numpy().tobytes()
        elif gt == F16:
            data = t.half().numpy().tobytes()
        elif gt == BF16:
            data = t.bfloat16().view(torch.int16).numpy().tobytes()
        else:
            data = ops.C.gguf_quant_host(t.view(-1), gt).numpy().tobytes()
        blobs.append((name, tuple(t.shape), gt, data))
    head = GGUF_MAGIC + struct.pack("<IQQ", 3, len(blobs), len(meta) + 1)
    kv = _w_str("general.alignment") + _w_value(align)
    for k, v in meta.items():
        kv += _w_str(k) + _w_value(v)
    infos, off = b"", 0
    offsets = []
    for name, shape, gt, data in blobs:
        offsets.append(off)
        infos += _w_str(name) + struct.pack("<I", len(shape)) + b"".join(struct.pack("<Q", d) for d in
                                                                         reversed(shape))
        infos += struct.pack("<IQ", gt, off)
        off += (len(data) + align - 1) // align * align
    with open(path, "wb") as f:
        hdr = head + kv + infos
        f.write(hdr)
        f.write(b"\0" * ((align - len(hdr) % align) % align))
        for (_, _, _, data) in blobs:
            f.write(data)
            f.write(b"\0" * ((align - len(data) % align) % align))


# ---------------------------------------------------------------------------
# native quantized layout: block rows straight to the device, no host dequantization
# ---------------------------------------------------------------------------
@dataclass
class QuantRows:
    """A quantized weight as GGUF block rows (uint8 [N, row_bytes], host mmap view)."""
    raw: torch.Tensor
    gtype: int
    K: int

    @property
    def rows(self) -> int:
        return self.raw.shape[0]


def _blocks(gt: int) -> tuple[int, int]:
    return BLOCK[gt]


class QuantLayer:
    """Builds one decoder layer of a dense Qwen3 / Llama GGUF file in the fused per-rank
    layout of models/layout.py, keeping quantized projections as block rows:

      w_qkv  q|k|v rows of this rank's heads (one QuantRows when the three share a
             block type, else a list of segments -- Q4_K_M stores attn_v as Q6_K);
      o_w    row-parallel: this rank's head columns, whole blocks;
      w_gu   gate/up rows of the rank's intermediate shard, interleaved row by row;
      w_d    row-parallel: the shard's columns on superblock boundaries (uneven shards
             when the intermediate size does not split evenly into whole superblocks).
    Tensors stored unquantized (norms, F16/BF16/F32 projections) come back as floats.
    """

    def __init__(self, g: "GGUFFile"):
        self.g = g

    def _raw2d(self, name: str) -> QuantRows:
        t = self.g.tensors[name]
        bb, bv = _blocks(t.gtype)
        N, K = t.shape
        return QuantRows(self.g.raw(name).view(N, K // bv * bb), t.gtype, K)

    def is_quant(self, name: str) -> bool:
        return self.g.tensors[name].gtype in (Q8_0, Q4_K, Q6_K)

    def rows(self, name: str, r0: int, r1: int):
        if not self.is_quant(name):
            return self.g.tensor(name)[r0:r1]
        q = self._raw2d(name)
        return QuantRows(q.raw[r0:r1], q.gtype, q.K)

    def cols(self, name: str, c0: int, c1: int):
        if not self.is_quant(name):
            return self.g.tensor(name)[:, c0:c1]
        q = self._raw2d(name)
        bb, bv = _blocks(q.gtype)
        if c0 % bv or c1 % bv:
            # not on block boundaries: this shard cannot stay quantized
            return self.g.tensor(name)[:, c0:c1]
        nblk = q.K // bv
        part = q.raw.view(q.rows, nblk, bb)[:, c0 // bv:c1 // bv].reshape(q.rows, -1)
        return QuantRows(part, q.gtype, c1 - c0)

    @staticmethod
    def cat_rows(parts: list):
        """Row concatenation; same-type quantized parts merge into one weight."""
        if all(isinstance(p, QuantRows) for p in parts) and len({(p.gtype, p.K) for p in parts}) == 1:
            return QuantRows(torch.cat([p.raw for p in parts], 0), parts[0].gtype, parts[0].K)
        if any(isinstance(p, QuantRows) for p in parts):
            # segments of different block types: merge runs of adjacent same-type parts
            segs: list = []
            for p in parts:
                last = segs[-1] if segs else None
                if isinstance(p, QuantRows) and isinstance(last, QuantRows) and (last.gtype, last.K) == (p.gtype, p.K):
                    segs[-1] = QuantRows(torch.cat([last.raw, p.raw], 0), p.gtype, p.K)
                elif isinstance(p, torch.Tensor) and isinstance(last, torch.Tensor):
                    segs[-1] = torch.cat([last, p], 0)
                else:
                    segs.append(p)
            return segs
        return torch.cat(parts, 0)

    @staticmethod
    def interleave(gt, up):
        if isinstance(gt, QuantRows) and isinstance(up, QuantRows) and gt.gtype == up.gtype:
            raw = torch.stack([gt.raw, up.raw], 1).reshape(-1, gt.raw.shape[1])
            return QuantRows(raw, gt.gtype, gt.K)
        return None

    def layer(self, cfg: ModelConfig, dims, i: int) -> dict:
        from ..models.layout import interleave_rows, norm_f32
        p = f"blk.{i}."
        g = self.g
        out: dict = {"ln1": norm_f32(cfg, g.tensor(p + "attn_norm.weight")),
                     "ln2": norm_f32(cfg, g.tensor(p + "ffn_norm.weight"))}
        D = cfg.head_dim
        hq0 = dims.rank * dims.hq
        q = self.rows(p + "attn_q.weight", hq0 * D, (hq0 + dims.hq) * D)
        k0, k1 = dims.kv_head0 * D, (dims.kv_head0 + dims.hkv) * D
        k = self.rows(p + "attn_k.weight", k0, k1)
        v = self.rows(p + "attn_v.weight", k0, k1)
        out["w_qkv"] = self.cat_rows([q, k, v])
        out["o_w"] = self.cols(p + "attn_output.weight", hq0 * D, (hq0 + dims.hq) * D)
        if cfg.qk_norm:
            out["q_norm"] = norm_f32(cfg, g.tensor(p + "attn_q_norm.weight"))
            out["k_norm"] = norm_f32(cfg, g.tensor(p + "attn_k_norm.weight"))
        if cfg.layer_uses_moe(i):
            out.update(self.moe(cfg, dims, i))
            return out
        i0, i1 = dims.inter0, dims.inter0 + dims.inter
        gate = self.rows(p + "ffn_gate.weight", i0, i1)
        up = self.rows(p + "ffn_up.weight", i0, i1)
        gu = self.interleave(gate, up)
        if gu is None:  # mixed block types: the fused SwiGLU rows fall back to bf16
            deq = lambda t: t if isinstance(t, torch.Tensor) else _dequant_rows(t)  # noqa: E731
            gu = interleave_rows(deq(gate), deq(up))
        out["w_gu"] = gu
        out["w_d"] = self.cols(p + "ffn_down.weight", i0, i1)
        return out


    def moe(self, cfg: ModelConfig, dims, i: int) -> dict:
        """Router (bf16) and the expert stacks of a qwen3moe layer. Whole experts on
        this rank (a single rank) keep their block rows: gate and up
        rows interleave per expert into [E * 2I] rows, down stays [E * H] rows. An
        expert sharded along its intermediate dim (tensor parallel) would split the
        down projection's superblocks, so such shards are dequantized."""
        from ..models.layout import interleave_rows
        p = f"blk.{i}."
        g = self.g
        E, I, H = cfg.num_experts, cfg.moe_intermediate_size, cfg.hidden_size
        out = {"router": g.tensor(p + "ffn_gate_inp.weight")}
        e0, ne = (dims.e0, dims.e_local) if dims.ep else (0, E)
        # (expert parallel ranks would need the quantized down kernel's cross-rank sum:
        # their local experts are dequantized for now)
        whole = dims.ws == 1
        names = [p + n for n in ("ffn_gate_exps.weight", "ffn_up_exps.weight", "ffn_down_exps.weight")]
        types = [g.tensors[n].gtype for n in names]
        if whole and types[0] == types[1] and all(t in (Q4_K, Q6_K) for t in types):
            bb, _ = _blocks(types[0])
            gate = g.raw(names[0]).view(E, I, -1)[e0:e0 + ne]
            up = g.raw(names[1]).view(E, I, -1)[e0:e0 + ne]
            gu = torch.stack([gate, up], 2).reshape(ne * 2 * I, gate.shape[-1])
            dn = g.raw(names[2]).view(E, H, -1)[e0:e0 + ne].reshape(ne * H, -1)
            out["w_gu"] = QuantExperts(gu, types[0], ne, 2 * I, H)
            out["w_d"] = QuantExperts(dn, types[2], ne, H, I)
            return out
        gate, up, down = (g.tensor(n) for n in names)
        if dims.ep:
            gate, up, down = gate[e0:e0 + ne], up[e0:e0 + ne], down[e0:e0 + ne]
            i0, i1 = 0, I
        else:
            per = I // dims.ws
            i0, i1 = dims.rank * per, (dims.rank + 1) * per
        out["w_gu"] = torch.stack([interleave_rows(gate[e, i0:i1], up[e, i0:i1]) for e in range(gate.shape[0])])
        out["w_d"] = down[:, :, i0:i1].contiguous()
        return out


@dataclass
class QuantExperts:
    """Expert stacks as GGUF block rows: uint8 [G * R, K / block * bytes]."""
    raw: torch.Tensor
    gtype: int
    G: int
    R: int
    K: int


def _dequant_rows(q: QuantRows) -> torch.Tensor:
    from .. import ops
    return ops.C.gguf_dequant_host(q.raw.contiguous().view(-1).clone(), q.gtype, q.rows * q.K).view(q.rows, q.K)


def quant_block_of(g: "GGUFFile", name: str) -> int:
    """Values per block of a tensor (1 for unquantized types)."""
    return BLOCK[g.tensors[name].gtype][1]
