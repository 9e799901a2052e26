"""Model runners: one interface over the CUDA model and the CPU reference model.

A runner owns a fixed pool of sequence slots and exposes prefill / batched decode /
snapshot / restore on slot ids. Snapshots capture everything a continuation needs
(arch/qwen3_5/snapshot.rs:32-311): attention K/V up to the cut, and a DEEP copy of
the GDN conv ring and recurrent state (the reference learned that sharing the GDN
state between a snapshot and a live sequence corrupts both, doc/learnings/p2.md).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch


@dataclass
class Snapshot:
    length: int
    kv: dict = field(default_factory=dict)     # layer -> (k [Hkv, L, D], v [Hkv, L, D])
    conv: dict = field(default_factory=dict)   # layer -> ring / conv state
    rec: dict = field(default_factory=dict)    # layer -> recurrent state
    ref_state: object = None                   # CPU reference model state
    rope_delta: int = 0                        # multimodal rotary offset at the cut

    @property
    def nbytes(self) -> int:
        n = 0
        for k, v in self.kv.values():
            n += k.numel() * k.element_size() + v.numel() * v.element_size()
        for d in (self.conv, self.rec):
            for t in d.values():
                n += t.numel() * t.element_size()
        if self.ref_state is not None:
            n += self.ref_state.nbytes()
        return n


class FastRunner:
    """CUDA runner over a FastModel's slot pools."""

    greedy_on_device = True

    def __init__(self, model, graph_steps: int = 8, prefill_chunk: int = 8192):
        self.m = model
        self.num_slots = model.max_slots - 1          # the last slot pads odd batches
        self.pad_slot = model.max_slots - 1
        self.graph_steps = graph_steps
        self.prefill_chunk = prefill_chunk
        self.max_len = model.max_len
        self.vocab = model.cfg.vocab_size
        self.host_pos = [0] * model.max_slots

    @staticmethod
    def bucket(n: int) -> int:
        for b in (1, 2, 4, 8):
            if n <= b:
                return b
        raise ValueError("decode batch larger than 8")

    def reset(self, slot: int):
        m = self.m
        m.pos[slot] = 0
        m.set_rope_delta(slot, 0)
        for t in m.rec.values():
            t[slot].zero_()
        for t in m.conv.values():
            t[slot].zero_()
        self.host_pos[slot] = 0

    def prefill(self, slot: int, tokens: list[int], p0: int) -> torch.Tensor:
        dev = self.m.device
        toks = torch.tensor(tokens, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        logits = None
        for s in range(0, len(tokens), self.prefill_chunk):
            logits = self.m.prefill(slot, toks[s:s + self.prefill_chunk], p0 + s)
        self.host_pos[slot] = p0 + len(tokens)
        self.m.check_errors()  # a timed-out wait makes the outputs invalid: poison, don't serve
        return logits

    def prefill_mm(self, slot: int, mm) -> torch.Tensor:
        """Prefill a multimodal prompt (runtime/multimodal.py MultimodalPrompt) at
        position 0 from its input embeddings and M-RoPE positions; later decode steps
        rotate at the prompt's next rotary position."""
        m = self.m
        emb = mm.embeds.to(m.device, torch.bfloat16)
        logits = m.prefill(slot, None, 0, embeds=emb, pos3=mm.pos3, next_pos=mm.next_pos)
        self.host_pos[slot] = len(mm.tokens)
        m.check_errors()
        return logits

    def decode(self, slots: list[int], tokens: list[int], steps: int) -> list[list[int]]:
        """Run `steps` greedy steps for the given slots starting from `tokens`; returns
        the produced tokens per slot. Pads to a captured batch size with the pad slot."""
        m = self.m
        B = self.bucket(len(slots))
        nb = m.capture(B, steps=steps)
        pad = B - len(slots)
        sl = list(slots) + [self.pad_slot] * pad
        tk = list(tokens) + [0] * pad
        nb.slots.copy_(torch.tensor(sl, dtype=torch.int32), non_blocking=True)
        nb.tok.copy_(torch.tensor(tk, dtype=torch.int32), non_blocking=True)
        nb.step.zero_()
        m.pos[self.pad_slot] = 0
        m.replay(nb)
        out = nb.out_tokens[:len(slots), :steps].cpu().tolist()
        m.check_errors()
        for s in slots:
            self.host_pos[s] += steps
        return out

    sample_on_device = True

    def decode_sampled(self, slots: list[int], tokens: list[int], steps: int, params: list,
                       histories: list[list[int]], draws: list[int], seeds: list[int]) -> list[list[int]]:
        """`steps` sampled steps on the device (temperature / top-k / top-p / repeat
        penalty per row, seeded draws), replayed from a captured graph; returns the
        tokens per slot. `draws` numbers each sequence's earlier device draws, so a
        seeded request gives the same tokens however its steps are grouped."""
        m = self.m
        B = self.bucket(len(slots))
        st = m.sampler
        for sl, p, h, d, sd in zip(slots, params, histories, draws, seeds):
            st.set_slot(sl, p.temperature, p.top_k, p.top_p, p.repeat_penalty, p.repeat_last_n, sd, d, h)
        pad = B - len(slots)
        if pad:
            st.set_slot(self.pad_slot, 0.0, 0, 1.0, 1.0, 1, 0, 0, [])
        nb = m.capture(B, steps=steps, sampled=True)
        sl = list(slots) + [self.pad_slot] * pad
        tk = list(tokens) + [0] * pad
        nb.slots.copy_(torch.tensor(sl, dtype=torch.int32), non_blocking=True)
        nb.tok.copy_(torch.tensor(tk, dtype=torch.int32), non_blocking=True)
        nb.step.zero_()
        m.pos[self.pad_slot] = 0
        m.replay(nb, sampled=True)
        out = nb.out_tokens[:len(slots), :steps].cpu().tolist()
        m.check_errors()
        for s in slots:
            self.host_pos[s] += steps
        return out

    def decode_logits(self, slots: list[int], tokens: list[int]) -> torch.Tensor:
        """One eager step returning f32 logits [n, V] (host-sampled requests)."""
        m = self.m
        B = self.bucket(len(slots))
        nb = m.buffers(B)
        pad = B - len(slots)
        nb.slots.copy_(torch.tensor(list(slots) + [self.pad_slot] * pad, dtype=torch.int32))
        nb.tok.copy_(torch.tensor(list(tokens) + [0] * pad, dtype=torch.int32))
        m.pos[self.pad_slot] = 0
        m.decode_step_launch(nb)
        for s in slots:
            self.host_pos[s] += 1
        lg = m.full_logits(nb.logits[:len(slots)].float()).cpu()
        m.check_errors()
        return lg

    def snapshot(self, slot: int, length: int) -> Snapshot:
        m = self.m
        snap = Snapshot(length=length)
        for i in m.kc:
            snap.kv[i] = (m.kc[i][slot, :, :length].clone(), m.vc[i][slot, :, :length].clone())
        for i in m.conv:
            snap.conv[i] = m.conv[i][slot].clone()
            snap.rec[i] = m.rec[i][slot].clone()
        snap.rope_delta = m._rope_delta_host[slot]
        return snap

    def restore(self, slot: int, snap: Snapshot):
        m = self.m
        L = snap.length
        for i, (k, v) in snap.kv.items():
            m.kc[i][slot, :, :L] = k
            m.vc[i][slot, :, :L] = v
        for i in snap.conv:
            m.conv[i][slot] = snap.conv[i]
            m.rec[i][slot] = snap.rec[i]
        m.pos[slot] = L
        m.set_rope_delta(slot, snap.rope_delta)
        self.host_pos[slot] = L


class RefRunner:
    """CPU runner over the fp32 reference model (tests, CPU serving)."""

    greedy_on_device = False

    def __init__(self, model, num_slots: int = 4, max_len: int = 4096):
        self.m = model
        self.num_slots = num_slots
        self.max_len = max_len
        self.vocab = model.cfg.vocab_size
        self.states = [model.new_state() for _ in range(num_slots)]
        self.host_pos = [0] * num_slots

    def reset(self, slot: int):
        self.states[slot] = self.m.new_state()
        self.host_pos[slot] = 0

    def prefill(self, slot: int, tokens: list[int], p0: int) -> torch.Tensor:
        assert self.states[slot].length == p0
        lg = self.m.forward(torch.tensor(tokens), self.states[slot])
        self.host_pos[slot] = p0 + len(tokens)
        return lg

    def prefill_mm(self, slot: int, mm) -> torch.Tensor:
        assert self.states[slot].length == 0
        lg = self.m.forward(None, self.states[slot], embeds=mm.embeds, pos3=mm.pos3, next_pos=mm.next_pos)
        self.host_pos[slot] = len(mm.tokens)
        return lg

    def decode_logits(self, slots: list[int], tokens: list[int]) -> torch.Tensor:
        out = [self.m.forward(torch.tensor([t]), self.states[s]) for s, t in zip(slots, tokens)]
        for s in slots:
            self.host_pos[s] += 1
        return torch.stack(out)

    def decode(self, slots: list[int], tokens: list[int], steps: int) -> list[list[int]]:
        res = [[] for _ in slots]
        cur = list(tokens)
        for _ in range(steps):
            lg = self.decode_logits(slots, cur)
            cur = [int(x) for x in lg.argmax(-1)]
            for r, t in zip(res, cur):
                r.append(t)
        return res

    def snapshot(self, slot: int, length: int) -> Snapshot:
        st = self.states[slot]
        assert st.length == length, "reference snapshots are taken at the current length"
        return Snapshot(length=length, ref_state=self.m.snapshot(st))

    def restore(self, slot: int, snap: Snapshot):
        self.states[slot] = self.m.restore(snap.ref_state)
        self.host_pos[slot] = snap.length
