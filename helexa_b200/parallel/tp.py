"""Tensor-parallel communicator for one process per GPU.

Reduction backends for the row-parallel layers (attention o_proj, GDN out_proj,
MLP down_proj, MoE block end -- the reference's two all-reduces per decoder layer,
tp/tp_linear.rs:285-293, tp/tp_qwen3_5.rs:1268-1271):

  "p2p"   (default) decode: the reduction runs inside the producing kernel: each warp
          of the row-parallel GEMV / MoE down stores its rows as (epoch, value) words
          into every peer's receive slot over NVLink and sums the peers' rows into the
          residual (csrc/tp_fused.cuh) -- no separate collective launch; prefill: the
          row-parallel GEMM writes into an exported staging buffer and one kernel does
          reduce-scatter + residual + RMSNorm + all-gather over peer memory
          (csrc/tp_prefill.cu)
  "p2p1"  a separate one-shot reduction kernel after the GEMV, over CUDA-IPC peer
          buffers, fused with the residual add (csrc/allreduce.cu)
  "nccl"  the reference-equivalent baseline: ncclAllReduce (through
          torch.distributed) of the row-parallel partial, then the residual add

All device waits are bounded and CUDA-graph safe.

Rendezvous and prefill-size reductions use torch.distributed (NCCL on GPUs, gloo on
CPU ranks in tests), standing in for the reference's hex-encoded ncclUniqueId sent
over worker stdin (tp/nccl_state.rs:120-359).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from .. import ops

_FLAG_BYTES = 4096


class TPError(RuntimeError):
    """A peer failed to arrive within the reduction timeout (see `check`)."""


class TPComm:
    def __init__(self, group=None, device: torch.device | None = None, mode: str | None = None,
                 max_elems: int = 8 * 16384, timeout_s: float = 5.0):
        self.group = group or dist.group.WORLD
        self.ws = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.device = device or torch.device("cpu")
        self.mode = mode or os.environ.get("HELEXA_TP_MODE", "p2p")
        if self.device.type != "cuda":
            self.mode = "host"
        self.timeout_s = timeout_s
        if self.mode not in ("p2p", "p2p1", "nccl", "host"):
            raise ValueError(f"unknown TP mode {self.mode!r}")
        self.fused = self.mode == "p2p"
        # prefill reduce-scatter / all-gather through NVLink multicast (NVLS) when the
        # devices support it (HELEXA_TP_NVLS=1); otherwise plain peer loads and stores
        self.nvls = self.device.type == "cuda" and os.environ.get("HELEXA_TP_NVLS", "0") == "1"
        self.nvls_error = None
        self.pf_mc = 0
        self.launches_per_reduce = 0 if self.fused else 1
        if self.mode in ("p2p", "p2p1"):
            self._init_p2p(max_elems)
        if self.fused:
            self._init_fused(max_elems)

    # ---- rendezvous of the IPC regions ----------------------------------
    def _init_p2p(self, max_elems: int):
        C = ops.C
        self.data_bytes = ((max_elems * 2 + 255) // 256) * 256
        region, handle = C.ipc_alloc(_FLAG_BYTES + 2 * self.data_bytes, self.device.index)
        self._region = region
        handles: list = [None] * self.ws
        dist.all_gather_object(handles, bytes(handle.numpy().tobytes()), group=self.group)
        self.bases: list[int] = []
        self._opened: list[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.bases.append(region.data_ptr())
            else:
                p = C.ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), self.device.index)
                self.bases.append(p)
                self._opened.append(p)
        self.epoch = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        dist.barrier(group=self.group)

    def _init_fused(self, max_elems: int):
        """Receive region of the fused path: 8-byte (epoch, value) words
        [parity][source rank][max_elems], exported to and opened by every peer
        (csrc/tp_fused.cuh)."""
        C = ops.C
        self.slot_elems = max_elems
        region, handle = C.ipc_alloc(2 * self.ws * max_elems * 8, self.device.index)
        self._fused_region = region
        handles: list = [None] * self.ws
        dist.all_gather_object(handles, bytes(handle.numpy().tobytes()), group=self.group)
        self.fused_bases: list[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.fused_bases.append(region.data_ptr())
            else:
                p = C.ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), self.device.index)
                self.fused_bases.append(p)
                self._opened.append(p)
        self.fused_epoch = torch.zeros(2, dtype=torch.int32, device=self.device)
        dist.barrier(group=self.group)

    # ---- prefill: fused reduce-scatter + residual + RMSNorm + all-gather --------------
    def prefill_region(self, max_tokens: int, hidden: int):
        """Lazily (collectively: every rank calls it at the same prefill) export the
        prefill region [flags | stage T x H | h T x H] (bf16) and open the peers'. Returns
        (stage, h) local views of `max_tokens * hidden` elements each."""
        need = max_tokens * hidden
        if getattr(self, "_pf_elems", 0) >= need and self._pf_hidden == hidden:
            return self._pf_stage, self._pf_h
        C = ops.C
        flag = C.rs_norm_ag_flag_bytes()
        nbytes = need * 2
        self._pf_stage_off = flag
        self._pf_h_off = flag + nbytes
        self.pf_mc = 0
        if self.nvls:
            region = self._nvls_region(flag + 2 * nbytes)
            if region is not None:
                self._pf_region = region
                self._pf_elems, self._pf_hidden = need, hidden
                self.pf_ctr = torch.zeros(2, dtype=torch.int32, device=self.device)
                region[:flag].zero_()
                bf = region[flag:flag + 2 * nbytes].view(torch.bfloat16)
                self._pf_stage, self._pf_h = bf[:need], bf[need:]
                torch.cuda.synchronize(self.device)
                dist.barrier(group=self.group)
                return self._pf_stage, self._pf_h
        region, handle = C.ipc_alloc(flag + 2 * nbytes, self.device.index)
        handles: list = [None] * self.ws
        dist.all_gather_object(handles, bytes(handle.numpy().tobytes()), group=self.group)
        old = getattr(self, "_pf_opened", [])
        if old:
            torch.cuda.synchronize(self.device)
            for p in old:
                ops.C.ipc_close(p)
        self._pf_opened = []
        self.pf_bases: list[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.pf_bases.append(region.data_ptr())
            else:
                p = C.ipc_open(torch.frombuffer(bytearray(h), dtype=torch.uint8), self.device.index)
                self.pf_bases.append(p)
                self._pf_opened.append(p)
        self._pf_region = region
        self._pf_elems, self._pf_hidden = need, hidden
        self.pf_ctr = torch.zeros(2, dtype=torch.int32, device=self.device)
        bf = region[flag:flag + 2 * nbytes].view(torch.bfloat16)
        self._pf_stage, self._pf_h = bf[:need], bf[need:]
        dist.barrier(group=self.group)
        return self._pf_stage, self._pf_h

    def _nvls_region(self, nbytes: int):
        """The prefill region in symmetric memory bound to an NVLink multicast object
        (torch's symmetric-memory rendezvous maps every rank's copy and the multicast
        address): the fused kernel then reduces with multimem.ld_reduce in the switch
        and broadcasts with multimem.st. None (peer-memory path) when the devices have
        no multicast support."""
        try:
            import torch.distributed._symmetric_memory as symm_mem
            g = self.group if self.group is not None else dist.group.WORLD
            try:
                symm_mem.enable_symm_mem_for_group(g.group_name)
            except Exception:
                pass
            t = symm_mem.empty(nbytes, dtype=torch.uint8, device=self.device)
            hdl = symm_mem.rendezvous(t, g.group_name)
            if not hdl.has_multicast_support():
                return None
            self.pf_bases = [int(p) for p in hdl.buffer_ptrs]
            self.pf_mc = int(hdl.multicast_ptr)
            self._pf_symm = hdl
            return t
        except Exception as e:  # no symmetric memory here: peer-memory path
            self.nvls_error = repr(e)
            return None

    def rs_norm_ag(self, x: torch.Tensor, w: torch.Tensor, eps: float):
        """x[own rows] += sum over ranks of the staged partials; every rank's h buffer
        receives RMSNorm(x) * w for all rows (csrc/tp_prefill.cu)."""
        T, H = x.shape
        if T * H > self._pf_elems:
            raise ValueError("prefill chunk larger than the exported region")
        # one warp per owned row, 8 per CTA, two CTAs per SM (all co-resident)
        rows = (T + self.ws - 1) // self.ws
        ctas = max(1, min(2 * self.sms_hint, (rows + 7) // 8))
        ops.C.rs_norm_ag(self.pf_bases, self.rank, self._pf_stage_off, self._pf_h_off, x, w, eps, self.pf_ctr,
                         self.err, self.timeout_s, ctas, self.pf_mc)

    @property
    def sms_hint(self) -> int:
        if not hasattr(self, "_sms"):
            self._sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        return self._sms

    def fused_args(self) -> tuple:
        """Trailing arguments of the fused kernels (gemv_ar, moe_down_ar)."""
        return (self.fused_bases, self.rank, self.slot_elems, self.fused_epoch, self.err, self.timeout_s)

    def close(self):
        if self.mode in ("p2p", "p2p1"):
            torch.cuda.synchronize(self.device)
            dist.barrier(group=self.group)
            for p in self._opened + getattr(self, "_pf_opened", []):
                ops.C.ipc_close(p)
            self._opened, self._pf_opened = [], []

    def error_code(self) -> int:
        """The device error word (0 = healthy); reading it synchronizes the device."""
        return int(self.err.item()) if self.mode in ("p2p", "p2p1") else 0

    def check(self):
        """Raise TPError if a device-side wait timed out since the last check."""
        e = self.error_code()
        if e:
            peer = e - 2000 if e >= 2000 else e - 1000
            raise TPError(f"rank {self.rank}: peer {peer} did not arrive within {self.timeout_s}s (code {e})")

    def all_gather_rows(self, t: torch.Tensor) -> torch.Tensor:
        """Concatenate every rank's `t` along dim -1 (vocab-parallel logits)."""
        parts = [torch.empty_like(t) for _ in range(self.ws)]
        dist.all_gather(parts, t.contiguous(), group=self.group)
        return torch.cat(parts, -1)

    # ---- reductions -------------------------------------------------------
    def all_reduce_(self, t: torch.Tensor) -> torch.Tensor:
        """Sum in place across ranks (prefill-sized tensors)."""
        if self.mode in ("p2p", "p2p1") and t.numel() * 2 <= self.data_bytes and t.dtype == torch.bfloat16:
            flat = t.view(-1)
            ops.C.ar_oneshot(self.bases, self.rank, flat, flat, flat, self.data_bytes, self.epoch, self.err,
                             self._ctas(flat.numel()), self.timeout_s)
            return t
        dist.all_reduce(t, group=self.group)
        return t

    def _ctas(self, n: int) -> int:
        return max(1, min(64, (n + 2047) // 2048))

    def reduce_residual(self, partial: torch.Tensor, x: torch.Tensor):
        """x += sum over ranks of `partial` (decode-size [B, hidden] bf16)."""
        if self.mode in ("p2p", "p2p1"):
            ops.C.ar_oneshot(self.bases, self.rank, partial.view(-1), x.view(-1), None, self.data_bytes,
                             self.epoch, self.err, self._ctas(partial.numel()), self.timeout_s)
        else:
            dist.all_reduce(partial, group=self.group)
            x.add_(partial)
