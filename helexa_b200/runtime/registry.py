"""Model registry: load / unload / list, single-flight loads, poison recovery.

Mirrors the reference's CandleHarness registry (harness/candle.rs:45-885, load 3818,
unload 4147, recovery 3675-3741): a `ModelSpec` names the source and placement; loads
of the same id are single-flight; unload refuses while requests are in flight unless
forced; a poisoned model is unloaded and reloaded from its retained spec while it
advertises `recovering`. `HELEXA_DEBUG_POISON=<model_id>` forces one recovery (the
reference's NEURON_DEBUG_POISON test hook).
"""
from __future__ import annotations

import asyncio
import os
import threading
from dataclasses import asdict, dataclass, field

import torch

from ..weights.loader import resolve_source
from .admission import AdmissionConfig, AdmissionController
from .context_limit import ContextProfile, derive_limit
from .preflight import PreflightError, preflight
from .engine import Engine
from .prefix_cache import PrefixCache
from .runner import FastRunner, RefRunner
from .sampling import GenerationDefaults
from .serving import ServedModel
from .tokenizer import load_tokenizer


@dataclass
class ModelSpec:
    model_id: str
    source: str
    harness: str = "helexa"
    quant: str | None = None
    tensor_parallel: int = 1
    devices: list[int] | None = None
    max_len: int = 16384
    max_batch: int = 4
    prefix_cache_mb: int = 1024
    prefix_cache_entries: int = 8
    max_in_flight: int | None = None
    max_queue_depth: int = 16
    max_wait_s: float = 60.0
    max_per_principal: int = 0
    device: str | None = None       # "cuda" / "cpu" (default: cuda when available)

    @classmethod
    def from_dict(cls, d: dict) -> "ModelSpec":
        known = {k: v for k, v in d.items() if k in cls.__dataclass_fields__}
        if "model_id" not in known:
            raise ValueError("model_id is required")
        known.setdefault("source", d.get("model") or known["model_id"])
        return cls(**known)


class LoadError(RuntimeError):
    def __init__(self, message: str, code: str = "load_failed", hint: str = ""):
        super().__init__(message)
        self.code, self.hint = code, hint


# free device memory kept back from the KV sizing (activations, graphs, workspace)
FLOOR_BYTES = int(os.environ.get("HELEXA_VRAM_FLOOR_MB", "1500")) << 20


def free_device_bytes(dev: int) -> int:
    """Free memory of a device including what PyTorch's caching allocator holds but is
    not using (that memory is reusable by the next allocation, so it is not "used")."""
    free, _ = torch.cuda.mem_get_info(dev)
    return free + max(0, torch.cuda.memory_reserved(dev) - torch.cuda.memory_allocated(dev))


def plan_max_len(cfg, spec: "ModelSpec", free_bytes: int, weight_bytes: int) -> int:
    """KV length per slot that fits the tightest device after the weights, for the
    spec's slot count (context_limit.rs: free memory -> context)."""
    tp = max(1, spec.tensor_parallel)
    prof = ContextProfile.from_config(cfg, tp)
    lim = derive_limit(prof, max(0, free_bytes - weight_bytes), floor_bytes=FLOOR_BYTES,
                       concurrent=spec.max_batch + 1)
    return max(0, min(spec.max_len, cfg.max_position_embeddings, lim.context))


def build_served_model(spec: ModelSpec) -> ServedModel:
    src = resolve_source(spec.source)
    cfg = src.config
    use_cuda = (spec.device or ("cuda" if torch.cuda.is_available() else "cpu")) == "cuda"
    devs_free = None
    if use_cuda:
        ids = spec.devices or list(range(spec.tensor_parallel))
        devs_free = [free_device_bytes(d) for d in ids]
    try:
        kind = src.kind
        if kind == "dir":
            from ..weights.loader import classify_dir
            kind = classify_dir(src.path)
        preflight(kind, cfg, spec.tensor_parallel, spec.quant, devs_free)
    except PreflightError as e:
        raise LoadError(e.message, e.code, e.hint) from e
    if spec.tensor_parallel > 1:
        if not use_cuda:
            return _build_tp_cpu(spec, src, cfg)
        return _build_tp(spec, src, cfg, devs_free)
    tok = load_tokenizer(src.path, cfg.vocab_size)
    max_len = min(spec.max_len, cfg.max_position_embeddings)
    if use_cuda:
        bpp = {"Q4_K": 0.5625, "Q4_K_M": 0.6, "Q6_K": 0.82, "Q8_0": 1.0625}.get((spec.quant or "").upper(), 2.0)
        # bf16 weights exist before in-situ quantization, so size KV for the bf16 load
        max_len = plan_max_len(cfg, spec, devs_free[0], int(cfg.param_count() * max(bpp, 2.0)))
        if max_len < 256:
            raise LoadError(f"only {max_len} tokens of KV fit beside the weights", "insufficient_memory",
                            "lower max_batch or use more tensor-parallel ranks")
        from ..models.fast import FastModel
        dev = torch.device("cuda", (spec.devices or [0])[0])
        kw = dict(max_slots=spec.max_batch + 1, max_len=max_len)
        if src.kind == "preset":
            model = FastModel.random(cfg, dev, **kw)
        elif src.kind == "gguf":
            from ..weights.gguf import GGUFFile
            g = GGUFFile(src.path)
            model = FastModel.from_gguf(cfg, g, dev, **kw)
        else:
            from ..weights.loader import SafetensorsDir
            st = SafetensorsDir(src.path)
            model = FastModel.from_hf(cfg, st.get, dev, **kw)
        if spec.quant:  # in-situ quantization of the dense projections (ISQ)
            model.quantize_(spec.quant.upper())
        runner = FastRunner(model)
        kv_bpt = cfg.kv_bytes_per_token()
        vget = None
        if cfg.vision and src.kind == "preset":
            from ..models.vision import VisionConfig, random_vision_weights
            vget = random_vision_weights(VisionConfig.from_dict(cfg.vision)).__getitem__
        elif cfg.vision and src.kind != "gguf":
            vget = st.get
        embed_table, vdev = model.embed_w, dev
    else:
        from ..models.reference import ReferenceModel
        if src.kind == "preset":
            from ..weights.random_init import random_weights
            w = random_weights(cfg, seed=0)
        elif src.kind == "gguf":
            from ..weights.gguf import GGUFFile
            g = GGUFFile(src.path)
            w = g.hf_state_dict()
        else:
            from ..weights.loader import SafetensorsDir
            st = SafetensorsDir(src.path)
            w = {k: st.get(k) for k in st.keys()}
        model = ReferenceModel(cfg, w)
        runner = RefRunner(model, num_slots=spec.max_batch, max_len=max_len)
        kv_bpt = 0
        vget = w.__getitem__ if cfg.vision and src.kind != "gguf" else None
        embed_table, vdev = w["model.embed_tokens.weight"], "cpu"
    pc = PrefixCache(spec.prefix_cache_mb << 20, spec.prefix_cache_entries) if spec.prefix_cache_mb else None
    im_start = tok.token_id("<|im_start|>")
    engine = Engine(runner, prefix_cache=pc, im_start_id=im_start, max_batch=spec.max_batch)
    adm = AdmissionController(AdmissionConfig(max_in_flight=spec.max_in_flight or spec.max_batch,
                                              max_queue_depth=spec.max_queue_depth, max_wait_s=spec.max_wait_s,
                                              max_per_principal=spec.max_per_principal))
    defaults = GenerationDefaults.from_dir(src.path) if src.path and os.path.isdir(src.path) else \
        GenerationDefaults()
    sm = ServedModel(model_id=spec.model_id, engine=engine, tokenizer=tok, config=cfg, admission=adm,
                     defaults=defaults, devices=spec.devices or ([0] if use_cuda else []),
                     tensor_parallel=spec.tensor_parallel, spec=asdict(spec), kv_bytes_per_token=kv_bpt)
    if vget is not None:
        # vision tower beside the LM (a GGUF LM carries its tower in a separate mmproj
        # file, which this node does not load: such models serve text only)
        from .multimodal import VisionFrontend
        sm.vision = VisionFrontend.from_weights(cfg, vget, embed_table, tok, device=vdev)
        sm.capabilities = sorted(set(sm.capabilities) | {"vision"})
    if use_cuda:
        # KV pools are preallocated for every slot at max_len, so the admission budget is
        # that pool (a request reserves its prompt + output tokens against it)
        adm.set_kv_budget_mb((kv_bpt * max_len * spec.max_batch) >> 20)
        devs = list(sm.devices)
        sm.free_vram_mb = lambda: min(free_device_bytes(d) for d in devs) >> 20
    return sm


def _build_tp(spec, src, cfg, devs_free):
    from .tp_pool import build_tp_served_model
    return build_tp_served_model(spec, src, cfg, devs_free)


def _build_tp_cpu(spec, src, cfg):
    """tensor_parallel > 1 without GPUs: gloo rank processes that each run the full
    fp32 reference model of a preset (the pool's host logic, no sharding). The
    `HELEXA_DEBUG_TP_FAIL=<rank>:<prefill length>` hook makes that rank raise on such a
    prefill (host-side fault injection for recovery tests)."""
    from .tp_pool import serve_runner, spawn_pool
    if src.kind != "preset":
        raise LoadError("tensor_parallel > 1 on the CPU serves presets only", "bad_tensor_parallel")
    args = {"preset": src.preset, "max_slots": spec.max_batch + 1, "max_len": min(spec.max_len, 4096)}
    fail = os.environ.get("HELEXA_DEBUG_TP_FAIL")
    if fail:
        r, n = fail.split(":")
        args.update(fail_rank=int(r), fail_prefill_len=int(n))
    runner = spawn_pool(spec.tensor_parallel, "helexa_b200.runtime.tp_pool:cpu_ref_runner", args, backend="gloo",
                        init_timeout_s=300)
    return serve_runner(spec, src, cfg, runner, [], runner.max_len)


class ModelRegistry:
    def __init__(self):
        self.models: dict[str, ServedModel] = {}
        self.image_models: dict = {}  # model id -> image_serving.ServedImageModel
        self.specs: dict[str, ModelSpec] = {}
        self.loading: dict[str, asyncio.Future] = {}
        self.recovering: set[str] = set()
        self._lock = threading.Lock()
        self._debug_poison = os.environ.get("HELEXA_DEBUG_POISON")

    def get(self, model_id: str) -> ServedModel | None:
        m = self.models.get(model_id)
        if m is not None and self._debug_poison == model_id:
            self._debug_poison = None
            m.status = "poisoned"
        return m

    def list(self) -> list[dict]:
        out = []
        for mid, m in self.models.items():
            lim = m.limits
            out.append({"id": mid, "status": "recovering" if mid in self.recovering else m.status,
                        "devices": m.devices, "tensor_parallel": m.tensor_parallel,
                        "capabilities": m.capabilities,
                        "limit": {"context": lim.context, "input": lim.input, "output": lim.output},
                        "tool_call": True, "reasoning": True, "servable": m.status == "loaded"})
        out += [m.describe() for m in self.image_models.values()]
        for mid in self.loading:
            if mid not in self.models and mid not in self.image_models:
                out.append({"id": mid, "status": "loading"})
        return out

    async def load(self, spec: ModelSpec) -> ServedModel:
        if spec.model_id in self.models:
            return self.models[spec.model_id]
        from .image_serving import build_image_model, is_image_source
        if is_image_source(spec.source):
            if spec.model_id in self.image_models:
                return self.image_models[spec.model_id]
            if spec.tensor_parallel > 1:
                raise LoadError("image models load on one device", "unsupported_parallelism")
            m = await asyncio.to_thread(build_image_model, spec)
            self.image_models[spec.model_id] = m
            self.specs[spec.model_id] = spec
            return m
        fut = self.loading.get(spec.model_id)
        if fut is not None:
            return await asyncio.shield(fut)
        loop = asyncio.get_running_loop()
        fut = loop.create_future()
        self.loading[spec.model_id] = fut
        try:
            sm = await asyncio.to_thread(build_served_model, spec)
            self.models[spec.model_id] = sm
            self.specs[spec.model_id] = spec
            fut.set_result(sm)
            return sm
        except Exception as e:
            err = e if isinstance(e, LoadError) else LoadError(str(e))
            fut.set_exception(err)
            fut.exception()  # mark retrieved
            if err is e:
                raise
            raise err from e
        finally:
            self.loading.pop(spec.model_id, None)

    async def unload(self, model_id: str, force: bool = False) -> bool:
        im = self.image_models.pop(model_id, None)
        if im is not None:
            im.status = "unloading"
            del im
            if torch.cuda.is_available():
                torch.cuda.empty_cache()
            return True
        m = self.models.get(model_id)
        if m is None:
            return False
        if not force and (m.engine.in_flight or m.engine.queue_depth):
            raise LoadError(f"{model_id} has requests in flight")
        m.admission.close()
        m.status = "unloading"
        await asyncio.to_thread(m.engine.shutdown)
        close = getattr(m.engine.runner, "close", None)
        if close is not None:  # tensor-parallel pool: stop the rank processes
            await asyncio.to_thread(close)
        self.models.pop(model_id, None)
        del m
        if torch.cuda.is_available():
            torch.cuda.empty_cache()
        return True

    async def recover(self, model_id: str) -> ServedModel:
        """Single-flight unload + reload of a poisoned model from its retained spec."""
        if model_id in self.recovering:
            raise LoadError(f"{model_id} is recovering")
        spec = self.specs.get(model_id)
        if spec is None:
            raise LoadError(f"no retained spec for {model_id}")
        self.recovering.add(model_id)
        try:
            await self.unload(model_id, force=True)
            return await self.load(spec)
        finally:
            self.recovering.discard(model_id)

    async def unload_all(self):
        for mid in list(self.models) + list(self.image_models):
            await self.unload(mid, force=True)
