"""Node HTTP API (the reference's `neuron` routes, api.rs:43-55) plus the gateway-style
OpenAI / Anthropic endpoints, on FastAPI.

  GET  /version /discovery /health /models /v1/models
  POST /models/load /models/unload
  GET  /models/{id}/endpoint /models/{id}/capabilities
  POST /v1/chat/completions /v1/completions /v1/responses /v1/messages
  POST /v1/images/generations   (Z-Image models; a text model answers `wrong_modality` 400)

Chat handling (api.rs:313-389): `max_completion_tokens` aliases `max_tokens`; the
`x-include-thinking` header opts into reasoning output and is the default for
`enable_thinking`; the principal comes from gateway-stamped `x-helexa-*` headers; SSE
streams end with `[DONE]`. Admission refusals map to 429/503 with Retry-After and the
OpenAI error envelope (`rate_limit_exceeded`).
"""
from __future__ import annotations

import json
import os
import platform
import subprocess
import time

from fastapi import FastAPI, Request
from fastapi.responses import JSONResponse, StreamingResponse

from ..runtime.admission import AdmissionRejection
from ..runtime.registry import LoadError, ModelRegistry, ModelSpec
from ..runtime.serving import RequestError
from . import wire

START_TIME = time.time()


def _err(status: int, message: str, code: str, headers: dict | None = None) -> JSONResponse:
    return JSONResponse(wire.error_body(message, code), status_code=status, headers=headers)


def _reject(e: AdmissionRejection) -> JSONResponse:
    h = {"Retry-After": str(e.retry_after)} if e.retry_after else None
    code = "context_length_exceeded" if e.reason == "kv_unservable" else "rate_limit_exceeded"
    return _err(e.status, f"request rejected by admission control: {e.reason}", code, h)


def build_info() -> dict:
    sha = os.environ.get("HELEXA_GIT_SHA")
    if sha is None:
        try:
            sha = subprocess.run(["git", "rev-parse", "--short", "HEAD"], capture_output=True, text=True,
                                 cwd=os.path.dirname(__file__), timeout=5).stdout.strip() or "unknown"
        except Exception:
            sha = "unknown"
    import torch
    return {"name": "helexa-b200", "version": "0.1.0", "git_sha": sha, "torch": torch.__version__,
            "cuda": torch.version.cuda, "python": platform.python_version(), "target": "sm_100a"}


def classify_driver_mismatch(output: str) -> str | None:
    """The userspace NVML version when nvidia-smi failed with the "Driver/library version
    mismatch" error (driver libraries updated, kernel module not reloaded: every CUDA
    call on the host fails until a reboot), "unknown" without a version, None for any
    other failure (discovery.rs:103-158)."""
    if "Driver/library version mismatch" not in output:
        return None
    for line in output.splitlines():
        line = line.strip()
        if line.startswith("NVML library version:"):
            return line.split(":", 1)[1].strip() or "unknown"
    return "unknown"


def kernel_module_version(proc_text: str) -> str | None:
    """Loaded kernel-module version from /proc/driver/nvidia/version's NVRM line."""
    for line in proc_text.splitlines():
        if line.startswith("NVRM version:"):
            for tok in line.split():
                parts = tok.split(".")
                if len(parts) >= 2 and parts[0].isdigit() and parts[1].isdigit():
                    return tok
    return None


def discover_devices(run=None, proc_version: str | None = None) -> dict:
    """GPU inventory from nvidia-smi CSV (discovery.rs:205-240). A failing nvidia-smi is
    classified: a driver/library mismatch becomes `cuda_unavailable_reason` with the
    operator action. `run` and `proc_version` replace the subprocess / proc file in tests."""
    devices = []
    driver = None
    reason = None
    run = run or (lambda cmd: subprocess.run(cmd, capture_output=True, text=True, timeout=10))
    try:
        out = run(["nvidia-smi", "--query-gpu=index,name,memory.total,memory.free,driver_version,"
                   "compute_cap,temperature.gpu,utilization.gpu,power.draw",
                   "--format=csv,noheader,nounits"])
        if out.returncode != 0:
            user = classify_driver_mismatch((out.stdout or "") + (out.stderr or ""))
            if user is not None:
                if proc_version is None:
                    try:
                        with open("/proc/driver/nvidia/version") as f:
                            proc_version = f.read()
                    except OSError:
                        proc_version = ""
                km = kernel_module_version(proc_version) or "unknown"
                reason = (f"host NVIDIA driver/library mismatch (userspace NVML {user} vs loaded kernel module "
                          f"{km}): reboot the host to reload the kernel module; CUDA inference is unavailable "
                          "until then")
        for line in (out.stdout or "").strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 6:
                dev = {"index": int(f[0]), "name": f[1], "memory_total_mb": int(float(f[2])),
                       "memory_free_mb": int(float(f[3])), "compute_capability": f[5]}
                for key, i in (("temperature_c", 6), ("utilization_pct", 7), ("power_w", 8)):
                    try:
                        dev[key] = float(f[i])
                    except (IndexError, ValueError):
                        pass
                devices.append(dev)
                driver = f[4]
    except (OSError, subprocess.SubprocessError):
        pass
    out = {"devices": devices, "driver_version": driver, "hostname": platform.node()}
    if reason:
        out["cuda_unavailable_reason"] = reason
    return out


class HealthCache:
    """Latest device reading, refreshed every `interval_s` by a background task
    (health.rs: nvidia-smi every 5 s) so /health never blocks on nvidia-smi."""

    def __init__(self, interval_s: float = 5.0, probe=discover_devices):
        self.interval_s = interval_s
        self.probe = probe
        self.reading: dict = {"devices": [], "polled_at": None}

    def poll_once(self):
        try:
            r = self.probe()
            self.reading = {"devices": r.get("devices", []), "polled_at": time.time(),
                            **({"cuda_unavailable_reason": r["cuda_unavailable_reason"]}
                               if "cuda_unavailable_reason" in r else {})}
        except Exception:  # keep the last known reading
            pass

    async def run(self):
        import asyncio
        while True:
            await asyncio.to_thread(self.poll_once)
            await asyncio.sleep(self.interval_s)


def create_app(registry: ModelRegistry | None = None, default_models: list[dict] | None = None) -> FastAPI:
    reg = registry or ModelRegistry()
    app = FastAPI(title="helexa-b200 node")
    app.state.registry = reg
    app.state.activation = {"pending": [], "failed": {}, "ready": []}
    app.state.shutting_down = False
    app.state.health_cache = HealthCache(float(os.environ.get("HELEXA_HEALTH_POLL_S", "5")))

    @app.middleware("http")
    async def _refuse_while_shutting_down(request, call_next):
        # graceful shutdown (the reference's SHUTTING_DOWN flag): admission closes first,
        # in-flight requests finish, then every model unloads
        if app.state.shutting_down and request.url.path.startswith("/v1/"):
            return JSONResponse(wire.error_body("node is shutting down", "shutting_down"), 503,
                                headers={"Retry-After": "5"})
        return await call_next(request)

    @app.on_event("startup")
    async def _prewarm():
        import asyncio
        app.state.health_task = asyncio.get_running_loop().create_task(app.state.health_cache.run())

        async def load_defaults():
            for d in default_models or []:
                if app.state.shutting_down:
                    break
                spec = ModelSpec.from_dict(d)
                app.state.activation["pending"].append(spec.model_id)
                for attempt in range(3):
                    try:
                        await reg.load(spec)
                        app.state.activation["ready"].append(spec.model_id)
                        break
                    except Exception as e:  # retried with backoff (startup.rs:50)
                        app.state.activation["failed"][spec.model_id] = str(e)
                        await asyncio.sleep(2 ** attempt)
                app.state.activation["pending"].remove(spec.model_id)
        if default_models:
            asyncio.get_running_loop().create_task(load_defaults())

    @app.on_event("shutdown")
    async def _shutdown():
        app.state.shutting_down = True
        t = getattr(app.state, "health_task", None)
        if t is not None:
            t.cancel()
        await reg.unload_all()

    # ---- node surface ---------------------------------------------------------
    @app.get("/version")
    async def version():
        return build_info()

    @app.get("/discovery")
    async def discovery():
        return discover_devices()

    @app.get("/capabilities")
    async def capabilities_of_source(source: str):
        """Capabilities of an unloaded model directory, from its files alone."""
        from ..weights.loader import discover_capabilities
        path = source.split(":", 1)[1] if source.startswith("dir:") else source
        if not os.path.isdir(path):
            return _err(404, f"{path} is not a directory on this node", "not_found")
        return {"source": source, "capabilities": discover_capabilities(path)}

    @app.get("/health")
    async def health():
        models = {}
        for mid, m in reg.models.items():
            r = m.admission.rejections
            models[mid] = {"status": m.status, "in_flight": m.engine.in_flight,
                           "queue_depth": m.engine.queue_depth + m.admission.queue_depth,
                           "rejections": r.__dict__, "kv_budget_mb": m.admission.kv_budget_mb,
                           "kv_available_mb": m.admission.kv_available_mb(),
                           "prefill_tok_s": round(m.ema.prefill_tok_s, 1),
                           "decode_tok_s": round(m.ema.decode_tok_s, 1)}
        hc = app.state.health_cache.reading
        status = "unavailable" if "cuda_unavailable_reason" in hc else "ok"
        return {"status": status, "uptime_s": round(time.time() - START_TIME, 1), "models": models,
                "activation": app.state.activation, "devices": hc}

    @app.get("/models")
    async def models():
        return {"models": reg.list()}

    @app.get("/v1/models")
    async def v1_models():
        return {"object": "list", "data": [{"id": m["id"], "object": "model", "owned_by": "helexa",
                                            "created": int(START_TIME), "limit": m.get("limit")}
                                           for m in reg.list() if m.get("status") == "loaded"]}

    @app.post("/models/load")
    async def load(req: Request):
        body = await req.json()
        try:
            spec = ModelSpec.from_dict(body)
            m = await reg.load(spec)
        except LoadError as e:
            return _err(422, str(e) + (f" ({e.hint})" if e.hint else ""),
                        "model_load_failed" if e.code == "load_failed" else e.code)
        except (ValueError, FileNotFoundError, KeyError) as e:
            return _err(422, str(e), "model_load_failed")
        lim = getattr(m, "limits", None)
        return {"status": "loaded", "model_id": m.model_id, "limit": lim.__dict__ if lim is not None else None,
                "capabilities": m.capabilities}

    @app.post("/models/unload")
    async def unload(req: Request):
        body = await req.json()
        try:
            ok = await reg.unload(body["model_id"], force=bool(body.get("force", False)))
        except LoadError as e:
            return _err(409, str(e), "model_busy")
        if not ok:
            return _err(404, f"model {body['model_id']} is not loaded", "model_not_found")
        return {"status": "unloaded", "model_id": body["model_id"]}

    @app.get("/models/{model_id}/endpoint")
    async def endpoint(model_id: str, request: Request):
        if reg.get(model_id) is None:
            return _err(404, f"model {model_id} is not loaded", "model_not_found")
        return {"model_id": model_id, "base_url": str(request.base_url).rstrip("/") + "/v1"}

    @app.get("/models/{model_id}/capabilities")
    async def capabilities(model_id: str):
        m = reg.get(model_id)
        if m is None:
            return _err(404, f"model {model_id} is not loaded", "model_not_found")
        return {"model_id": model_id, "capabilities": m.capabilities, "tool_call": True, "reasoning": True,
                "limit": m.limits.__dict__}

    # ---- inference -------------------------------------------------------------
    def _model_for(body: dict):
        mid = body.get("model")
        m = reg.get(mid) if mid else (next(iter(reg.models.values())) if len(reg.models) == 1 else None)
        if m is None:
            raise RequestError(f"model {mid!r} is not loaded", 404, "model_not_found")
        if m.status == "poisoned":
            import asyncio
            asyncio.get_running_loop().create_task(reg.recover(m.model_id))
            raise RequestError(f"model {m.model_id} is recovering", 503, "model_recovering")
        return m

    def _principal(request: Request):
        return request.headers.get("x-helexa-account") or request.headers.get("x-helexa-key-id")

    def _include(request: Request) -> bool:
        return request.headers.get("x-include-thinking", "").lower() in ("1", "true", "yes")

    async def _run(request: Request, body: dict, kind: str):
        try:
            m = _model_for(body)
            if "max_completion_tokens" in body and "max_tokens" not in body:
                body["max_tokens"] = body["max_completion_tokens"]
            inc = _include(request)
            principal = _principal(request)
            prompt_ids = None
            if kind == "completions":
                prompt = body.get("prompt", "")
                prompt_ids = m.tokenizer.encode(prompt if isinstance(prompt, str) else "".join(prompt))
                if not prompt_ids:
                    raise RequestError("empty prompt")
            if body.get("stream"):
                gen = m.stream(body, principal, inc, prompt_ids)
                first = await gen.__anext__()  # admission / validation errors surface before the 200

                async def events():
                    yield first
                    async for ev in gen:
                        yield ev
                if kind == "chat":
                    body_iter = wire.chat_sse(events(), inc)
                elif kind == "completions":
                    body_iter = wire.completion_sse(events())
                elif kind == "responses":
                    body_iter = wire.responses_sse(events(), m.model_id)
                else:
                    body_iter = wire.anthropic_sse(events(), m.model_id, inc)
                return StreamingResponse(body_iter, media_type="text/event-stream",
                                         headers={"Cache-Control": "no-cache", "X-Accel-Buffering": "no"})
            start, text, reasoning, tools, fin = await m.complete(body, principal, inc, prompt_ids)
            if kind == "chat":
                return wire.chat_response(start, text, reasoning, tools, fin, inc)
            if kind == "completions":
                return {"id": start.id, "object": "text_completion", "created": start.created, "model": m.model_id,
                        "choices": [{"index": 0, "text": text, "finish_reason": fin.reason}],
                        "usage": wire.usage_obj(fin)}
            if kind == "responses":
                return wire.responses_object(m.model_id, text, tools, fin)
            return wire.anthropic_message(m.model_id, text, reasoning, tools, fin, inc)
        except AdmissionRejection as e:
            return _reject(e)
        except RequestError as e:
            return _err(e.status, str(e), e.code)
        except ValueError as e:
            return _err(400, str(e), "invalid_request_error")

    @app.post("/v1/chat/completions")
    async def chat(request: Request):
        return await _run(request, await request.json(), "chat")

    @app.post("/v1/completions")
    async def completions(request: Request):
        return await _run(request, await request.json(), "completions")

    @app.post("/v1/responses")
    async def responses(request: Request):
        body = await request.json()
        try:
            chat_body = wire.responses_to_chat(body)
        except ValueError as e:
            return _err(400, str(e), "unsupported_parameter")
        chat_body["model"] = body.get("model")
        return await _run(request, chat_body, "responses")

    @app.post("/v1/messages")
    async def messages(request: Request):
        body = await request.json()
        chat_body = wire.anthropic_to_openai(body)
        chat_body["model"] = body.get("model")
        return await _run(request, chat_body, "anthropic")

    @app.post("/v1/images/generations")
    async def images(request: Request):
        from ..runtime.image_serving import ImageRequestError
        body = await request.json()
        mid = body.get("model")
        im = reg.image_models.get(mid) if mid else (
            next(iter(reg.image_models.values())) if len(reg.image_models) == 1 else None)
        if im is None:
            if mid in reg.models:
                return _err(400, f"model {mid!r} does not generate images", "wrong_modality")
            return _err(404, f"image model {mid!r} is not loaded", "model_not_found")
        try:
            return await im.generate(body)
        except ImageRequestError as e:
            return _err(e.status, str(e), e.code)

    return app


def main():
    import argparse

    import uvicorn
    ap = argparse.ArgumentParser(description="helexa-b200 node")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=13131)
    ap.add_argument("--config", help="TOML/JSON config with default_models")
    args = ap.parse_args()
    from ..config.settings import load_settings
    from ..utils.trace import setup_logging
    settings = load_settings(args.config)
    setup_logging(settings.get("log"), settings.get("log_format"))
    app = create_app(default_models=settings.get("default_models", []))
    uvicorn.run(app, host=settings.get("host", args.host), port=int(settings.get("port", args.port)))


if __name__ == "__main__":
    main()
