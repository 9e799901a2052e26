"""Speculative acceptance, context-limit derivation, preflight checks, settings."""
import pytest

from helexa_b200.config import get_preset
from helexa_b200.config.settings import load_settings
from helexa_b200.runtime.context_limit import ContextProfile, derive_limit, kv_reservation_mb
from helexa_b200.runtime.preflight import PreflightError, preflight
from helexa_b200.runtime.speculative import greedy_accept


def test_greedy_accept():
    a = greedy_accept([1, 2, 3, 4], [1, 2, 9, 4, 5])
    assert (a.accepted, a.bonus) == (2, 9) and a.committed([1, 2, 3, 4]) == [1, 2, 9]
    a = greedy_accept([1, 2], [1, 2, 7])
    assert a.committed([1, 2]) == [1, 2, 7]
    with pytest.raises(ValueError):
        greedy_accept([1], [1])


def test_context_limit():
    cfg = get_preset("qwen3-next-80b-a3b")
    p = ContextProfile.from_config(cfg)
    assert p.kv_bytes_per_token == 2 * 12 * 2 * 256 * 2   # only full-attention layers hold KV
    lim = derive_limit(p, free_bytes_tightest=20 << 30, prefill_tok_s=10000, max_prefill_s=1.0)
    assert lim.input == 10000 and lim.context <= cfg.max_position_embeddings and lim.kv_budget_mb > 0
    p8 = ContextProfile.from_config(cfg, tp=8)
    assert p8.kv_bytes_per_token == p.kv_bytes_per_token // 2   # 2 KV heads -> 1 per rank (replicated)
    assert kv_reservation_mb(p, 8192, 512) >= (8704 * p.kv_bytes_per_token) >> 20


def test_preflight():
    nxt = get_preset("qwen3-next-80b-a3b")
    preflight("dense", nxt, tp=8)                       # KV heads replicate at TP8
    with pytest.raises(PreflightError) as e:
        preflight("dense", nxt, tp=3)
    assert e.value.code == "bad_tensor_parallel"
    with pytest.raises(PreflightError) as e:
        preflight("diffusers", None)
    assert e.value.code == "wrong_modality"
    q32 = get_preset("qwen3-32b")
    preflight("gguf", q32, tp=4, quant="Q4_K")
    preflight("gguf", q32, tp=8, quant="Q4_K_M")     # uneven superblock split of down_proj
    tiny = get_preset("tiny-qwen3")
    with pytest.raises(PreflightError) as e:
        preflight("gguf", tiny, tp=4, quant="Q4_K")   # fewer superblocks than ranks
    assert e.value.code == "quant_shard_misaligned"
    with pytest.raises(PreflightError) as e:
        preflight("dense", nxt, tp=1, free_bytes_per_device=[80 << 30])
    assert e.value.code == "insufficient_memory" and "error" in e.value.to_json()


def test_settings_env_override(tmp_path):
    f = tmp_path / "c.json"
    f.write_text('{"port": 1, "admission": {"max_in_flight": 2}}')
    s = load_settings(str(f), env={"HELEXA_PORT": "8080", "HELEXA_ADMISSION__MAX_QUEUE_DEPTH": "9",
                                   "OTHER": "x"})
    assert s == {"port": 8080, "admission": {"max_in_flight": 2, "max_queue_depth": 9}}


def test_tp_smoke_cli_gloo():
    """The TP smoke check spawns ranks, pings them and verifies a sanity all-reduce."""
    from helexa_b200.parallel.smoke import run
    ok, line = run(2, cpu=True, timeout_s=120)
    assert ok, line
    assert line.startswith("status=ok ranks=2 backend=gloo")


def test_node_refuses_requests_while_shutting_down():
    from fastapi.testclient import TestClient
    from helexa_b200.server.app import create_app
    app = create_app()
    with TestClient(app) as c:
        app.state.shutting_down = True
        r = c.post("/v1/chat/completions", json={"model": "x", "messages": []})
        assert r.status_code == 503 and r.headers.get("retry-after") == "5"
        assert c.get("/version").status_code == 200


def test_capability_discovery_from_files(tmp_path):
    import json
    from helexa_b200.weights.loader import discover_capabilities
    text = tmp_path / "text"
    text.mkdir()
    (text / "config.json").write_text(json.dumps({"model_type": "qwen3"}))
    (text / "model.safetensors").write_bytes(b"")
    assert discover_capabilities(str(text)) == ["chat", "completion"]
    vis = tmp_path / "vis"
    vis.mkdir()
    (vis / "config.json").write_text(json.dumps({"model_type": "qwen3_5", "vision_config": {}}))
    assert "vision" in discover_capabilities(str(vis))
    img = tmp_path / "img"
    img.mkdir()
    (img / "model_index.json").write_text("{}")
    assert discover_capabilities(str(img)) == ["image"]


def test_capabilities_endpoint(tmp_path):
    from fastapi.testclient import TestClient
    from helexa_b200.server.app import create_app
    (tmp_path / "model_index.json").write_text("{}")
    with TestClient(create_app()) as c:
        assert c.get("/capabilities", params={"source": str(tmp_path)}).json()["capabilities"] == ["image"]
        assert c.get("/capabilities", params={"source": str(tmp_path / "nope")}).status_code == 404


def test_device_discovery_driver_mismatch_and_health_cache():
    """A failing nvidia-smi with the driver/library mismatch message becomes an
    operator-facing reason (userspace NVML version vs the loaded kernel module); a normal
    run parses the inventory; the health cache keeps the last reading."""
    import subprocess as sp

    from helexa_b200.server.app import HealthCache, classify_driver_mismatch, discover_devices
    msg = "Failed to initialize NVML: Driver/library version mismatch\nNVML library version: 580.159\n"
    assert classify_driver_mismatch(msg) == "580.159"
    assert classify_driver_mismatch("No devices were found") is None
    bad = lambda cmd: sp.CompletedProcess(cmd, 18, stdout=msg, stderr="")  # noqa: E731
    proc = "NVRM version: NVIDIA UNIX Open Kernel Module for x86_64  580.126.09  Release Build\n"
    d = discover_devices(run=bad, proc_version=proc)
    assert d["devices"] == [] and "580.159" in d["cuda_unavailable_reason"]
    assert "580.126.09" in d["cuda_unavailable_reason"]
    ok = lambda cmd: sp.CompletedProcess(cmd, 0, stdout="0, NVIDIA B200, 183359, 180000, 580.159, 10.0, 31, 0, 140.5\n",
                                         stderr="")  # noqa: E731
    d = discover_devices(run=ok)
    assert d["driver_version"] == "580.159" and d["devices"][0]["memory_free_mb"] == 180000
    assert d["devices"][0]["power_w"] == 140.5
    calls = []
    hc = HealthCache(probe=lambda: calls.append(1) or discover_devices(run=ok))
    hc.poll_once()
    assert hc.reading["devices"][0]["name"] == "NVIDIA B200" and hc.reading["polled_at"]
    hc.probe = lambda: (_ for _ in ()).throw(RuntimeError("smi hung"))
    hc.poll_once()  # a failed poll keeps the last known reading
    assert hc.reading["devices"][0]["name"] == "NVIDIA B200"


def test_structured_logging_and_spans(capsys):
    import json as _json

    from helexa_b200.utils.trace import request_span, setup_logging, span
    log = setup_logging("DEBUG", "json")
    with span("unit.work", items=3):
        pass
    request_span("req-1", "m", None, 10, 4, 5, 12.5, 40.0, "stop")
    lines = [_json.loads(x) for x in capsys.readouterr().err.strip().splitlines()]
    assert lines[0]["span"] == "unit.work" and lines[0]["items"] == 3 and lines[0]["ms"] >= 0
    assert lines[1]["request_id"] == "req-1" and lines[1]["cached_tokens"] == 4 and lines[1]["principal"] == "anonymous"
    setup_logging("WARNING", "text")
    assert log.level == 30
