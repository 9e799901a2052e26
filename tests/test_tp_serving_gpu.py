"""Tensor-parallel serving through the node API on 2 GPUs: `POST /models/load` with
`tensor_parallel: 2` spawns one rank process per GPU (NCCL + the fused peer-memory
reductions), and greedy chat completions through the HTTP app match the TP=1 load of
the same preset. Skipped where the box exposes fewer than 2 GPUs."""
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.timeout(900)
def test_tp2_http_matches_tp1(tmp_path):
    from fastapi.testclient import TestClient

    from helexa_b200.config import get_preset
    from helexa_b200.server.app import create_app
    from helexa_b200.weights.random_init import random_weights, save_safetensors
    from test_fast_model_gpu import _realistic
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    # unit-scale norms and decisive routing: plain N(0, 0.02) weights give near-tied
    # logits everywhere, where any change of bf16 summation order flips the arg-max
    cfg = get_preset("tiny-qwen3-next")
    torch.manual_seed(0)
    save_safetensors(_realistic(cfg, random_weights(cfg, seed=0, std=0.05)), cfg, str(tmp_path))
    body = {"messages": [{"role": "user", "content": "tell me a story about a robot"}], "max_tokens": 10,
            "temperature": 0}
    with TestClient(create_app()) as c:
        outs = {}
        for tp in (1, 2):
            mid = f"tp{tp}"
            r = c.post("/models/load", json={"model_id": mid, "source": str(tmp_path), "device": "cuda",
                                             "tensor_parallel": tp, "max_batch": 2, "max_len": 1024})
            assert r.status_code == 200, r.text
            j = c.post("/v1/chat/completions", json=dict(body, model=mid)).json()
            assert j["choices"][0]["finish_reason"] in ("length", "stop"), j
            outs[tp] = j["choices"][0]["message"]["content"]
            assert c.post("/models/unload", json={"model_id": mid}).status_code == 200
        # TP's different bf16 summation order may flip a near-tied step late in the
        # completion, so compare its opening
        assert outs[2][:4] == outs[1][:4], outs
