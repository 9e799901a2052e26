"""Vision-language path on the GPU: the vision tower with the tcgen05 GEMM against its
fp32 CPU run, and a multimodal prefill (image tokens spliced in, M-RoPE positions)
plus decode with the rotary offset on the CUDA model against the fp32 reference."""
import dataclasses

import pytest
import torch

pytestmark = pytest.mark.gpu


def _cos(a, b):
    return torch.nn.functional.cosine_similarity(a.float().flatten().cpu(), b.float().flatten().cpu(), dim=0).item()


def test_vision_tower_cuda_matches_cpu():
    from helexa_b200.models.vision import VisionConfig, VisionTower, random_vision_weights
    vc = VisionConfig(depth=2, hidden_size=128, intermediate_size=256, num_heads=2, num_position_embeddings=64,
                      out_hidden_size=256, patch_size=8)
    w = random_vision_weights(vc, seed=4, std=0.05)
    img = torch.rand(3, 64, 96) * 2 - 1
    a = VisionTower(vc, w).forward(img)
    b = VisionTower(vc, w, device="cuda").forward(img)
    assert b.shape == a.shape and _cos(a, b) > 0.995


def test_multimodal_prefill_and_decode_match_reference():
    from helexa_b200.config import get_preset
    from helexa_b200.models.fast import FastModel
    from helexa_b200.models.reference import ReferenceModel
    from helexa_b200.models.vision import VisionTower, random_vision_weights, tiny_vision_config
    from helexa_b200.models.vlm import VisionLanguage
    from helexa_b200.weights.random_init import random_weights
    from test_fast_model_gpu import _realistic
    cfg = dataclasses.replace(get_preset("tiny-qwen3"), mrope_section=[11, 11, 10], mrope_interleaved=True)
    torch.manual_seed(0)
    w = _realistic(cfg, random_weights(cfg, seed=0, std=0.05))
    ref = ReferenceModel(cfg, w)
    fm = FastModel.from_hf(cfg, w, "cuda", max_slots=2, max_len=256)
    vc = tiny_vision_config(out_hidden=cfg.hidden_size)
    tower = VisionTower(vc, random_vision_weights(vc, seed=2, std=0.05))
    vl = VisionLanguage(ref.w["model.embed_tokens.weight"], tower)
    img = torch.rand(3, 24, 32) * 2 - 1                            # 3 x 4 LM tokens
    g = torch.Generator().manual_seed(1)
    t1 = torch.randint(0, cfg.vocab_size, (10,), generator=g).tolist()
    t2 = torch.randint(0, cfg.vocab_size, (7,), generator=g).tolist()
    emb, pos3, nxt = vl.build([("text", t1), ("image", img), ("text", t2)])
    st = ref.new_state()
    want = ref.forward(None, st, embeds=emb, pos3=pos3, next_pos=nxt)
    got = fm.prefill(0, None, 0, embeds=emb.cuda(), pos3=pos3, next_pos=nxt)
    assert _cos(got, want) > 0.995
    assert st.rope_delta < 0 and fm._rope_delta_host[0] == st.rope_delta
    nb = fm.buffers(1)
    nb.slots.fill_(0)
    tok = int(want.argmax())
    for _ in range(4):  # teacher-forced decode: the rotary offset applies in decode attention
        nb.tok.fill_(tok)
        fm.decode_step_launch(nb)
        wl = ref.forward(torch.tensor([tok]), st)
        assert _cos(nb.logits[0], wl) > 0.995
        tok = int(wl.argmax())


def test_cuda_served_chat_with_image():
    """The node serves an image chat on CUDA: registry builds the tower beside the
    FastModel, the engine prefills the spliced embeddings through FastRunner.prefill_mm
    and decodes in captured graphs at the shifted rotary position."""
    from fastapi.testclient import TestClient
    from helexa_b200.server.app import create_app
    from test_multimodal_cpu import _messages, _png
    with TestClient(create_app()) as c:
        r = c.post("/models/load", json={"model_id": "vl", "source": "preset:tiny-qwen3-vl", "device": "cuda",
                                         "max_batch": 2, "max_len": 512})
        assert r.status_code == 200, r.text
        body = {"model": "vl", "messages": _messages(_png()), "max_tokens": 6, "temperature": 0}
        r = c.post("/v1/chat/completions", json=body)
        assert r.status_code == 200, r.text
        u = r.json()["usage"]
        assert u["prompt_tokens"] > 64 and 1 <= u["completion_tokens"] <= 6
