"""Image inputs end to end on the CPU: chat content parts -> preprocessing -> vision
tower -> pad expansion + M-RoPE positions -> one embedding prefill in the engine ->
decode at the shifted rotary position; and the HTTP route that carries them."""
import base64
import io

import pytest
import torch
from fastapi.testclient import TestClient

from helexa_b200.config import get_preset


def _png(w=20, h=28, seed=0) -> str:
    from PIL import Image
    g = torch.Generator().manual_seed(seed)
    arr = (torch.rand(h, w, 3, generator=g) * 255).to(torch.uint8).numpy()
    buf = io.BytesIO()
    Image.fromarray(arr).save(buf, format="PNG")
    return "data:image/png;base64," + base64.b64encode(buf.getvalue()).decode()


def _messages(uri):
    return [{"role": "user", "content": [{"type": "text", "text": "describe "},
                                         {"type": "image_url", "image_url": {"url": uri}},
                                         {"type": "text", "text": " briefly"}]}]


def test_frontend_expands_pads_and_engine_matches_reference():
    from helexa_b200.models.reference import ReferenceModel
    from helexa_b200.runtime.engine import Engine
    from helexa_b200.runtime.multimodal import VisionFrontend, request_images
    from helexa_b200.runtime.runner import RefRunner
    from helexa_b200.runtime.sampling import SamplingParams
    from helexa_b200.runtime.tokenizer import ByteTokenizer
    from helexa_b200.weights.random_init import random_weights
    cfg = get_preset("tiny-qwen3-vl")
    w = random_weights(cfg, seed=0, std=0.05)
    tok = ByteTokenizer(cfg.vocab_size)
    fe = VisionFrontend.from_weights(cfg, w.__getitem__, w["model.embed_tokens.weight"], tok)
    uri = _png()
    ids = tok.encode(tok.apply_chat_template(_messages(uri)))
    pad = tok.token_id("<|image_pad|>")
    assert ids.count(pad) == 1 and request_images(_messages(uri)) == [uri]
    mm = fe.build(ids, [uri])
    # 20 x 28 px is below the 64-token floor: resized to a multiple of 8 px with >= 64 merged tokens
    n_img = mm.tokens.count(pad)
    assert n_img >= 64 and len(mm.tokens) == len(ids) - 1 + n_img == mm.embeds.shape[0]
    assert mm.pos3.shape == (3, len(mm.tokens)) and mm.next_pos < len(mm.tokens)

    # the oracle: the reference model fed the same embeddings, greedy
    ref = ReferenceModel(cfg, w)
    st = ref.new_state()
    lg = ref.forward(None, st, embeds=mm.embeds, pos3=mm.pos3, next_pos=mm.next_pos)
    want = [int(lg.argmax())]
    for _ in range(5):
        want.append(int(ref.forward(torch.tensor([want[-1]]), st).argmax()))

    eng = Engine(RefRunner(ReferenceModel(cfg, w), num_slots=2, max_len=512), max_batch=2)
    try:
        got, fin = eng.generate(mm.tokens, SamplingParams(max_tokens=6, temperature=0.0, repeat_penalty=1.0), mm=mm)
    finally:
        eng.shutdown()
    assert got == want and fin.prompt_tokens == len(mm.tokens)


def test_mismatched_placeholders_are_refused():
    from helexa_b200.runtime.multimodal import VisionFrontend
    from helexa_b200.runtime.tokenizer import ByteTokenizer
    from helexa_b200.weights.random_init import random_weights
    cfg = get_preset("tiny-qwen3-vl")
    w = random_weights(cfg, seed=0)
    tok = ByteTokenizer(cfg.vocab_size)
    fe = VisionFrontend.from_weights(cfg, w.__getitem__, w["model.embed_tokens.weight"], tok)
    with pytest.raises(ValueError):
        fe.build(tok.encode("no placeholder"), [_png()])
    with pytest.raises(ValueError):
        fe.build(tok.encode("<|image_pad|>"), ["https://example.com/cat.png"])


def test_http_chat_with_image():
    from helexa_b200.server.app import create_app
    app = create_app()
    with TestClient(app) as c:
        for mid, src in (("vl", "preset:tiny-qwen3-vl"), ("text", "preset:tiny-qwen3")):
            r = c.post("/models/load", json={"model_id": mid, "source": src, "device": "cpu", "max_batch": 2,
                                             "max_len": 512})
            assert r.status_code == 200, r.text
        caps = {m["id"]: m for m in c.get("/models").json()["models"]}
        body = {"model": "vl", "messages": _messages(_png()), "max_tokens": 4, "temperature": 0}
        r = c.post("/v1/chat/completions", json=body)
        assert r.status_code == 200, r.text
        u = r.json()["usage"]
        assert u["prompt_tokens"] > 64 and u["completion_tokens"] <= 4
        body["model"] = "text"
        r = c.post("/v1/chat/completions", json=body)
        assert r.status_code == 400 and "image" in r.text
        assert "vl" in caps
