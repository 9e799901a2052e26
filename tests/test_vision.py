"""Vision tower, image preprocessing and M-RoPE on CPU: the tower against HF
transformers' Qwen3VLVisionModel on the same random weights (fp32), smart_resize and
data-URI decoding, and the multimodal rotary position ids / axis maps."""
import base64
import io

import pytest
import torch

from helexa_b200.models.vision import VisionTower, patchify, random_vision_weights, tiny_vision_config


def test_vision_tower_matches_hf():
    from transformers.models.qwen3_vl.configuration_qwen3_vl import Qwen3VLVisionConfig
    from transformers.models.qwen3_vl.modeling_qwen3_vl import Qwen3VLVisionModel
    vc = tiny_vision_config(out_hidden=96)
    w = random_vision_weights(vc, seed=3, std=0.05)
    hcfg = Qwen3VLVisionConfig(depth=vc.depth, hidden_size=vc.hidden_size, hidden_act=vc.hidden_act,
                               intermediate_size=vc.intermediate_size, num_heads=vc.num_heads,
                               in_channels=vc.in_channels, patch_size=vc.patch_size,
                               spatial_merge_size=vc.spatial_merge_size, temporal_patch_size=vc.temporal_patch_size,
                               out_hidden_size=vc.out_hidden_size, num_position_embeddings=vc.num_position_embeddings,
                               deepstack_visual_indexes=[])
    hcfg._attn_implementation = "eager"
    hf = Qwen3VLVisionModel(hcfg).eval()
    sd = {k[len("model.visual."):]: v for k, v in w.items()}
    missing, unexpected = hf.load_state_dict(sd, strict=False)
    assert not unexpected and not [m for m in missing if "deepstack" not in m], (missing, unexpected)
    torch.manual_seed(0)
    img = torch.rand(3, 24, 40) * 2 - 1          # 6 x 10 patches -> 3 x 5 LM tokens
    patches, grid = patchify(img, vc)
    with torch.no_grad():
        out = hf(patches, torch.tensor([grid]))
    want = out.pooler_output if hasattr(out, "pooler_output") else out[0]
    got = VisionTower(vc, w).forward(img)
    assert got.shape == (15, 96)
    torch.testing.assert_close(got, want, atol=2e-5, rtol=1e-4)


def test_smart_resize_and_preprocess():
    from PIL import Image

    from helexa_b200.runtime.preprocess import PreprocessProfile, decode_image, preprocess, smart_resize
    assert smart_resize(448, 448, 32, 64 * 32 * 32, 1024 * 32 * 32) == (448, 448)
    h, w = smart_resize(1000, 3000, 32, 4 * 32 * 32, 256 * 32 * 32)
    assert h % 32 == 0 and w % 32 == 0 and h * w <= 256 * 32 * 32 and abs(w / h - 3) < 0.35
    h, w = smart_resize(10, 12, 32, 16 * 32 * 32, 1024 * 32 * 32)
    assert h * w >= 16 * 32 * 32
    im = Image.new("RGB", (50, 30), (255, 0, 128))
    buf = io.BytesIO()
    im.save(buf, format="PNG")
    uri = "data:image/png;base64," + base64.b64encode(buf.getvalue()).decode()
    prof = PreprocessProfile(factor=32, min_pixels=32 * 32, max_pixels=64 * 32 * 32)
    x = preprocess(decode_image(uri), prof)
    assert x.shape[0] == 3 and x.shape[1] % 32 == 0 and x.shape[2] % 32 == 0
    assert torch.allclose(x[0], torch.ones_like(x[0])) and torch.allclose(x[1], -torch.ones_like(x[1]))
    with pytest.raises(ValueError):
        decode_image("https://example.com/x.png")


def test_mrope_positions_and_axes():
    from helexa_b200.models.mrope import mrope_axis_map, mrope_positions
    ax = mrope_axis_map(32, [11, 11, 10], interleaved=True)
    assert ax[0] == 0 and ax[1] == 1 and ax[2] == 2 and ax[3] == 0 and (ax == 1).sum() == 11 and (ax == 2).sum() == 10
    ax2 = mrope_axis_map(32, [16, 8, 8], interleaved=False)
    assert (ax2[:16] == 0).all() and (ax2[16:24] == 1).all() and (ax2[24:] == 2).all()
    # text only: the three axes carry the same running position
    pos, nxt = mrope_positions([("text", 5)])
    assert pos.tolist() == [[0, 1, 2, 3, 4]] * 3 and nxt == 5
    # text, a 2 x 3 image, text: the image shares its start position in t and spans h / w
    pos, nxt = mrope_positions([("text", 2), ("image", 2, 3), ("text", 2)])
    t, h, w = pos.tolist()
    assert t[:2] == [0, 1] and t[2:8] == [2] * 6 and h[2:8] == [2, 2, 2, 3, 3, 3] and w[2:8] == [2, 3, 4] * 2
    assert t[8:] == [5, 6] and h[8:] == [5, 6] and nxt == 7


def _vl_cfg():
    import dataclasses

    from helexa_b200.config import get_preset
    c = get_preset("tiny-qwen3")
    return dataclasses.replace(c, mrope_section=[11, 11, 10], mrope_interleaved=True)


def test_reference_mrope_text_only_equals_plain_rope():
    from helexa_b200.models.mrope import mrope_positions
    from helexa_b200.models.reference import ReferenceModel
    from helexa_b200.weights.random_init import random_weights
    cfg = _vl_cfg()
    m = ReferenceModel(cfg, random_weights(cfg, seed=1))
    toks = torch.randint(0, cfg.vocab_size, (20,), generator=torch.Generator().manual_seed(0))
    a = m.forward(toks, m.new_state())
    pos, nxt = mrope_positions([("text", 20)])
    st = m.new_state()
    b = m.forward(None, st, embeds=m.w["model.embed_tokens.weight"][toks], pos3=pos, next_pos=nxt)
    torch.testing.assert_close(a, b, atol=1e-5, rtol=1e-5)
    assert st.rope_delta == 0


def test_vision_language_prefill_on_reference():
    """An image between text runs: the image tokens share rotary positions, so decode
    continues at a rotary position behind the cache length (rope_delta < 0)."""
    from helexa_b200.models.reference import ReferenceModel
    from helexa_b200.models.vlm import VisionLanguage
    from helexa_b200.weights.random_init import random_weights
    cfg = _vl_cfg()
    m = ReferenceModel(cfg, random_weights(cfg, seed=1))
    vc = tiny_vision_config(out_hidden=cfg.hidden_size)
    tower = VisionTower(vc, random_vision_weights(vc, seed=2))
    vl = VisionLanguage(m.w["model.embed_tokens.weight"], tower)
    img = torch.rand(3, 16, 24) * 2 - 1                       # 2 x 3 LM tokens
    emb, pos3, nxt = vl.build([("text", [1, 2, 3]), ("image", img), ("text", [4, 5])])
    assert emb.shape == (11, cfg.hidden_size) and nxt == 3 + 3 + 2
    st = m.new_state()
    lg = m.forward(None, st, embeds=emb, pos3=pos3, next_pos=nxt)
    assert torch.isfinite(lg).all() and st.length == 11 and st.rope_delta == nxt - 11
