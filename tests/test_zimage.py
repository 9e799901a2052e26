"""Z-Image pipeline: request helpers, sampler, tiling, PNG, and the DiT / VAE / pipeline
on tiny configs (CPU fp32), plus the GPU DiT against the fp32 oracle.

Mirrors the reference's unit tests of harness/image.rs:578-652 (dims, steps, prompt
wrapping, megapixel-steps, layout / class detection, PNG round trip)."""
import math

import pytest
import torch

from helexa_b200.config import get_preset
from helexa_b200.models import zimage as zi
from helexa_b200.models.reference import ReferenceModel
from helexa_b200.weights.random_init import random_weights as lm_random_weights


def test_validate_dims_and_steps():
    assert zi.validate_dims(1024, 768) == (96, 128)
    for bad in ((0, 64), (1000, 1024), (4096, 1024)):
        with pytest.raises(ValueError):
            zi.validate_dims(*bad)
    assert zi.validate_steps(9) == 9
    for bad in (0, 51):
        with pytest.raises(ValueError):
            zi.validate_steps(bad)


def test_prompt_size_units_layout():
    assert zi.format_prompt("a cat") == "<|im_start|>user\na cat<|im_end|>\n<|im_start|>assistant\n"
    assert zi.parse_size(None) == (1024, 1024)
    assert zi.parse_size("512x768") == (512, 768)
    assert zi.parse_size("2048X1024") == (2048, 1024)
    for bad in ("1024", "axb", "1024x"):
        with pytest.raises(ValueError):
            zi.parse_size(bad)
    assert math.isclose(zi.megapixel_steps(1000, 1000, 9, False), 9.0)
    assert math.isclose(zi.megapixel_steps(1000, 1000, 9, True), 18.0)
    assert zi.is_diffusers_layout(["model_index.json", "vae/config.json"])
    assert not zi.is_diffusers_layout(["config.json"])
    assert zi.is_supported_pipeline_class('{"_class_name": "ZImagePipeline"}')
    assert not zi.is_supported_pipeline_class('{"_class_name": "FluxPipeline"}')
    assert not zi.is_supported_pipeline_class("not json")


def test_image_quant_parse():
    assert zi.parse_image_quant("q8_0") == "Q8_0" and zi.parse_image_quant("Q8") == "Q8_0"
    for bad in ("q4_k", "fp8", ""):
        with pytest.raises(ValueError):
            zi.parse_image_quant(bad)


def test_png_roundtrip():
    g = torch.Generator().manual_seed(0)
    rgb = torch.randint(0, 256, (5, 7, 3), generator=g, dtype=torch.uint8)
    png = zi.encode_png(rgb, 7, 5)
    assert png[:8] == b"\x89PNG\r\n\x1a\n"
    w, h, raw = zi.decode_png(png)
    assert (w, h) == (7, 5) and raw == rgb.numpy().tobytes()
    with pytest.raises(ValueError):
        zi.encode_png(rgb, 8, 5)


def test_sampler_grid():
    mu = zi.calculate_shift(256)
    assert math.isclose(mu, zi.BASE_SHIFT) and math.isclose(zi.calculate_shift(4096), zi.MAX_SHIFT)
    s = zi.FlowMatchEuler(9, zi.calculate_shift(4096))
    assert len(s) == 9 and s.sigmas[0] == 1.0 and s.sigmas[-1] == 0.0 and s.sigmas[-2] == 0.0
    assert all(a >= b for a, b in zip(s.sigmas, s.sigmas[1:]))
    # the shift moves mass toward high noise: every interior sigma is above the linear grid
    lin = torch.linspace(1, 0, 9).tolist()
    assert all(a > b for a, b in zip(s.sigmas[1:-2], lin[1:-1]))
    x = torch.zeros(4)
    v = torch.ones(4)
    x1 = s.step(v, x)
    assert torch.allclose(x1, torch.full((4,), s.sigmas[1] - 1.0))


def test_patchify_roundtrip_and_positions():
    lat = torch.randn(16, 8, 12)
    tok, grid = zi.patchify(lat, 2)
    assert tok.shape == (24, 64) and grid == (4, 6)
    assert torch.equal(zi.unpatchify(tok, grid, 2, 16), lat)
    # token (r, c) holds latent[:, 2r:2r+2, 2c:2c+2] ordered (py, px, ch)
    assert torch.equal(tok[1 * 6 + 2].view(2, 2, 16).permute(2, 0, 1), lat[:, 2:4, 4:6])
    img, cap = zi.positions(5, grid, "cpu")
    assert cap[:, 0].tolist() == [1, 2, 3, 4, 5] and cap[:, 1:].abs().sum() == 0
    assert (img[:, 0] == 33).all()  # padded caption length 32, + 1
    assert img[7].tolist() == [33, 1, 1]


class _PointVae:
    factor = 8

    def decode(self, z):
        return z[:, :3].repeat_interleave(8, 2).repeat_interleave(8, 3)


def test_tiled_decode_blends_to_the_full_decode():
    assert zi.tile_positions(100, 64, 16) == [0, 36]
    assert zi.tile_positions(150, 64, 16) == [0, 48, 86]
    assert zi.tile_positions(64, 64, 16) == [0]
    z = torch.randn(1, 16, 40, 50)
    full = _PointVae().decode(z)
    tiled = zi.tiled_decode(_PointVae(), z, tile=16, overlap=4)
    assert tiled.shape == full.shape
    assert torch.allclose(tiled, full, atol=1e-5)


def _tiny_pipeline(device="cpu"):
    lm_cfg = get_preset("tiny-qwen3")
    te = zi.TextEncoder(ReferenceModel(lm_cfg, lm_random_weights(lm_cfg, seed=1)))
    dcfg = zi.tiny_dit_config(cap_feat_dim=lm_cfg.hidden_size)
    dw = zi.random_weights(zi.dit_weight_shapes(dcfg), seed=2, std=0.05)
    vcfg = zi.tiny_vae_config()
    vw = zi.random_weights(zi.vae_decoder_shapes(vcfg), seed=3, std=0.05)
    dit = zi.ZImageDiT(dcfg, dw, device)
    vae = zi.VaeDecoder(vcfg, vw, device if device == "cpu" else device)
    return zi.ZImagePipeline(dit, vae, te, tile=8, overlap=2), (dcfg, dw, lm_cfg)


def test_dit_forward_shapes_and_conditioning():
    pipe, (dcfg, dw, _) = _tiny_pipeline()
    lat = torch.randn(16, 8, 8)
    cap = torch.randn(6, dcfg.cap_feat_dim)
    y = pipe.dit.forward(lat, 0.3, cap)
    assert y.shape == lat.shape and torch.isfinite(y).all()
    # timestep and caption both condition the output
    assert not torch.allclose(y, pipe.dit.forward(lat, 0.7, cap))
    assert not torch.allclose(y, pipe.dit.forward(lat, 0.3, cap[:4]))


def test_pipeline_generates_deterministic_image():
    pipe, _ = _tiny_pipeline()
    toks = [5, 17, 99, 3]
    a = pipe.generate(toks, width=32, height=48, steps=3, seed=7)
    b = pipe.generate(toks, width=32, height=48, steps=3, seed=7)
    assert a.rgb.shape == (48, 32, 3) and a.rgb.dtype == torch.uint8
    assert torch.equal(a.rgb, b.rgb)
    assert a.timing.steps == 3 and not a.timing.cfg
    c = pipe.generate(toks, width=32, height=48, steps=3, seed=7, negative_prompt=[1, 2], guidance_scale=4.0)
    assert c.timing.cfg
    png = zi.encode_png(a.rgb, 32, 48)
    assert zi.decode_png(png)[2] == a.rgb.numpy().tobytes()
    # latents 4x6 decode through tiles of 8 latents with 2 overlap (two tiles each way
    # at 8x upsampling would need > 8 latents; force tiling with a smaller tile)
    pipe.tile, pipe.overlap = 2, 1
    d = pipe.generate(toks, width=32, height=48, steps=2, seed=7)
    assert d.rgb.shape == (48, 32, 3)


@pytest.mark.gpu
def test_dit_ops_match_torch():
    from helexa_b200 import ops
    C = ops.C
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    T, D, H, Dh = 300, 192, 3, 64
    x = torch.randn(T, D, device=dev, generator=g).bfloat16()
    w = torch.rand(D, device=dev, generator=g) + 0.5
    sc = torch.randn(D, device=dev, generator=g) * 0.1
    y = torch.empty_like(x)
    C.dit_norm_mod(x, w, sc, y, 1e-5)
    ref = zi._rms(x.float(), w, 1e-5) * (1 + sc)
    assert (y.float() - ref).abs().max() < 0.05
    o = torch.randn(T, D, device=dev, generator=g).bfloat16()
    gate = torch.tanh(torch.randn(D, device=dev, generator=g))
    x2 = x.clone()
    C.dit_gate_res(x2, o, w, gate, 1e-5)
    ref = x.float() + zi._rms(o.float(), w, 1e-5) * gate
    assert (x2.float() - ref).abs().max() < 0.05
    qkv = torch.randn(T, 3 * H * Dh, device=dev, generator=g).bfloat16()
    qw = torch.rand(Dh, device=dev, generator=g) + 0.5
    kw = torch.rand(Dh, device=dev, generator=g) + 0.5
    ang = torch.rand(T, Dh // 2, device=dev, generator=g) * 20
    q = torch.empty(T, H * Dh, dtype=torch.bfloat16, device=dev)
    k = torch.empty(H, T, Dh, dtype=torch.bfloat16, device=dev)
    v = torch.empty_like(k)
    C.dit_qk_rope(qkv, qw, kw, ang, H, Dh, 1e-5, q, k, v)
    qf, kf, vf = qkv.float().view(T, 3, H, Dh).unbind(1)
    rq = zi._rope_torch(zi._rms(qf, qw, 1e-5), ang)
    rk = zi._rope_torch(zi._rms(kf, kw, 1e-5), ang)
    assert (q.float().view(T, H, Dh) - rq).abs().max() < 0.05
    assert (k.float().transpose(0, 1) - rk).abs().max() < 0.05
    assert torch.equal(v.transpose(0, 1), qkv.view(T, 3, H, Dh)[:, 2])


@pytest.mark.gpu
@pytest.mark.parametrize("D", [64, 128])
def test_bidirectional_attention_kernel(D):
    from helexa_b200 import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(1)
    T, H = 333, 2
    q = torch.randn(T, H * D, device=dev, generator=g).bfloat16()
    k = torch.randn(H, T, D, device=dev, generator=g).bfloat16()
    v = torch.randn(H, T, D, device=dev, generator=g).bfloat16()
    o = torch.empty(T, H * D, dtype=torch.bfloat16, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ops.C.attn_prefill_tc(q, k, v, o, H, 0, D ** -0.5, None, 0, err, causal=False)
    torch.cuda.synchronize()
    assert err.item() == 0
    ref = torch.nn.functional.scaled_dot_product_attention(q.float().view(T, H, D).transpose(0, 1), k.float(), v.float())
    ref = ref.transpose(0, 1).reshape(T, H * D)
    assert (o.float() - ref).abs().max() < 0.03


@pytest.mark.gpu
def test_dit_gpu_matches_fp32_oracle():
    dev = torch.device("cuda", 0)
    dcfg = zi.tiny_dit_config(cap_feat_dim=256)
    dw = zi.random_weights(zi.dit_weight_shapes(dcfg), seed=2, std=0.05)
    cpu = zi.ZImageDiT(dcfg, dw, "cpu")
    gpu = zi.ZImageDiT(dcfg, dw, dev)
    g = torch.Generator().manual_seed(3)
    lat = torch.randn(16, 24, 20, generator=g)
    cap = torch.randn(37, 256, generator=g)
    for t in (0.1, 0.8):
        a = cpu.forward(lat, t, cap)
        b = gpu.forward(lat, t, cap).float().cpu()
        cos = torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0).item()
        assert cos > 0.995, cos
    assert gpu.err.item() == 0


@pytest.mark.gpu
def test_quantized_dit_tracks_bf16():
    dev = torch.device("cuda", 0)
    dcfg = zi.tiny_dit_config(cap_feat_dim=256)
    dw = zi.random_weights(zi.dit_weight_shapes(dcfg), seed=2, std=0.05)
    a = zi.ZImageDiT(dcfg, dw, dev)
    b = zi.ZImageDiT(dcfg, dw, dev)
    b.quantize_("q8_0")
    g = torch.Generator().manual_seed(4)
    lat, cap = torch.randn(16, 16, 16, generator=g), torch.randn(9, 256, generator=g)
    ya, yb = a.forward(lat, 0.5, cap).float(), b.forward(lat, 0.5, cap).float()
    assert torch.nn.functional.cosine_similarity(ya.flatten(), yb.flatten(), dim=0).item() > 0.995


@pytest.mark.gpu
def test_pipeline_on_gpu():
    pipe, _ = _tiny_pipeline(torch.device("cuda", 0))
    r = pipe.generate([5, 17, 99, 3], width=64, height=64, steps=3, seed=1)
    assert r.rgb.shape == (64, 64, 3)


def test_images_api_on_cpu():
    import base64

    from fastapi.testclient import TestClient

    from helexa_b200.server.app import create_app
    with TestClient(create_app()) as c:
        r = c.post("/models/load", json={"model_id": "zimg", "source": "preset:tiny-z-image", "device": "cpu"})
        assert r.status_code == 200, r.text
        assert r.json()["capabilities"] == ["image"]
        ms = {m["id"]: m for m in c.get("/models").json()["models"]}
        assert ms["zimg"]["capabilities"] == ["image"]
        body = {"model": "zimg", "prompt": "a red cube", "size": "32x48", "num_steps": 2, "seed": 3}
        r = c.post("/v1/images/generations", json=body)
        assert r.status_code == 200, r.text
        j = r.json()
        w, h, raw = zi.decode_png(base64.b64decode(j["data"][0]["b64_json"]))
        assert (w, h) == (32, 48) and len(raw) == 32 * 48 * 3
        assert math.isclose(j["usage"]["helexa_image_units"], zi.megapixel_steps(32, 48, 2, False))
        assert j["usage"]["helexa_timing"]["steps"] == 2
        # same seed, same image
        r2 = c.post("/v1/images/generations", json=body)
        assert r2.json()["data"][0]["b64_json"] == j["data"][0]["b64_json"]
        for bad, code in (({"n": 2}, "unsupported_parameter"), ({"response_format": "url"}, "unsupported_parameter"),
                          ({"output_format": "jpeg"}, "unsupported_parameter"), ({"size": "33x48"}, "invalid_size"),
                          ({"size": "big"}, "invalid_size"), ({"num_steps": 0}, "invalid_request_error")):
            r = c.post("/v1/images/generations", json={**body, **bad})
            assert r.status_code == 400 and r.json()["error"]["code"] == code, (bad, r.text)
        r = c.post("/v1/images/generations", json={**body, "model": "nope"})
        assert r.status_code == 404
        assert c.post("/models/unload", json={"model_id": "zimg"}).status_code == 200
        assert "zimg" not in {m["id"] for m in c.get("/models").json()["models"]}


def test_load_pipeline_from_diffusers_directory(tmp_path):
    """A diffusers-layout directory (model_index.json, transformer/, vae/, text_encoder/)
    loads through the same tensor names the random-init path uses and generates."""
    import json

    from safetensors.torch import save_file

    from helexa_b200.runtime.image_serving import is_image_source, load_pipeline_dir
    from helexa_b200.weights.random_init import save_safetensors
    lm_cfg = get_preset("tiny-qwen3")
    dcfg = zi.tiny_dit_config(cap_feat_dim=lm_cfg.hidden_size)
    vcfg = zi.tiny_vae_config()
    (tmp_path / "model_index.json").write_text(json.dumps({"_class_name": "ZImagePipeline"}))
    for sub, cfg, shapes, seed in (("transformer", dcfg, zi.dit_weight_shapes(dcfg), 2),
                                   ("vae", vcfg, zi.vae_decoder_shapes(vcfg), 3)):
        (tmp_path / sub).mkdir()
        (tmp_path / sub / "config.json").write_text(json.dumps(cfg.to_json()))
        save_file(zi.random_weights(shapes, seed=seed, std=0.05), str(tmp_path / sub / "model.safetensors"))
    save_safetensors(lm_random_weights(lm_cfg, seed=1), lm_cfg, str(tmp_path / "text_encoder"))
    assert is_image_source(str(tmp_path)) and not is_image_source(str(tmp_path / "vae"))
    pipe = load_pipeline_dir(str(tmp_path), "cpu")
    assert pipe.dit.cfg == dcfg and pipe.vae.cfg == vcfg
    ref, _ = _tiny_pipeline()
    lat, cap = torch.randn(16, 8, 8), torch.randn(5, dcfg.cap_feat_dim)
    assert torch.allclose(pipe.dit.forward(lat, 0.4, cap), ref.dit.forward(lat, 0.4, cap), atol=1e-5)
    r = pipe.generate([3, 4, 5], width=32, height=32, steps=2, seed=0)
    assert r.rgb.shape == (32, 32, 3)
