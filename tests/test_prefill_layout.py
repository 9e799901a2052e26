"""The CUDA model's fused per-rank weight layout, checked through its torch-op prefill
path on the CPU against the reference model (covers GDN de-interleave, stacked
experts with the appended shared expert, gated q-proj split)."""
import pytest
import torch

import helexa_b200.models.fast as F
from helexa_b200.config import get_preset
from helexa_b200.models.reference import ReferenceModel
from helexa_b200.weights.random_init import random_weights
from test_fast_model_gpu import _cos, _realistic


@pytest.mark.parametrize("name", ["tiny-qwen3-next", "tiny-qwen3", "tiny-qwen3-moe"])
def test_prefill_layout_cpu(name, monkeypatch):
    monkeypatch.setattr(F, "_allow_cpu_prefill", True)
    cfg = get_preset(name)
    torch.manual_seed(0)
    w = _realistic(cfg, random_weights(cfg, seed=0, std=0.05))
    ref = ReferenceModel(cfg, w)
    fm = F.FastModel.from_hf(cfg, w, "cpu", max_slots=2, max_len=256)
    prompt = torch.randint(0, cfg.vocab_size, (80,), generator=torch.Generator().manual_seed(1))
    st = ref.new_state()
    want = ref.forward(prompt, st)
    got = fm.prefill(1, prompt[:50].int(), 0)           # two chunks: state carried across
    got = fm.prefill(1, prompt[50:].int(), 50)
    assert _cos(got, want) > 0.995
    assert int(fm.pos[1]) == 80
