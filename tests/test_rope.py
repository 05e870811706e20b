"""RoPE scaling (CPU): YaRN frequencies and cos/sin scale against the transformers
implementation, configs carrying YaRN through the checkpoint reader, and a YaRN model
loaded from a transformers checkpoint that matches its forward."""
from __future__ import annotations

import math

import pytest
import torch

from oscar_b200.models import loader as L
from oscar_b200.ops import functional as F

# the reference serve script's override (rope_type yarn, factor 4, original 262144)
SERVE_YARN = {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 262144}


def _hf_yarn(params: dict, max_pos: int):
    tr = pytest.importorskip("transformers")
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

    cfg = tr.Qwen3_5TextConfig(head_dim=256, max_position_embeddings=max_pos,
                               rope_parameters={"rope_theta": 1e7, "partial_rotary_factor": 0.25, **params})
    return ROPE_INIT_FUNCTIONS["yarn"](cfg, "cpu")


@pytest.mark.parametrize("params,max_pos", [
    (SERVE_YARN, 262144),
    ({"rope_type": "yarn", "factor": 8.0, "original_max_position_embeddings": 4096}, 32768),
    ({"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 64, "beta_fast": 16,
      "beta_slow": 2, "truncate": False}, 256),
    ({"rope_type": "yarn", "factor": 2.0, "original_max_position_embeddings": 1024, "mscale": 0.7,
      "mscale_all_dim": 0.3}, 2048),
])
def test_yarn_matches_transformers(params, max_pos):
    inv_hf, scale_hf = _hf_yarn(params, max_pos)
    inv, scale = F.rope_inv_freq(64, 1e7, params, max_pos)
    assert torch.allclose(inv.float(), inv_hf.float(), rtol=1e-6, atol=0)
    assert math.isclose(scale, scale_hf, rel_tol=1e-9)


def test_yarn_tables_scale_and_default():
    inv, scale = F.rope_inv_freq(64, 1e7, SERVE_YARN, 262144)
    assert scale == pytest.approx(0.1 * math.log(4.0) + 1)
    base, one = F.rope_inv_freq(64, 1e7, None)
    assert one == 1.0 and torch.equal(inv[:2], base[:2]) and torch.allclose(inv[-1], base[-1] / 4)
    cos, sin = F.rope_tables(16, 64, 1e7, "cpu", SERVE_YARN)
    assert torch.allclose(cos[0], torch.full((32,), scale, dtype=torch.float32))
    with pytest.raises(ValueError):
        F.rope_inv_freq(64, 1e7, {"rope_type": "longrope"})


def test_checkpoint_config_carries_yarn():
    from oscar_b200.models.config import tiny

    raw = L.hf_config(tiny())
    raw["rope_parameters"] = {**raw["rope_parameters"], **SERVE_YARN, "beta_fast": 16}
    cfg = L.config_from_hf(raw)
    assert cfg.rope_scaling == {**SERVE_YARN, "beta_fast": 16}
    assert L.config_from_hf(L.hf_config(cfg)).rope_scaling == cfg.rope_scaling
    raw["rope_parameters"]["rope_type"] = "dynamic"
    with pytest.raises(L.CheckpointError, match="dynamic"):
        L.config_from_hf(raw)


def test_yarn_model_matches_transformers_forward(tmp_path):
    """One attention layer with YaRN over a short original context (the ramp and the cos/sin
    scale both act on the test prompt's positions)."""
    tr = pytest.importorskip("transformers")
    from oscar_b200.engine.engine import LLMEngine

    prompt = list(range(3, 200, 2)) + [5] * 40
    rope = {"rope_type": "yarn", "rope_theta": 1e7, "partial_rotary_factor": 0.25, "factor": 4.0,
            "original_max_position_embeddings": 32, "mrope_section": [11, 11, 10]}
    torch.manual_seed(0)
    hc = tr.Qwen3_5TextConfig(
        vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=1, layer_types=["full_attention"],
        num_attention_heads=6, num_key_value_heads=1, head_dim=256, linear_num_key_heads=2,
        linear_num_value_heads=6, linear_key_head_dim=128, linear_value_head_dim=128, max_position_embeddings=8192,
        rope_parameters=rope)
    hf = tr.Qwen3_5ForCausalLM(hc).float().eval()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            if "norm" in n:
                p.add_(torch.randn_like(p) * 0.2)
            if "q_proj" in n or "k_proj" in n:
                p.mul_(8.0)  # sharper attention, so the positions' encoding matters
    hf.save_pretrained(str(tmp_path), safe_serialization=True)
    with torch.no_grad():
        ref = hf.model(torch.tensor([prompt]), use_cache=False).last_hidden_state[0].float()

    def hidden(scaling_override=None):
        cfg = L.config_from_hf(str(tmp_path))
        if scaling_override is not None:
            cfg.rope_scaling = scaling_override or None
        m = L.from_pretrained(str(tmp_path), device="cpu", kv_mode="bf16", mtp=False, config=cfg)
        assert (cfg.rope_scaling or {}).get("rope_type") == (None if scaling_override == {} else "yarn")
        eng = LLMEngine(m, num_blocks=64, max_slots=4, max_batched_tokens=512, num_spec=0)
        eng.add_request(prompt, 2)
        eng.step()
        return eng.last[0].float()

    err = float((hidden() - ref).norm() / ref.norm())
    plain = float((hidden({}) - ref).norm() / ref.norm())
    assert err < 0.05, err
    assert plain > 2 * err, (plain, err)  # without the scaling the forward is clearly off


def test_serve_flag_applies_the_override():
    import json

    from oscar_b200.serve.__main__ import build, parse

    args = parse(["--model", "qwen35-tiny", "--device", "cpu", "--num-blocks", "16", "--max-num-seqs", "2",
                  "--max-batched-tokens", "256", "--rope-scaling", json.dumps(SERVE_YARN)])
    _, _, model, eng, _ = build(args)
    assert model.cfg.rope_scaling == SERVE_YARN
    scale = 0.1 * math.log(4.0) + 1
    assert torch.allclose(model.rope[0][0], torch.full_like(model.rope[0][0], scale))
    assert len(eng.generate([list(range(5, 40))], 3)[0]) == 3
