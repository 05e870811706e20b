"""Hugging Face Qwen3.5 checkpoint loading (CPU).

* the exporter and the loader are inverse mappings (TP1 round trip);
* every rank of a TP2 / TP4 load holds the same slices as the random-init model of that
  rank, whose slicing the constructors define independently of the loader;
* a ``transformers`` ``Qwen3_5ForCausalLM`` saved with ``save_pretrained`` and loaded
  here gives the same final hidden states up to the W8A8 quantisation (the bounds were
  set from measured errors: 2.7 % for one GDN layer, 3.4 % for one attention layer and
  5.8 % for four layers; a flipped conv tap order gives 65 %, swapped ``b`` / ``a``
  rows 18 %, swapped query / gate rows 40 %);
* missing, misshapen and unexpected tensors are errors.
"""
from __future__ import annotations

import json
import os

import pytest
import torch

from oscar_b200.engine.engine import LLMEngine
from oscar_b200.models import loader as L
from oscar_b200.models.config import tiny
from oscar_b200.models.qwen35 import FullAttentionLayer, HybridModel, QLinear
from oscar_b200.parallel.groups import TPGroup

PROMPT = list(range(3, 200, 2)) + [5] * 40


def _same_weight(a: QLinear, b: QLinear, what: str):
    """Same dequantised weight: identical codes where a row reaches +-127, else within
    half a quantisation step of the re-quantised row."""
    assert a.q.shape == b.q.shape, what
    d = (L.dequantize(a) - L.dequantize(b)).abs()
    tol = 0.5 * torch.maximum(a.s, b.s)[:, None] * 1.001 + 1e-12
    assert bool((d <= tol).all()), what


def _tensors(model: HybridModel):
    """(name, value) of every weight of one rank, in a fixed order."""
    out = [("embed", model.embed), ("lm_head", model.lm_head), ("final_norm", model.final_norm)]
    parts = list(enumerate(model.layers))
    if model.mtp is not None:
        t = model.mtp
        out += [("mtp.fc", t.fc), ("mtp.norm_emb", t.norm_emb), ("mtp.norm_hid", t.norm_hid),
                ("mtp.final_norm", t.final_norm)]
        parts.append(("mtp", (t.layer, t.mlp)))
    for i, (mixer, mlp) in parts:
        names = (["qkv", "o", "q_norm", "k_norm"] if isinstance(mixer, FullAttentionLayer) else
                 ["inp", "out", "conv_w", "A_log", "dt_bias", "norm_w"]) + ["input_norm", "post_norm"]
        out += [(f"{i}.{n}", getattr(mixer, n)) for n in names]
        out += [(f"{i}.gate_up", mlp.gate_up), (f"{i}.down", mlp.down)]
    return out


def _assert_same_model(a: HybridModel, b: HybridModel):
    for (n, x), (_, y) in zip(_tensors(a), _tensors(b)):
        if isinstance(x, QLinear):
            _same_weight(x, y, n)
        else:
            assert x.shape == y.shape and torch.allclose(x.float(), y.float(), rtol=0, atol=1e-6), n


def _hidden(model: HybridModel, prompt=PROMPT) -> torch.Tensor:
    eng = LLMEngine(model, num_blocks=64, max_slots=4, max_batched_tokens=512, num_spec=0)
    eng.add_request(prompt, 2)
    eng.step()
    return eng.last[0].float().clone()


def test_config_round_trip_and_nested_form():
    cfg = tiny(num_layers=8)
    raw = L.hf_config(cfg)
    got = L.config_from_hf(raw)
    for k in ("vocab_size", "hidden_size", "intermediate_size", "num_layers", "num_attention_heads",
              "num_key_value_heads", "head_dim", "linear_num_key_heads", "linear_num_value_heads",
              "rope_theta", "partial_rotary_factor", "num_mtp_layers", "layer_types"):
        assert getattr(got, k) == getattr(cfg, k), k
    nested = L.config_from_hf({"model_type": "qwen3_5", "text_config": raw, "vision_config": {}})
    assert nested.layer_types == cfg.layer_types
    with pytest.raises(L.CheckpointError, match="head_dim"):
        L.config_from_hf({**raw, "head_dim": 128})
    with pytest.raises(L.CheckpointError, match="mixture-of-experts"):
        L.config_from_hf({**raw, "num_experts": 8})


@pytest.fixture(scope="module")
def exported(tmp_path_factory):
    """A random-init TP1 model written in the Hugging Face layout (fp32, several shards)."""
    cfg = tiny(num_layers=4)
    model = HybridModel(cfg, device="cpu", seed=3)
    path = str(tmp_path_factory.mktemp("ckpt"))
    L.save_hf_checkpoint(model, path, dtype=torch.float32, max_shard_bytes=4 << 20)
    return model, path


def test_export_writes_a_sharded_hf_directory(exported):
    _, path = exported
    files = sorted(os.listdir(path))
    shards = [f for f in files if f.endswith(".safetensors")]
    assert "config.json" in files and len(shards) > 1
    with open(os.path.join(path, "model.safetensors.index.json")) as f:
        index = json.load(f)["weight_map"]
    assert index["model.layers.3.self_attn.q_proj.weight"] in shards
    assert "model.layers.0.linear_attn.in_proj_qkv.weight" in index and "mtp.fc.weight" in index


def _requantized(model: HybridModel) -> HybridModel:
    """``model`` with every W8A8 weight re-quantised from its dequantised values, as the
    loader quantises the exported ones: rows whose codes never reach +-127 get the scale
    ``max|w| / 127`` and new codes."""
    objs = [model] + [o for pair in model.layers for o in pair]
    if model.mtp is not None:
        objs += [model.mtp, model.mtp.layer, model.mtp.mlp]
    for o in objs:
        for k, v in list(vars(o).items()):
            if isinstance(v, QLinear):
                setattr(o, k, L.quantize_rows(L.dequantize(v), "cpu"))
    return model


def test_tp1_round_trip(exported):
    """Loading the export gives the model back, bit for bit after re-quantisation.  (The
    forward is compared exactly, not within a tolerance: the random-init model is
    chaotic - scaling one projection by 1 + 1e-4 moves its final hidden states by 6 %.)"""
    model, path = exported
    loaded = L.from_pretrained(path, device="cpu", seed=3)  # seed: the same random KV rotations
    assert loaded.mtp is not None
    _assert_same_model(model, loaded)
    expect = _requantized(HybridModel(model.cfg, device="cpu", seed=3))
    assert torch.equal(_hidden(expect), _hidden(loaded))


@pytest.mark.parametrize("world", [2, 4])
def test_tp_slices_match_the_random_init_ranks(exported, tmp_path, world):
    """A TP load takes, on every rank, the slices the constructors take from the logical
    model: query heads, replicated KV heads (1 KV head over 2 / 4 ranks), GDN key and
    value heads, MLP columns, vocabulary rows."""
    model, path = exported
    cfg = model.cfg
    if cfg.linear_num_key_heads % world:
        # 4 ranks need 4 GDN key heads: export a model of that shape
        cfg = tiny(num_layers=4, num_attention_heads=12, num_key_value_heads=2, linear_num_key_heads=4,
                   linear_num_value_heads=12)
        path = str(tmp_path / "ckpt4")
        L.save_hf_checkpoint(HybridModel(cfg, device="cpu", seed=3), path, dtype=torch.float32)
    for rank in range(world):
        tp = TPGroup(rank=rank, world=world)
        _assert_same_model(HybridModel(cfg, tp, device="cpu", seed=3), L.from_pretrained(path, tp=tp, device="cpu"))


def test_reader_reads_row_ranges(exported):
    _, path = exported
    r = L.CheckpointReader(path)
    name = "model.layers.0.linear_attn.in_proj_qkv.weight"
    full = r.full(name)
    assert torch.equal(r.rows(name, [(0, 3), (256, 260)]), torch.cat([full[0:3], full[256:260]]))
    assert r.shape(name) == tuple(full.shape)


def test_missing_misshapen_and_unexpected_tensors(exported):
    model, path = exported
    sd = L.hf_state_dict(model, dtype=torch.float32)
    cfg = model.cfg

    def load(d, **kw):
        with L.no_random_init():
            m = HybridModel(cfg, device="cpu", mtp=kw.pop("mtp", True))
        return L.load_checkpoint(m, d, **kw)

    rep = load(dict(sd))
    assert rep.mtp_loaded and not rep.unused and rep.root == "model."
    bad = dict(sd)
    del bad["model.layers.1.linear_attn.A_log"]
    with pytest.raises(L.CheckpointError, match="A_log"):
        load(bad)
    bad = dict(sd)
    bad["model.layers.3.self_attn.k_norm.weight"] = torch.zeros(7)
    with pytest.raises(L.CheckpointError, match="k_norm"):
        load(bad)
    bad = dict(sd)
    bad["model.layers.0.mlp.gate_proj.bias"] = torch.zeros(cfg.intermediate_size)
    with pytest.raises(L.CheckpointError, match="bias"):
        load(bad)
    assert load(bad, strict=False).unused == ["model.layers.0.mlp.gate_proj.bias"]
    no_mtp = {k: v for k, v in sd.items() if not k.startswith("mtp.")}
    with pytest.raises(L.CheckpointError, match="MTP"):
        load(no_mtp)
    assert not load(no_mtp, mtp=False).mtp_loaded
    # multimodal prefix, tied lm_head, vision tower ignored
    mm = {("model.language_model." + k[len("model."):] if k.startswith("model.") else k): v
          for k, v in sd.items() if k != "lm_head.weight"}
    mm["model.visual.blocks.0.attn.qkv.weight"] = torch.zeros(3, 3)
    rep = load(mm)
    assert rep.root == "model.language_model." and rep.tied_lm_head
    assert rep.unused == ["model.visual.blocks.0.attn.qkv.weight"]


def _hf_model(types, tmp_path):
    tr = pytest.importorskip("transformers")
    torch.manual_seed(0)
    hc = tr.Qwen3_5TextConfig(
        vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=len(types), layer_types=types,
        num_attention_heads=6, num_key_value_heads=1, head_dim=256, linear_num_key_heads=2,
        linear_num_value_heads=6, linear_key_head_dim=128, linear_value_head_dim=128, max_position_embeddings=8192,
        rope_parameters={"rope_type": "default", "rope_theta": 1e7, "partial_rotary_factor": 0.25,
                         "mrope_section": [11, 11, 10]})
    hf = tr.Qwen3_5ForCausalLM(hc).float().eval()
    with torch.no_grad():  # norms away from their init so the 1 + w convention is exercised
        for n, p in hf.named_parameters():
            if "norm" in n or "dt_bias" in n:
                p.add_(torch.randn_like(p) * 0.2)
    path = str(tmp_path / "hf")
    hf.save_pretrained(path, safe_serialization=True, max_shard_size="2MB")
    with torch.no_grad():
        ref = hf.model(torch.tensor([PROMPT]), use_cache=False).last_hidden_state[0].float()
    return path, ref


@pytest.mark.parametrize("types,bound", [
    (["linear_attention"], 0.045),
    (["full_attention"], 0.05),
    (["linear_attention", "linear_attention", "linear_attention", "full_attention"], 0.085),
])
@pytest.mark.parametrize("kv", ["bf16", "int2"])
def test_transformers_checkpoint_matches_hf_forward(tmp_path, types, bound, kv):
    path, ref = _hf_model(types, tmp_path)
    model = L.from_pretrained(path, device="cpu", kv_mode=kv, mtp=False)
    hid = _hidden(model)
    err = float((hid - ref).norm() / ref.norm())
    cos = torch.nn.functional.cosine_similarity(hid, ref, dim=-1)
    assert err < bound, err
    assert float(cos.min()) > 0.99


def test_serve_and_rotation_calibration_take_a_checkpoint(exported, tmp_path, monkeypatch):
    """``python -m oscar_b200.serve --weights DIR`` builds the checkpoint's model (same
    tokens as loading it directly), and ``gen_rotations --weights DIR`` calibrates on it."""
    from oscar_b200.kv import rotation as Rt
    from oscar_b200.kv.gen_rotations import main as gen_main
    from oscar_b200.serve.__main__ import build, parse

    _, path = exported
    args = parse(["--weights", path, "--device", "cpu", "--num-blocks", "64", "--max-num-seqs", "4",
                  "--max-batched-tokens", "512", "--seed", "3"])
    _, _, model, eng, mans = build(args)
    assert mans[0]["layer_ids"] == [3] and model.cfg.num_layers == 4
    direct = LLMEngine(L.from_pretrained(path, device="cpu", seed=3), num_blocks=64, max_slots=4,
                       max_batched_tokens=512)
    prompts = [list(range(5, 60)), list(range(9, 30))]
    assert eng.generate(prompts, 4) == direct.generate(prompts, 4)
    out = tmp_path / "rot.pt"
    monkeypatch.setenv("OSCAR_ASCEND_CALIB_TOKEN_CAP", "64")
    assert gen_main(["--out", str(out), "--weights", path, "--num-prompts", "2", "--prompt-len", "64",
                     "--device", "cpu"]) == 0
    assert sorted(Rt.load_checkpoint(str(out))) == [3]


def test_eos_token_ids(tmp_path):
    (tmp_path / "config.json").write_text(json.dumps({"text_config": {"eos_token_id": 7}}))
    assert L.eos_token_ids(str(tmp_path)) == [7]
    (tmp_path / "generation_config.json").write_text(json.dumps({"eos_token_id": [3, 9]}))
    assert L.eos_token_ids(str(tmp_path)) == [3, 9]
