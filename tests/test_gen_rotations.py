"""Rotation calibration end to end on CPU (reference intent: ``tests/test_calib.py``,
``tests/test_gen_rotations.py``): capture -> objectives -> U.H.P_br -> v2 checkpoint
that the strict loader accepts and the model can run with."""
import torch

from oscar_b200.engine.engine import LLMEngine
from oscar_b200.kv import rotation as Rt
from oscar_b200.kv.gen_rotations import main as gen_main
from oscar_b200.models.config import tiny
from oscar_b200.models.qwen35 import HybridModel


def test_gen_rotations_cli_and_use(tmp_path, monkeypatch):
    out = tmp_path / "oscar_rotations.pt"
    monkeypatch.setenv("OSCAR_ASCEND_CALIB_TOKEN_CAP", "96")
    assert gen_main(["--out", str(out), "--model", "qwen35-tiny", "--layers", "8", "--num-prompts", "2",
                     "--prompt-len", "80", "--device", "cpu"]) == 0
    ck = Rt.load_checkpoint(str(out))
    assert sorted(ck) == [3, 7]
    raw = torch.load(out, weights_only=False)
    assert raw["format_version"] == 2
    for lid in (3, 7):
        for mode in ("k", "v"):
            R = Rt.get_layer_rotation(str(out), lid, 256, "cpu", mode=mode, strict=True)
            assert torch.allclose(R @ R.t(), torch.eye(256), atol=1e-4)
    # the serving model runs with the calibrated rotations
    m = HybridModel(tiny(num_layers=8), device="cpu", rotation=str(out))
    eng = LLMEngine(m, num_blocks=32, max_slots=2, max_batched_tokens=256)
    outs = eng.generate([list(range(4, 60))], 3)
    assert len(outs[0]) == 3
