"""Host-side step-metadata checks (``OSCAR_CHECK_STEPS=1``): a whole CPU generation
passes them, and each class of corrupted metadata the kernels would index with is
caught with a message naming it."""
import copy

import numpy as np
import pytest

from oscar_b200.engine import checks
from oscar_b200.engine.engine import LLMEngine
from oscar_b200.models.config import tiny
from oscar_b200.models.qwen35 import P_MAX, HybridModel
from oscar_b200.ops import attention as A


def _engine():
    m = HybridModel(tiny(num_layers=4), device="cpu", seed=3)
    return LLMEngine(m, num_blocks=64, max_slots=4, max_batched_tokens=512, num_spec=3)


def test_generation_passes_step_checks(monkeypatch):
    monkeypatch.setenv("OSCAR_CHECK_STEPS", "1")
    eng = _engine()
    out = eng.generate([list(range(5, 300)), list(range(40, 170))], 6)
    assert all(len(o) == 6 for o in out)


def _one_step_arrays():
    """Metadata of a mixed step (one prefill chunk, one verify) plus its attention plan."""
    eng = _engine()
    eng.add_request(list(range(5, 300)), 4)
    eng.step()  # prefill of the first request
    eng.add_request(list(range(40, 100)), 4)
    captured = {}
    orig = eng._arrays

    def spy(*a, **k):
        arrays, meta = orig(*a, **k)
        captured.setdefault("am", (copy.deepcopy(arrays), dict(meta)))  # the step's main phase
        return arrays, meta

    eng._arrays = spy
    eng.step()  # verify of request 0 + prefill of request 1
    arrays, meta = captured["am"]
    plan = A.plan_attention_host(meta["q_start"], meta["seq_lens"], eng.g, eng.Hk, 148)
    arrays.update(work=plan[0], item_first=plan[1], item_count=plan[2], tiles=plan[5])
    meta.update(max_rb=plan[3], n_work=plan[4], n_short=plan[6],
                n_tiles=int((plan[5][:, 2] >= 0).sum()) if plan[4] > plan[6] else 0)
    kw = dict(num_blocks=eng.bm.num_blocks, max_slots=eng.slots.n, g=eng.g, stage_rows=eng.stage_rows,
              max_pending=P_MAX)
    return arrays, meta, kw


def test_clean_step_with_plan_passes():
    arrays, meta, kw = _one_step_arrays()
    assert meta["n_tiles"] > 0  # the prefill request is paired into tiles
    checks.check_step(arrays, meta, **kw)


def _corrupt(name, arrays, meta):
    a = copy.deepcopy(arrays)
    m = dict(meta)
    if name == "block_out_of_pool":
        bt = np.array(a["bt"]).copy()
        bt[0, 0] = 10_000
        a["bt"] = bt
    elif name == "slot_mismatch":
        s = np.array(a["slots"]).copy()
        s[0] += 1
        a["slots"] = s
    elif name == "positions":
        p = np.array(a["positions"]).copy()
        p[-1] += 1
        a["positions"] = p
    elif name == "req_slot":
        a["req_slot"] = [0, 0]
    elif name == "work_past_keys":
        w = np.array(a["work"]).copy()
        w[0, 3] += 128
        a["work"] = w
    elif name == "tile_item":
        t = np.array(a["tiles"]).copy()
        t[0, 2] = 0 if t[0, 2] != 0 else 1
        a["tiles"] = t
    elif name == "item_count":
        c = np.array(a["item_count"]).copy()
        c[0] = 0
        a["item_count"] = c
    return a, m


@pytest.mark.parametrize("name", ["block_out_of_pool", "slot_mismatch", "positions", "req_slot", "work_past_keys",
                                  "tile_item", "item_count"])
def test_corrupted_metadata_is_caught(name):
    arrays, meta, kw = _one_step_arrays()
    bad, m = _corrupt(name, arrays, meta)
    with pytest.raises(checks.StepMetadataError):
        checks.check_step(bad, m, **kw)
