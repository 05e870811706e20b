"""Cross-check of this package's CPU oracle against the reference's own CPU code.

Every GPU test compares a kernel with ``oscar_b200.kv.oracle`` / ``kv.format``.  These
tests pin that oracle to the reference itself: the unmodified ``oscar_ascend`` package
installed in ``baseline/_ref`` (``pip --no-deps``) is imported with ``vllm``,
``vllm_ascend`` and ``torch_npu`` hidden, which sends it down its pure-torch CPU paths
(``oscar_ascend/backend.py:67-81``).  Compared, on the same inputs:

* ``format.quantize`` / ``dequant`` (``oscar_ascend/format.py:51-97``): byte-identical
  codes, identical fp16 scale/zero;
* the write path: the reference's rotate + sort-threshold clip
  (``backend.py:129-147``) and ``oscar_store_ref`` (``kernels/store_kernel.py:54-102``)
  against ``oracle.store_ref`` on the page-packed pool, compared as 160-byte logical
  slots;
* the staging write (``backend.py:418-481``): owner tags and fp32 staged values against
  the host seat plan the engine uploads (``engine/staging.py``) and ``oracle.StagingArena``;
* multi-query paged attention in rotated space (``kernels/paged_attention.py:20-64``) at
  the config-1 shape (Hq 6, Hk 1, D 256, 24,579-token history + 4-token MTP chunk,
  staging window on) against ``oracle.paged_attention_ref`` within 1e-4.

The module is skipped when ``baseline/_ref`` is absent (a checkout without the
reference install).
"""
from __future__ import annotations

import importlib.abc
import importlib.util
import math
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oscar_b200.engine import staging as host_staging
from oscar_b200.kv import format as fmt
from oscar_b200.kv import oracle as O

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
HIDDEN = ("vllm", "vllm_ascend", "torch_npu")


class _Hide(importlib.abc.MetaPathFinder):
    def find_spec(self, name, path=None, target=None):
        if name.split(".")[0] in HIDDEN:
            raise ModuleNotFoundError(f"{name} hidden for the reference's CPU path")
        return None


@pytest.fixture(scope="module")
def ref():
    if not (REF / "oscar_ascend" / "__init__.py").is_file():
        pytest.skip("reference not installed in baseline/_ref")
    saved = {k: sys.modules.pop(k) for k in list(sys.modules) if k.split(".")[0] in HIDDEN}
    hide = _Hide()
    real_find_spec = importlib.util.find_spec

    def find_spec(name, package=None):
        return None if name.split(".")[0] in HIDDEN else real_find_spec(name, package)

    sys.meta_path.insert(0, hide)
    sys.path.insert(0, str(REF))
    importlib.util.find_spec = find_spec
    try:
        import oscar_ascend.backend as backend
        import oscar_ascend.format as rformat
        from oscar_ascend.kernels import paged_attention, store_kernel
    finally:
        importlib.util.find_spec = real_find_spec
        sys.meta_path.remove(hide)
        sys.path.remove(str(REF))
        sys.modules.update(saved)
    return SimpleNamespace(format=rformat, store=store_kernel, paged=paged_attention, backend=backend)


def _impl(ref, sink=128, recent=256, staging=8192, head=256, hk=1, rk=None, rv=None):
    """A stand-in ``self`` for the reference backend's unbound methods (only the fields
    those methods read)."""
    cfg = SimpleNamespace(sink_tokens=sink, recent_tokens=recent, staging_tokens=staging)
    return SimpleNamespace(_oscar=cfg, _oscar_cfg=cfg, _oscar_warned_quantile=True, num_kv_heads=hk,
                           head_size=head, _layer_rots=lambda layer, dev: (rk, rv))


def _qr(D, g):
    return torch.linalg.qr(torch.randn(D, D, generator=g, dtype=torch.float64))[0].float()


def test_quantize_dequant_identical(ref):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(4096, 256, generator=g) * torch.rand(4096, 1, generator=g) * 4
    x[:64] = torch.round(x[:64] * 2) / 2          # exact half-step ties
    x[64:80] = 0.25                               # constant vectors (scale floor)
    p_r, s_r, z_r = ref.format.quantize(x)
    p_o, s_o, z_o = fmt.quantize(x)
    assert torch.equal(p_r, p_o)
    assert torch.equal(s_r, s_o) and torch.equal(z_r, z_o)
    assert torch.equal(ref.format.dequant(p_r, s_r, z_r, 256), fmt.dequant(p_o, s_o, z_o, 256))


def test_store_slots_identical(ref):
    g = torch.Generator().manual_seed(2)
    N, hk, D, nb = 700, 2, 256, 12
    k = torch.randn(N, hk, D, generator=g).to(torch.bfloat16).float()
    v = torch.randn(N, hk, D, generator=g).to(torch.bfloat16).float()
    Rk, Rv = _qr(D, g), _qr(D, g)
    slots = torch.randperm(nb * fmt.PAGE, generator=g)[:N]
    slots[::97] = -1                               # padding tokens are skipped
    impl = _impl(ref, hk=hk)
    bk = ref.backend.AscendOscarAttentionBackendImpl
    k_rot = bk._rotate_clip(impl, k, Rk, 0.96)
    v_rot = bk._rotate_clip(impl, v, Rv, 0.92)
    kc = torch.zeros(nb, fmt.PAGE, hk, D, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    ref.store.oscar_store_ref(k_rot, v_rot, kc, vc, slots)

    pool = torch.zeros(nb, hk, fmt.page_head_bytes(D), dtype=torch.uint8)
    O.store_ref(k, v, pool, slots, Rk, Rv, 0.96, 0.92)
    s = slots[slots >= 0].long()
    b, o = s // fmt.PAGE, s % fmt.PAGE
    ours = fmt.pool_to_slots(pool, b, o, D)                        # [n, hk, 160]
    k8, v8 = kc.view(torch.uint8), vc.view(torch.uint8)            # [nb, 128, hk, 512]
    theirs = torch.cat([k8[b, o, :, :96], v8[b, o, :, :64]], dim=-1)
    assert torch.equal(ours, theirs)


def test_staging_write_identical(ref):
    g = torch.Generator().manual_seed(3)
    hk, D = 1, 256
    Rk, Rv = _qr(D, g), _qr(D, g)
    # two requests continuing a chunk each, plus a decode row of a third; physical
    # blocks from a shuffled pool so seats collide on the hashed rows
    seqs, qlen = [9000, 300, 4100], [1500, 300, 4]
    bt = torch.randperm(400, generator=g)[:3 * 72].view(3, 72)
    slot, pos, seq_of = [], [], []
    for r, (s, n) in enumerate(zip(seqs, qlen)):
        p = torch.arange(s - n, s)
        slot.append(bt[r, p // fmt.PAGE] * fmt.PAGE + p % fmt.PAGE)
        pos.append(p)
        seq_of.append(torch.full((n,), s))
    slot, pos, seq_of = torch.cat(slot), torch.cat(pos), torch.cat(seq_of)
    slot[5] = -1
    N = slot.numel()
    key = torch.randn(N, hk * D, generator=g)
    value = torch.randn(N, hk * D, generator=g)

    impl = _impl(ref, hk=hk, rk=Rk, rv=Rv)
    bk = ref.backend.AscendOscarAttentionBackendImpl
    layer = SimpleNamespace()
    bk._ensure_staging(impl, layer, (torch.zeros(1, fmt.PAGE, hk, D),))
    md = SimpleNamespace(num_actual_tokens=N, slot_mapping=slot, query_start_loc_cpu=[0, 1500, 1800, 1804],
                         seq_lens_list=seqs)
    bk._staging_write(impl, layer, key, value, md)

    rows = O.staging_rows(128, 256, 8192)
    assert rows == layer._oscar_stage_rows
    k_rot = key.view(N, hk, D) @ Rk
    v_rot = value.view(N, hk, D) @ Rv
    arena = O.StagingArena(rows, hk, D)
    arena.write(O.seat_plan(slot, pos, seq_of, rows, 128, 256), k_rot, v_rot)
    assert torch.equal(arena.owner.long(), layer._oscar_slot_owner)
    kept = layer._oscar_slot_owner >= 0
    assert torch.equal(arena.k[kept], layer._oscar_stage_k[kept])
    assert torch.equal(arena.v[kept], layer._oscar_stage_v[kept])

    # the host plan the engine uploads (numpy) describes the same arena
    stage_seat, owner_seat, owner_val = host_staging.seat_plan(slot.numpy(), pos.numpy(), seq_of.numpy(), rows,
                                                               128, 256)
    own = np.full(rows * fmt.PAGE, -1, dtype=np.int64)
    own[owner_seat] = owner_val
    assert np.array_equal(own.reshape(rows, fmt.PAGE)[np.asarray(layer._oscar_slot_owner) != -1],
                          np.asarray(layer._oscar_slot_owner)[np.asarray(layer._oscar_slot_owner) != -1])
    written = {int(s) for s in stage_seat if s >= 0}
    assert written == {int(s) for s in torch.nonzero(kept.view(-1)).view(-1)}


def test_paged_attention_config1(ref):
    """Config 1: Hq 6, Hk 1, D 256, 24,579 history + 4-token chunk, seed 0, clip
    0.96 / 0.92, sink 128, recent 256, staging 8192."""
    g = torch.Generator().manual_seed(0)
    hq, hk, D, hist, n = 6, 1, 256, 24579, 4
    q = torch.randn(n, hq, D, generator=g).to(torch.bfloat16).float()
    k = torch.randn(hist + n, hk, D, generator=g).to(torch.bfloat16).float()
    v = torch.randn(hist + n, hk, D, generator=g).to(torch.bfloat16).float()
    Rk, Rv = _qr(D, g), _qr(D, g)
    pages = (hist + n + 127) // 128
    nb = pages + 9
    bt = torch.randperm(nb, generator=g)[:pages].to(torch.int32).view(1, -1)
    p = torch.arange(hist)
    slots = bt[0, p // fmt.PAGE].long() * fmt.PAGE + p % fmt.PAGE

    # reference: its clip, its store, its staging write, its attention
    impl = _impl(ref, hk=hk, rk=Rk, rv=Rv)
    bk = ref.backend.AscendOscarAttentionBackendImpl
    kc = torch.zeros(nb, fmt.PAGE, hk, D, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    ref.store.oscar_store_ref(bk._rotate_clip(impl, k[:hist], Rk, 0.96), bk._rotate_clip(impl, v[:hist], Rv, 0.92),
                              kc, vc, slots)
    layer = SimpleNamespace()
    bk._ensure_staging(impl, layer, (kc,))
    md = SimpleNamespace(num_actual_tokens=hist, slot_mapping=slots, query_start_loc_cpu=[0, hist],
                         seq_lens_list=[hist])
    bk._staging_write(impl, layer, k[:hist].view(hist, -1), v[:hist].view(hist, -1), md)
    stage = (layer._oscar_stage_k, layer._oscar_stage_v, layer._oscar_slot_owner)
    scale = 1 / math.sqrt(D)
    theirs = ref.paged.oscar_paged_attention_ref(q @ Rk, k[hist:] @ Rk, v[hist:] @ Rv, kc, vc, bt, [0, n],
                                                 [hist + n], scale, stage)

    # this package's oracle on its own page-packed pool and arena
    pool = torch.zeros(nb, hk, fmt.page_head_bytes(D), dtype=torch.uint8)
    k_rot, v_rot = O.store_ref(k[:hist], v[:hist], pool, slots, Rk, Rv, 0.96, 0.92)
    rows = O.staging_rows(128, 256, 8192)
    arena = O.StagingArena(rows, hk, D)
    arena.write(O.seat_plan(slots, p, torch.full((hist,), hist), rows, 128, 256), k_rot, v_rot)
    ours = O.paged_attention_ref(q @ Rk, k[hist:] @ Rk, v[hist:] @ Rv, pool, bt, [0, n], [hist + n], scale, arena)
    err = float((ours - theirs).norm() / theirs.norm())
    assert err <= fmt.DECODE_TOL, err
