"""Numeric probes run before serving: ``python -m oscar_b200.serve.probes``.

The reference gates its launch on three probe scripts (``delivery/probe_oscar.py``,
``probe_paged.py``, ``probe_prefill.py``); these are the same gates for the sm_100a
kernels, each against the CPU oracle of :mod:`oscar_b200.kv.oracle`:

* ``store``        - fused store (no rotation): INT2 bytes identical to the oracle's,
                     negative slots write nothing;
* ``dequant``      - slot round trip within ``DEQUANT_TOL`` (1e-5);
* ``decode_ref``   - the paged oracle equals SDPA on the dequantised cache (1e-4);
* ``paged``        - multi-request paged attention, non-monotonic block tables, q_len
                     1 / 4 / 2, prefixes 0 / 129 / 257, staging hits and misses,
                     empty KV splits; kernel vs oracle at 1e-2 (both kernels);
* ``long``         - 16,387-token prefix with 16:1 GQA, kernel vs oracle at 1e-2;
* ``full_backend`` - the config-1 shape: 24,579-token history + 4-token MTP chunk,
                     6:1 GQA, rotations, clip 0.96/0.92, staging window on and off,
                     rotate -> store -> attend -> merge vs the oracle at 1e-2.

Without a GPU only the CPU-side probes run.  Exit status 0 iff every probe passed.
"""
from __future__ import annotations

import json
import sys
import time

import numpy as np
import torch

from ..kv import format as fmt
from ..kv import oracle as O
from ..ops import attention as A
from ..ops import functional as F


def _rel(a, b) -> float:
    a, b = a.float().cpu(), b.float().cpu()
    return float((a - b).norm() / (b.norm() + 1e-30))


def probe_dequant() -> dict:
    g = torch.Generator().manual_seed(0)
    k = torch.randn(64, 2, 256, generator=g) * 3
    v = torch.randn(64, 2, 256, generator=g)
    slot = fmt.make_slot_bytes(k, v)
    kd, vd = fmt.parse_slot_bytes(slot, 256)
    sk, zk = fmt.vector_scales(k)
    ref = fmt.codes(k, sk, zk).float() * sk + zk
    err = float((kd - ref).abs().max())
    return {"ok": err <= fmt.DEQUANT_TOL, "max_abs": err}


def probe_decode_ref() -> dict:
    g = torch.Generator().manual_seed(1)
    hq, hk, D, n = 8, 1, 256, 300
    pool = torch.zeros(4, hk, fmt.page_head_bytes(D), dtype=torch.uint8)
    k = torch.randn(n, hk, D, generator=g)
    v = torch.randn(n, hk, D, generator=g)
    slots = torch.arange(n)
    O.store_ref(k, v, pool, slots)
    bt = torch.arange(4, dtype=torch.int32).view(1, 4)
    q = torch.randn(1, hq, D, generator=g)
    kn = torch.randn(1, hk, D, generator=g)
    vn = torch.randn(1, hk, D, generator=g)
    out = O.paged_attention_ref(q, kn, vn, pool, bt, [0, 1], [n + 1], 1 / 16)
    kh, vh = fmt.dequant_tokens(pool, torch.zeros(n, dtype=torch.long) + slots // 128, slots % 128, D)
    ref = O.sdpa_causal(q, torch.cat([kh, kn]), torch.cat([vh, vn]), 1 / 16, n)
    err = _rel(out, ref)
    return {"ok": err <= fmt.DECODE_TOL, "rel": err}


def _random_pool(nb, hk, D, g):
    pool = torch.randint(0, 256, (nb, hk, fmt.page_head_bytes(D)), dtype=torch.uint8, generator=g)
    _, _, ks, kz, vs, vz = fmt.page_views(pool, D)
    ks.copy_((torch.rand(ks.shape, generator=g) * 0.5 + 0.2).half())
    vs.copy_((torch.rand(vs.shape, generator=g) * 0.5 + 0.2).half())
    kz.copy_((-torch.rand(kz.shape, generator=g) - 0.3).half())
    vz.copy_((-torch.rand(vz.shape, generator=g) - 0.3).half())
    return pool


def _paged_case(seqs, qlens, hq, hk, seed, stage_pages=(), dev="cuda", use_tc=True):
    g = torch.Generator().manual_seed(seed)
    D = 256
    R = len(seqs)
    pages = [(s + 127) // 128 for s in seqs]
    nb = sum(pages) + 3
    perm = torch.randperm(nb, generator=g)  # non-monotonic block tables
    bt = torch.zeros(R, max(pages), dtype=torch.int32)
    k = 0
    for r in range(R):
        bt[r, :pages[r]] = perm[k:k + pages[r]]
        k += pages[r]
    pool = _random_pool(nb, hk, D, g)
    rows = 8
    sk = torch.randn(rows * 128, hk, D, generator=g)
    sv = torch.randn(rows, hk, D, 128, generator=g)
    owner = torch.full((rows * 128,), -1, dtype=torch.int32)
    for r, p, cnt in stage_pages:  # staging hits on (request, page), first cnt tokens
        b = int(bt[r, p])
        owner.view(rows, 128)[b % rows, :cnt] = b
    T = sum(qlens)
    q = torch.randn(T, hq, D, generator=g).half()
    kf = torch.randn(T, hk, D, generator=g).half()
    vf = torch.randn(T, hk, D, generator=g).half()
    q_start = [0] + list(np.cumsum(qlens))
    kw = dict(Hq=hq, Hk=hk, D=D, scale=1 / 16, kv_mode=0, kc=None, vc=None, q_start=q_start, seq_lens=seqs,
              RvT=None, gate=None, gate_ld=0, gate_hstride=0, want_bf16=True, want_q=False)
    ref, _, _ = A.attention(q, kf, vf, pool=pool, stage=(sk, sv, owner, rows), block_tables=bt, q_start_t=None,
                            seq_lens_t=None, plan=None, tok_req=None, **kw)
    d = lambda t: t.to(dev)  # noqa: E731
    tok_req = torch.repeat_interleave(torch.arange(R), torch.tensor(qlens)).to(torch.int32)
    plan = A.plan_attention(q_start, seqs, hq // hk, hk, F.num_sms(torch.device(dev)), dev)
    old = A.USE_TC
    A.USE_TC = use_tc
    try:
        out, _, _ = A.attention(d(q), d(kf), d(vf), pool=d(pool), stage=(d(sk), d(sv), d(owner), rows),
                                block_tables=d(bt), q_start_t=d(torch.tensor(q_start, dtype=torch.int32)),
                                seq_lens_t=d(torch.tensor(seqs, dtype=torch.int32)), plan=plan, tok_req=d(tok_req),
                                **kw)
        torch.cuda.synchronize()
    finally:
        A.USE_TC = old
    return _rel(out, ref)


def probe_paged() -> dict:
    errs = {}
    for use_tc in (True, False):
        # prefixes 0 / 129 / 257 with q_len 1 / 4 / 2, staging hit on request 2's first page
        errs[f"tc={use_tc}"] = _paged_case([1, 133, 259], [1, 4, 2], 8, 1, 3, stage_pages=[(2, 0, 60)],
                                           use_tc=use_tc)
    worst = max(errs.values())
    return {"ok": worst <= 1e-2, "rel": errs}


def probe_long() -> dict:
    err = _paged_case([16387 + 4], [4], 16, 1, 5, stage_pages=[(0, 0, 128), (0, 128, 3)])
    return {"ok": err <= 1e-2, "rel": err}


def probe_store() -> dict:
    from ..ops import attention as Aop
    g = torch.Generator().manual_seed(7)
    hq, hk, D, T = 6, 1, 256, 200
    n = hq * 2 * D + 2 * hk * D
    qkv = (torch.randn(T, n, generator=g) * 2).to(torch.bfloat16)
    slots = torch.randperm(4 * 128, generator=g)[:T].to(torch.int32)
    slots[5] = -1
    res = {}
    for dev in ("cpu", "cuda"):
        pool = torch.zeros(4, hk, fmt.page_head_bytes(D), dtype=torch.uint8, device=dev)
        qo = torch.empty(T, hq, D, dtype=torch.float16, device=dev)
        kf = torch.empty(T, hk, D, dtype=torch.float16, device=dev)
        vf = torch.empty_like(kf)
        Aop.kv_store(qkv.to(dev), q_off=0, q_head_stride=2 * D, k_off=hq * 2 * D, v_off=hq * 2 * D + hk * D, Hq=hq,
                     Hk=hk, D=D, q_norm_w=None, k_norm_w=None, eps=1e-6, norm_offset=1.0,
                     positions=torch.arange(T, dtype=torch.int32, device=dev), rope_cos=None, rope_sin=None,
                     rot_dim=0, Rk=None, Rv=None, k_clip_idx=245, v_clip_idx=235, q_out=qo, k_fresh=kf,
                     v_fresh=vf, kv_mode=0, pool=pool, kc=None, vc=None, slots=slots.to(dev))
        res[dev] = pool.cpu()
    diff = int((res["cpu"] != res["cuda"]).sum())
    return {"ok": diff == 0, "byte_diff": diff}


def probe_full_backend() -> dict:
    """Config-1 shape through the model's FULL-attention layer path (rotate, clip,
    quantise, stage, attend, merge) for window on / off, vs the oracle."""
    from ..config import OscarConfig
    out = {}
    for window in (True, False):
        out[f"window={window}"] = _full_backend_case(window)
    worst = max(out.values())
    return {"ok": worst <= 1e-2, "rel": out}


def _full_backend_case(window: bool, hist: int = 24579, qlen: int = 4) -> float:
    g = torch.Generator().manual_seed(0)
    hq, hk, D = 6, 1, 256
    Rk = torch.linalg.qr(torch.randn(D, D, generator=g, dtype=torch.float64))[0].float()
    Rv = torch.linalg.qr(torch.randn(D, D, generator=g, dtype=torch.float64))[0].float()
    k = torch.randn(hist, hk, D, generator=g).to(torch.bfloat16).float()
    v = torch.randn(hist, hk, D, generator=g).to(torch.bfloat16).float()
    pages = (hist + qlen + 127) // 128
    pool = torch.zeros(pages, hk, fmt.page_head_bytes(D), dtype=torch.uint8)
    slots = torch.arange(hist)
    k_rot, v_rot = O.store_ref(k, v, pool, slots, Rk, Rv, 0.96, 0.92)
    rows = O.staging_rows(128, 256, 8192)
    stage = None
    if window:
        stage = O.StagingArena(rows, hk, D)
        pos = torch.arange(hist)
        plan = O.seat_plan(slots, pos, torch.full((hist,), hist + qlen), rows, 128, 256)
        stage.write(plan, k_rot, v_rot)
    q = torch.randn(qlen, hq, D, generator=g).to(torch.bfloat16).float()
    kn = torch.randn(qlen, hk, D, generator=g).to(torch.bfloat16).float()
    vn = torch.randn(qlen, hk, D, generator=g).to(torch.bfloat16).float()
    bt = torch.arange(pages, dtype=torch.int32).view(1, -1)
    ref = O.oscar_attention_ref(q, kn, vn, pool, bt, [0, qlen], [hist + qlen], 1 / 16, Rk, Rv, stage)
    dev = "cuda"
    d = lambda t: t.to(dev)  # noqa: E731
    st = None
    if stage is not None:
        st = (d(stage.k.view(rows * 128, hk, D)), d(stage.v.permute(0, 2, 3, 1).contiguous()),
              d(stage.owner.view(-1).to(torch.int32)), rows)
    qr, knr, vnr = (q @ Rk).half(), (kn @ Rk).half(), (vn @ Rv).half()
    plan_ = A.plan_attention([0, qlen], [hist + qlen], hq // hk, hk, F.num_sms(torch.device(dev)), dev)
    out, _, _ = A.attention(d(qr), d(knr), d(vnr), Hq=hq, Hk=hk, D=D, scale=1 / 16, kv_mode=0, pool=d(pool), kc=None,
                            vc=None, stage=st, block_tables=d(bt), q_start_t=d(torch.tensor([0, qlen], dtype=torch.int32)),
                            seq_lens_t=d(torch.tensor([hist + qlen], dtype=torch.int32)), q_start=[0, qlen],
                            seq_lens=[hist + qlen], plan=plan_, tok_req=d(torch.zeros(qlen, dtype=torch.int32)),
                            RvT=d(Rv.t().contiguous()), gate=None, gate_ld=0, gate_hstride=0, want_bf16=True,
                            want_q=False)
    torch.cuda.synchronize()
    return _rel(out.view(qlen, hq, D), ref)


CPU_PROBES = {"dequant": probe_dequant, "decode_ref": probe_decode_ref}
GPU_PROBES = {"store": probe_store, "paged": probe_paged, "long": probe_long, "full_backend": probe_full_backend}


def run(gpu: bool | None = None) -> dict:
    gpu = torch.cuda.is_available() if gpu is None else gpu
    probes = dict(CPU_PROBES)
    if gpu:
        probes.update(GPU_PROBES)
    res = {}
    for name, fn in probes.items():
        t0 = time.perf_counter()
        try:
            r = fn()
        except Exception as e:  # noqa: BLE001 - a probe that raises fails
            r = {"ok": False, "error": repr(e)}
        r["s"] = round(time.perf_counter() - t0, 2)
        res[name] = r
    return res


def main() -> int:
    res = run()
    print(json.dumps(res, indent=1, default=str))
    return 0 if all(r["ok"] for r in res.values()) else 1


if __name__ == "__main__":
    sys.exit(main())
