"""Single-GPU attention sweep (reference tool:
``tools/benchmark_attention.py:25-205``).

Head geometry of one TP4 rank of the target model: Hq = 6, Hk = 1, head_dim 256,
128-token pages.  Paged decode / MTP-verify attention over INT2 pages at history
lengths 1024 / 8192 / 32768, batch 1-32, 1-4 query tokens, plus a prefill
continuation of 9256 new tokens over a 15360-token INT2 history.  Variants:

* ``int2_tc``   - the tcgen05/TMEM kernels (decode/verify items of <= 32 rows; prefill
                  chunks in tiles of 128 rows),
* ``int2_mma``  - the warp-level mma.sync kernel,
* ``bf16_tc``   - the same attention over a BF16 KV cache (the uncompressed baseline) on
                  the tcgen05 BF16 kernel (TMA-fed, <= 32 rows per item),
* ``bf16``      - BF16 KV on the warp-level mma.sync kernel.

Each variant is checked against the first one on the merged output (rtol 1e-2),
then the attention kernel alone is timed with CUDA events, L2 flushed before every
sample, median of warm samples.  Reported: microseconds, bytes of KV the kernel must
read, achieved GB/s and its fraction of the measured HBM copy bandwidth.

    python -m oscar_b200.bench.attention [--hist 1024,8192,32768] [--batch 1,8,32] [--qlen 1,4] [--trace]
"""
from __future__ import annotations

import argparse
import json
import math
import os

import numpy as np
import torch

from ..kv import format as fmt
from ..ops import attention as A
from ..ops import functional as F
from ..ops._ext import ext
from .harness import compare_calls, peak_hbm_gbs


def _peak_gbs() -> float:
    return peak_hbm_gbs()


def build_case(hist: int, batch: int, qlen: int, hq: int = 6, hk: int = 1, D: int = 256, seed: int = 0,
               staging: bool = True, device="cuda"):
    """Random INT2 + BF16 caches holding ``hist`` tokens of history per request."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    seqs = [hist + qlen] * batch
    pages = [(s + 127) // 128 for s in seqs]
    nb = sum(pages) + 4
    perm = torch.randperm(nb, generator=g)
    bt = torch.zeros(batch, max(pages), dtype=torch.int32)
    k = 0
    for r in range(batch):
        bt[r, :pages[r]] = perm[k:k + pages[r]]
        k += pages[r]
    dev = torch.device(device)
    pool = torch.randint(0, 256, (nb, hk, fmt.page_head_bytes(D)), dtype=torch.uint8, generator=g)
    _, _, ks, kz, vs, vz = fmt.page_views(pool, D)
    ks.copy_((torch.rand(ks.shape, generator=g) * 0.5 + 0.2).half())
    vs.copy_((torch.rand(vs.shape, generator=g) * 0.5 + 0.2).half())
    kz.copy_((-torch.rand(kz.shape, generator=g) - 0.3).half())
    vz.copy_((-torch.rand(vz.shape, generator=g) - 0.3).half())
    kc = torch.randn(nb, 128, hk, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(nb, 128, hk, D, generator=g).to(torch.bfloat16)
    T = batch * qlen
    q = torch.randn(T, hq, D, generator=g).half()
    kf = torch.randn(T, hk, D, generator=g).half()
    vf = torch.randn(T, hk, D, generator=g).half()
    q_start = [0] + list(np.cumsum([qlen] * batch))
    for r in range(batch):  # the store writes the current chunk into the BF16 cache first
        for i in range(qlen):
            pos = hist + i
            kc[int(bt[r, pos // 128]), pos % 128] = kf[r * qlen + i].to(torch.bfloat16)
            vc[int(bt[r, pos // 128]), pos % 128] = vf[r * qlen + i].to(torch.bfloat16)
    stage = None
    if staging:
        rows = 64
        sk = torch.randn(rows * 128, hk, D, generator=g)
        sv = torch.randn(rows, hk, D, 128, generator=g)
        owner = torch.full((rows * 128,), -1, dtype=torch.int32)
        for r in range(batch):  # sink page and the last two pages of every request
            for p in {0, pages[r] - 2, pages[r] - 1}:
                if p >= 0:
                    b = int(bt[r, p])
                    owner.view(rows, 128)[b % rows] = b
            # the current chunk's tokens are staged with their own (fresh) values, as the
            # store kernel does in serving
            for i in range(qlen):
                pos = hist + i
                b, off = int(bt[r, pos // 128]), pos % 128
                t = r * qlen + i
                sk[(b % rows) * 128 + off] = kf[t].float()
                sv[b % rows, :, :, off] = vf[t].float()
        stage = (sk.to(dev), sv.to(dev), owner.to(dev), rows)
    d = lambda t: t.to(dev)  # noqa: E731
    tok_req = torch.repeat_interleave(torch.arange(batch), torch.tensor([qlen] * batch)).to(torch.int32)
    # the work list a serving step uses: fixed splits for decode / verify items
    sms = F.num_sms(dev)
    fixed = A.decode_splits(q_start, hq // hk, hk, sms) if qlen * hq // hk <= A.LONG_ROWS else 0
    wt, first, count, max_rb, n_work, tt, n_short, rpi_short = A.plan_attention_host(
        q_start, seqs, hq // hk, hk, sms, fixed_splits=fixed)
    n_tiles = int((tt[:, 2] >= 0).sum()) if n_work > n_short else 0
    plan = A.AttnPlan(torch.from_numpy(wt).to(dev), torch.from_numpy(first).to(dev), torch.from_numpy(count).to(dev),
                      max_rb, n_work, torch.from_numpy(tt).to(dev), n_tiles, n_short, rpi_short)
    return dict(q=d(q), kf=d(kf), vf=d(vf), pool=d(pool), kc=d(kc), vc=d(vc), bt=d(bt), stage=stage,
                q_start=q_start, seqs=seqs, q_start_t=d(torch.tensor(q_start, dtype=torch.int32)),
                seq_lens_t=d(torch.tensor(seqs, dtype=torch.int32)), tok_req=d(tok_req), plan=plan, hq=hq, hk=hk,
                D=D, pages=sum(pages), T=T)


def _attention(c, kv_mode: int, use_tc: bool):
    A.USE_TC = use_tc
    out, _, _ = A.attention(c["q"], c["kf"], c["vf"], Hq=c["hq"], Hk=c["hk"], D=c["D"], scale=1 / 16,
                            kv_mode=kv_mode, pool=c["pool"], kc=c["kc"], vc=c["vc"],
                            stage=c["stage"] if kv_mode == 0 else None, block_tables=c["bt"],
                            q_start_t=c["q_start_t"], seq_lens_t=c["seq_lens_t"], q_start=c["q_start"],
                            seq_lens=c["seqs"], plan=c["plan"], tok_req=c["tok_req"], RvT=None, gate=None,
                            gate_ld=0, gate_hstride=0, want_bf16=True, want_q=False)
    return out


def _kernel_only(c, kv_mode: int, use_tc: bool):
    plan = c["plan"]
    po = torch.empty(plan.n_work * c["hk"] * A.ROWS * c["D"], dtype=torch.float32, device=c["q"].device)
    pl = torch.empty(plan.n_work * c["hk"] * A.ROWS, dtype=torch.float32, device=c["q"].device)
    sk, sv, own, rows = c["stage"] if (kv_mode == 0 and c["stage"] is not None) else (None, None, None, 0)
    A.USE_TC = use_tc
    rpi = A._rpi(plan, c["q_start"], c["hq"] // c["hk"])
    tiles = plan.tiles if (use_tc and plan.n_tiles > 0) else None
    e = ext()

    def run():
        e.paged_attention(c["q"], c["kf"], c["vf"], c["hq"], c["hk"], c["D"], 1 / 16, kv_mode, c["pool"], c["kc"],
                          c["vc"], sk, sv, own, rows, c["bt"], c["q_start_t"], c["seq_lens_t"], plan.work, po, pl,
                          None, rpi, tiles, plan.n_tiles if tiles is not None else 0, plan.n_short, None, 0, 0)
        return None

    return run


def kv_bytes(c, kv_mode: int) -> int:
    D = c["D"]
    per_page = fmt.page_head_bytes(D) + 512 if kv_mode == 0 else 2 * 128 * D * 2
    return c["pages"] * c["hk"] * per_page


def run_case(hist, batch, qlen, iters=10, variants=("int2_tc", "int2_mma", "bf16_tc", "bf16"), hk=1,
             staging=True):
    c = build_case(hist, batch, qlen, hq=6 * hk, hk=hk, staging=staging)
    rows = qlen * c["hq"] // c["hk"]
    vs = [v for v in variants if not (v == "bf16_tc" and rows > 32)]
    # numerics: merged outputs against the first variant
    outs = {}
    for v in vs:
        outs[v] = _attention(c, 0 if v.startswith("int2") else 1, v.endswith("_tc")).float()
    ref = outs[vs[0]]
    errs = {v: float((outs[v] - ref).norm() / ref.norm()) for v in vs}
    # variants that read the same cache must agree (the BF16 cache is another cache)
    for fam in ("int2", "bf16"):
        fv = [v for v in vs if v.startswith(fam)]
        for v in fv[1:]:
            e = float((outs[v] - outs[fv[0]]).norm() / outs[fv[0]].norm())
            assert e < 1e-2, f"{v} disagrees with {fv[0]}: {e:.3e}"
    fns = {v: _kernel_only(c, 0 if v.startswith("int2") else 1, v.endswith("_tc")) for v in vs}
    tim = compare_calls(fns, iters=iters, flush=True)
    peak = _peak_gbs()
    res = []
    for v in vs:
        kvm = 0 if v.startswith("int2") else 1
        by = kv_bytes(c, kvm)
        us = tim[v].median_ms * 1e3
        gbs = by / (us * 1e-6) / 1e9
        res.append({"variant": v, "hist": hist, "batch": batch, "qlen": qlen, "us": round(us, 2),
                    "kv_bytes": by, "gbs": round(gbs, 1), "frac_hbm_of_measured": round(gbs / peak, 3),
                    "n_work": c["plan"].n_work, "rel_err_vs_first": round(errs[v], 5)})
    A.USE_TC = os.environ.get("OSCAR_ATTN_TC", "1") != "0"
    return res


# Event slots of the tcgen05 decode kernel's per-CTA timeline (globaltimer ns, 96 per CTA):
# 0 start, 1 setup done, 2 softmax role done, 3 end; 8+i page i copy issued, 16+i S(i)
# issued, 24+i K(i) converted, 32+i V(i) converted, 40+i P(i) written; for pages 0-3 the
# softmax marks 48+4i S ready, 49+4i S loaded, 50+4i P buffer free, 51+4i maxima agreed,
# 64+4i metadata loaded, 65+4i score loop done, slot 80+i the score loop's clock64 cycles,
# 84+i K(i) conversion started, 88+i K(i) seen by the MMA issuer, 92+i V(i) conversion started;
# clock64 cycles (pages 0-3): 96+i K conversion issue, 100+i its TMEM store wait, 104+i / 108+i
# the same for V, 112+i issuing the S MMAs.  128 slots per CTA.
TRACE_EVENTS = {"issue": (8, 16), "qk": (16, 24), "kdone": (24, 32), "vdone": (32, 40), "pdone": (40, 48)}


def trace_case(hist: int, batch: int, qlen: int, show: int = 3, hk: int = 1, staging: bool = True) -> dict:
    """Per-CTA timeline of the tcgen05 INT2 decode kernel (one traced launch after warm-up).

    Returns the kernel span, the CTA duration quantiles and, for the ``show`` longest CTAs,
    every recorded event relative to the CTA's start (µs)."""
    c = build_case(hist, batch, qlen, hq=6 * hk, hk=hk, staging=staging)
    fn = _kernel_only(c, 0, True)
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    n_cta = c["plan"].n_work * c["hk"]
    buf = torch.zeros(n_cta * 128, dtype=torch.int64, device=c["q"].device)
    ext().attn_tc_trace(buf.data_ptr())
    try:
        fn()
        torch.cuda.synchronize()
    finally:
        ext().attn_tc_trace(0)
    t = buf.view(n_cta, 128).cpu().numpy().astype(np.float64)
    started = t[:, 0] > 0
    t0 = t[started, 0].min()
    rel = np.where(t[:, :80] > 0, (t[:, :80] - t0) / 1000.0, np.nan)
    dur = rel[:, 3] - rel[:, 0]
    out = {"hist": hist, "batch": batch, "qlen": qlen, "ctas": int(n_cta),
           "span_us": round(float(np.nanmax(rel[:, 3])), 2),
           "cta_us_min_med_max": [round(float(np.nanmin(dur)), 2), round(float(np.nanmedian(dur)), 2),
                                  round(float(np.nanmax(dur)), 2)], "ctas_shown": []}
    for idx in np.argsort(-np.nan_to_num(dur))[:show]:
        r = rel[idx]
        ev = {k: [round(float(x - r[0]), 2) for x in r[a:b] if not np.isnan(x)] for k, (a, b) in TRACE_EVENTS.items()}
        ev["softmax_pages"] = [[round(float(x - r[0]), 2) for x in r[48 + 4 * q:52 + 4 * q] if not np.isnan(x)]
                               for q in range(4)]
        ev["score_loop_cycles"] = [int(t[idx, 80 + q]) for q in range(4)]
        ext_rel = np.where(t[idx, 84:96] > 0, (t[idx, 84:96] - t0) / 1000.0 - r[0], np.nan)
        ev["kstart"] = [round(float(x), 2) for x in ext_rel[0:4] if not np.isnan(x)]
        ev["mma_kfull"] = [round(float(x), 2) for x in ext_rel[4:8] if not np.isnan(x)]
        ev["vstart"] = [round(float(x), 2) for x in ext_rel[8:12] if not np.isnan(x)]
        cyc = t[idx, 96:116].astype(np.int64)
        ev["cycles_k_issue"], ev["cycles_k_stwait"] = cyc[0:4].tolist(), cyc[4:8].tolist()
        ev["cycles_v_issue"], ev["cycles_v_stwait"] = cyc[8:12].tolist(), cyc[12:16].tolist()
        ev["cycles_s_mma_issue"] = cyc[16:20].tolist()
        out["ctas_shown"].append({"cta": int(idx), "work": c["plan"].work[idx % c["plan"].n_work].tolist(),
                                  "dur_us": round(float(dur[idx]), 2), "events": ev})
    return out


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--hist", default="1024,8192,32768")
    ap.add_argument("--batch", default="1,8,32")
    ap.add_argument("--qlen", default="1,4")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--hk", type=int, default=1, help="KV heads (6 query heads each); 4 is the TP1 model")
    ap.add_argument("--variants", default="int2_tc,int2_mma,bf16_tc,bf16")
    ap.add_argument("--no-staging", action="store_true", help="no sink/recent staging window (all tokens INT2)")
    ap.add_argument("--prefill", action="store_true", help="also run the 9256-over-15360 continuation")
    ap.add_argument("--trace", action="store_true",
                    help="print the per-CTA timeline of the tcgen05 decode kernel instead of timing")
    args = ap.parse_args(argv)
    torch.cuda.init()
    if args.trace:
        for hist in map(int, args.hist.split(",")):
            for batch in map(int, args.batch.split(",")):
                for qlen in map(int, args.qlen.split(",")):
                    print(json.dumps(trace_case(hist, batch, qlen, hk=args.hk, staging=not args.no_staging)),
                          flush=True)
        return
    for hist in map(int, args.hist.split(",")):
        for batch in map(int, args.batch.split(",")):
            for qlen in map(int, args.qlen.split(",")):
                for r in run_case(hist, batch, qlen, args.iters, variants=tuple(args.variants.split(",")),
                                  hk=args.hk, staging=not args.no_staging):
                    print(json.dumps(r), flush=True)
    if args.prefill:
        for r in run_case(15360, 1, 9256, max(3, args.iters // 3), variants=("int2_tc", "int2_mma", "bf16")):
            print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
