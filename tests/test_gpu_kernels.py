"""sm_100a kernels vs the pure-torch fp32/fp64 references (GPU only)."""
import math

import numpy as np
import pytest
import torch

from oscar_b200.kv import format as fmt
from oscar_b200.kv.oracle import staging_rows
from oscar_b200.ops import attention as A
from oscar_b200.ops import functional as F
from oscar_b200.ops._ext import ext
from oscar_b200.ops.gdn import gdn_step
from oscar_b200.engine.staging import seat_plan

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp(min=1e-30)).item()


# ---------------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M,N,K", [(128, 1024, 1024), (32, 3072, 5120), (4, 512, 640), (300, 1024, 2048),
                                   (1000, 2304, 512), (200, 5120, 4352)])
def test_gemm_i8_bf16(M, N, K):
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N)
    x = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=DEV, generator=g)
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=DEV, generator=g)
    xs = torch.rand(M, device=DEV, generator=g) * 0.01 + 0.001
    ws = torch.rand(N, device=DEV, generator=g) * 0.01 + 0.001
    y = F.linear_i8(x, xs, w, ws)
    torch.cuda.synchronize()
    ref = (x.double() @ w.double().t()) * xs.double()[:, None] * ws.double()[None, :]
    assert y.shape == (M, N)
    assert _rel(y, ref) < 5e-3


@pytest.mark.parametrize("M,N,K", [(128, 5120, 6144), (16, 1280, 4352), (512, 640, 1536), (300, 1030, 1024),
                                   (24, 2050, 1024)])
def test_gemm_i8_accumulate_splitk(M, N, K):
    """Swapped (decode) and plain (prefill, 16-byte reductions) accumulate layouts, and the
    scalar fallback for rows that are not 16-byte aligned."""
    g = torch.Generator(device=DEV).manual_seed(N)
    x = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=DEV, generator=g)
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=DEV, generator=g)
    xs = torch.rand(M, device=DEV, generator=g) * 0.01
    ws = torch.rand(N, device=DEV, generator=g) * 0.01
    base = torch.randn(M, N, device=DEV)
    out = base.clone()
    F.linear_i8(x, xs, w, ws, out=out, accumulate=True)
    torch.cuda.synchronize()
    ref = base.double() + (x.double() @ w.double().t()) * xs.double()[:, None] * ws.double()[None, :]
    assert _rel(out, ref) < 1e-5


@pytest.mark.parametrize("M,N,K", [(128, 1024, 5120), (32, 3584, 5120), (100, 1030, 2048), (300, 1792, 5120)])
def test_gemm_i8_bf16_splitk(M, N, K):
    """bf16 GEMMs with fewer output tiles than SMs are split along K: the partials meet in
    the zeroed fp32 workspace and the last split of a tile writes bf16.  A second call is as
    accurate (the workspace and tile counters are left at zero; the fp32 order in which
    splits add up may differ between calls)."""
    plan = F.plan_gemm(M, N, K, F.num_sms(torch.device(DEV)), allow_split=True)
    assert plan.splits > 1
    g = torch.Generator(device=DEV).manual_seed(M + N)
    x = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=DEV, generator=g)
    w = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=DEV, generator=g)
    xs = torch.rand(M, device=DEV, generator=g) * 0.01 + 0.001
    ws = torch.rand(N, device=DEV, generator=g) * 0.01 + 0.001
    y1 = F.linear_i8(x, xs, w, ws)
    y2 = F.linear_i8(x, xs, w, ws)
    torch.cuda.synchronize()
    ref = (x.double() @ w.double().t()) * xs.double()[:, None] * ws.double()[None, :]
    assert _rel(y1, ref) < 5e-3 and _rel(y2, ref) < 5e-3
    assert _rel(y1, y2) < 1e-3
    wsb = F._SPLIT_WS[torch.device(DEV).index or 0]
    assert wsb[0].abs().max().item() == 0.0 and wsb[1].abs().max().item() == 0


def test_gemm_status_clean():
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    x = torch.randint(-127, 128, (64, 256), dtype=torch.int8, device=DEV)
    w = torch.randint(-127, 128, (256, 256), dtype=torch.int8, device=DEV)
    F.linear_i8(x, torch.ones(64, device=DEV), w, torch.ones(256, device=DEV), status=st)
    torch.cuda.synchronize()
    assert st.item() == 0


# ---------------------------------------------------------------------------- elementwise
def test_rmsnorm_quant_matches_ref():
    T, H = 37, 5120
    x = torch.randn(T, H, device=DEV)
    d = torch.randn(T, H, device=DEV)
    w = torch.randn(H, device=DEV) * 0.1
    xg = x.clone()
    q, s, y = F.rmsnorm_quant(xg, w, 1e-6, delta=d, want_bf16=True)
    xc = x.cpu().clone()
    qr, sr, yr = F.rmsnorm_quant(xc, w.cpu(), 1e-6, delta=d.cpu(), want_bf16=True)
    torch.cuda.synchronize()
    assert torch.allclose(xg.cpu(), xc)
    assert _rel(y.float().cpu(), yr.float()) < 1e-2
    assert (q.cpu().int() - qr.int()).abs().max().item() <= 1
    assert torch.allclose(s.cpu(), sr, rtol=1e-2)


def test_swiglu_and_act_quant():
    T, I = 19, 4352
    gu = torch.randn(T, 2 * I, device=DEV).to(torch.bfloat16)
    q, s = F.swiglu_quant(gu, I)
    qr, sr = F.swiglu_quant(gu.cpu(), I)
    assert (q.cpu().int() - qr.int()).abs().max().item() <= 1
    assert torch.allclose(s.cpu(), sr, rtol=1e-3)
    x = torch.randn(T, 6144, device=DEV).to(torch.bfloat16)
    q, s = F.act_quant(x)
    qr, sr = F.act_quant(x.cpu())
    assert (q.cpu().int() - qr.int()).abs().max().item() <= 1


def test_embed_argmax():
    V, H, T = 1000, 256, 9
    table = torch.randn(V, H, device=DEV).to(torch.bfloat16)
    tok = torch.randint(0, 2 * V, (T,), dtype=torch.int32, device=DEV)
    out = torch.empty(T, H, device=DEV)
    F.embed(tok, table, 500, out)
    ref = torch.empty(T, H)
    F.embed(tok.cpu(), table.cpu(), 500, ref)
    assert torch.equal(out.cpu(), ref)
    for V_ in (70000, 70003, 248320):  # 16-byte rows (vector path), odd rows (scalar path), 31 chunks
        logits = torch.randn(T, V_, device=DEV).to(torch.bfloat16)
        logits[1, 5] = logits[1, 60001] = 9.0  # a tie resolves to the lower index
        v, i = F.argmax(logits, 123)
        vr, ir = F.argmax(logits.cpu(), 123)
        keep = torch.arange(T) != 1
        assert torch.equal(i.cpu()[keep], ir[keep])
        assert int(i[1]) == 5 + 123


# ---------------------------------------------------------------------------- KV store
def _qkv_layout(Hq, Hk, D):
    q_off, qhs = 0, 2 * D
    k_off = Hq * 2 * D
    v_off = k_off + Hk * D
    return q_off, qhs, k_off, v_off, v_off + Hk * D


@pytest.mark.parametrize("rot", [False, True])
def test_kv_store_matches_ref(rot):
    """rot=False: no norm / RoPE / rotation, so the quantiser sees identical inputs and
    codes, meta and staging must be bit-exact.  rot=True: the full fused pipeline; the
    q/k norm and RoPE outputs may differ by one bf16 ulp (rsqrt rounding), so codes are
    compared statistically."""
    torch.manual_seed(0)
    Hq, Hk, D, T = 6, 1, 256, 300
    q_off, qhs, k_off, v_off, N = _qkv_layout(Hq, Hk, D)
    qkv = (torch.randn(T, N) * 2).to(torch.bfloat16)
    pos = torch.arange(T, dtype=torch.int32) + 5
    cos, sin = F.rope_tables(1024, 64, 1e7, "cpu")
    qn, kn = (torch.randn(D) * 0.1, torch.randn(D) * 0.1) if rot else (None, None)
    if not rot:
        cos = sin = None
    Rk = torch.linalg.qr(torch.randn(D, D)).Q.contiguous() if rot else None
    Rv = torch.linalg.qr(torch.randn(D, D)).Q.contiguous() if rot else None
    nb = 8
    slots = torch.randperm(nb * fmt.PAGE)[:T].to(torch.int32)
    slots[7] = -1
    rows = 4
    seq = np.full(T, T + 5)
    ss, os_, ov = seat_plan(slots.numpy().astype(np.int64), pos.numpy().astype(np.int64), seq, rows, 128, 256)
    outs = {}
    for dev in ("cpu", DEV):
        tens = lambda t: None if t is None else t.to(dev)  # noqa: E731
        pool = torch.zeros(nb, Hk, fmt.page_head_bytes(D), dtype=torch.uint8, device=dev)
        sk = torch.zeros(rows * 128, Hk, D, device=dev)
        sv = torch.zeros(rows, Hk, D, 128, device=dev)
        owner = torch.full((rows * 128,), -1, dtype=torch.int32, device=dev)
        qo = torch.empty(T, Hq, D, dtype=torch.float16, device=dev)
        kf = torch.empty(T, Hk, D, dtype=torch.float16, device=dev)
        vf = torch.empty_like(kf)
        A.kv_store(tens(qkv), q_off=q_off, q_head_stride=qhs, k_off=k_off, v_off=v_off, Hq=Hq, Hk=Hk, D=D,
                   q_norm_w=tens(qn), k_norm_w=tens(kn), eps=1e-6, norm_offset=1.0, positions=tens(pos),
                   rope_cos=tens(cos), rope_sin=tens(sin), rot_dim=64 if rot else 0, Rk=tens(Rk), Rv=tens(Rv), k_clip_idx=245,
                   v_clip_idx=235, q_out=qo, k_fresh=kf, v_fresh=vf, kv_mode=0, pool=pool, kc=None, vc=None,
                   slots=tens(slots), stage_k=sk, stage_v=sv, stage_seat=tens(torch.from_numpy(ss)),
                   owner=owner, owner_seat=tens(torch.from_numpy(os_)), owner_val=tens(torch.from_numpy(ov)))
        outs[dev] = [t.cpu() for t in (qo, kf, vf, pool, sk, sv, owner)]
    c, g = outs["cpu"], outs[DEV]
    assert _rel(g[0].float(), c[0].float()) < 2e-3
    assert _rel(g[1].float(), c[1].float()) < 2e-3
    assert torch.equal(g[6], c[6])
    assert _rel(g[4], c[4]) < (1e-3 if rot else 1e-7)
    # INT2 codes and meta: exact without rotation; with rotation a tiny fraction of
    # codes may sit on the other side of a rounding boundary (fp32 summation order).
    kc_c, vc_c, *mc = fmt.page_views(c[3], D)
    kc_g, vc_g, *mg = fmt.page_views(g[3], D)
    # 2-bit fields compared position by position (K token-major rows, V dim-major rows)
    codes_c = torch.cat([fmt.unpack(x, x.shape[-1] * 4).flatten() for x in (kc_c, vc_c)])
    codes_g = torch.cat([fmt.unpack(x, x.shape[-1] * 4).flatten() for x in (kc_g, vc_g)])
    diff = (codes_c != codes_g).float().mean().item()
    if rot:
        assert diff < 2e-3
    else:
        assert diff == 0.0
        for a, b in zip(mc, mg):
            assert torch.equal(a, b)


def test_kv_store_bf16_mode():
    Hq, Hk, D, T = 6, 1, 256, 40
    q_off, qhs, k_off, v_off, N = _qkv_layout(Hq, Hk, D)
    qkv = torch.randn(T, N).to(torch.bfloat16)
    pos = torch.arange(T, dtype=torch.int32)
    slots = torch.arange(T, dtype=torch.int32) + 3
    res = {}
    for dev in ("cpu", DEV):
        kc = torch.zeros(2, 128, Hk, D, dtype=torch.bfloat16, device=dev)
        vc = torch.zeros_like(kc)
        qo = torch.empty(T, Hq, D, dtype=torch.float16, device=dev)
        kf = torch.empty(T, Hk, D, dtype=torch.float16, device=dev)
        vf = torch.empty_like(kf)
        A.kv_store(qkv.to(dev), q_off=q_off, q_head_stride=qhs, k_off=k_off, v_off=v_off, Hq=Hq, Hk=Hk, D=D,
                   q_norm_w=None, k_norm_w=None, eps=1e-6, norm_offset=1.0, positions=pos.to(dev), rope_cos=None,
                   rope_sin=None, rot_dim=0, Rk=None, Rv=None, k_clip_idx=-1, v_clip_idx=-1, q_out=qo, k_fresh=kf,
                   v_fresh=vf, kv_mode=1, pool=None, kc=kc, vc=vc, slots=slots.to(dev))
        res[dev] = (kc.cpu(), vc.cpu())
    assert torch.equal(res["cpu"][0], res[DEV][0]) and torch.equal(res["cpu"][1], res[DEV][1])


# ---------------------------------------------------------------------------- attention
def _build_cache(dev, Hk, D, seqs, qlens, seed, stage_rows=0, kv_mode=0):
    """Fill a cache for requests with histories `seqs - qlens` through the store op."""
    torch.manual_seed(seed)
    R = len(seqs)
    pages = [(s + fmt.PAGE - 1) // fmt.PAGE for s in seqs]
    nb = sum(pages) + 2
    perm = torch.randperm(nb)
    bt = torch.zeros(R, max(pages), dtype=torch.int32)
    k = 0
    for r in range(R):
        bt[r, :pages[r]] = perm[k:k + pages[r]]
        k += pages[r]
    return nb, bt


@pytest.mark.parametrize("use_tc", [True, False], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("case", ["decode", "mtp", "mixed", "bf16", "long", "prefill", "bf16_prefill"])
def test_paged_attention_matches_ref(case, use_tc, monkeypatch):
    """``mixed`` / ``prefill`` run prefill chunks (tcgen05 prefill kernel: fresh-only and
    INT2-history tiles, staged tokens, two KV heads) next to short verify/decode requests
    in the same step; ``bf16_prefill`` the same plan over a BF16 cache."""
    _attention_case(case, use_tc, monkeypatch, window=False)


@pytest.mark.parametrize("use_tc", [True, False], ids=["tcgen05", "mma_sync"])
@pytest.mark.parametrize("case", ["mtp", "long", "prefill"])
def test_paged_attention_window_staging(case, use_tc, monkeypatch):
    """The per-request window layout of the staging arena: rows come from each request's
    state slot and logical page (sink pages and a ring of recent pages), in all three INT2
    attention kernels (decode/verify tcgen05, warp-level, prefill tcgen05)."""
    _attention_case(case, use_tc, monkeypatch, window=True)


def _attention_case(case, use_tc, monkeypatch, window):
    if not use_tc and case in ("mixed", "prefill"):
        pytest.skip("same kernel as the tcgen05 run")
    monkeypatch.setattr(A, "USE_TC", use_tc)
    torch.manual_seed(1)
    Hq, Hk, D = (12, 2, 256) if case == "prefill" else (6, 1, 256)
    g = Hq // Hk
    if case == "decode":
        seqs, qlens = [700, 1200, 129], [1, 1, 1]
    elif case == "mtp":
        seqs, qlens = [2000, 513, 4100], [4, 4, 4]
    elif case == "mixed":
        seqs, qlens = [300, 1000], [300, 37]
    elif case == "long":
        seqs, qlens = [16384, 9000, 24579], [4, 4, 4]
    elif case == "prefill":
        seqs, qlens = [1500, 700, 1003], [200, 64, 3]
    elif case == "bf16_prefill":
        seqs, qlens = [1500, 403], [200, 3]
    else:
        seqs, qlens = [900, 260], [4, 4]
    kv_mode = 1 if case.startswith("bf16") else 0
    R = len(seqs)
    nb, bt = _build_cache("cpu", Hk, D, seqs, qlens, 3)
    pool = torch.zeros(nb, Hk, fmt.page_head_bytes(D), dtype=torch.uint8)
    kc = torch.randn(nb, 128, Hk, D).to(torch.bfloat16)
    vc = torch.randn(nb, 128, Hk, D).to(torch.bfloat16)
    # random INT2 pages (codes + plausible meta)
    kcod, vcod, ks, kz, vs, vz = fmt.page_views(pool, D)
    kcod.copy_(torch.randint(0, 256, kcod.shape, dtype=torch.uint8))
    vcod.copy_(torch.randint(0, 256, vcod.shape, dtype=torch.uint8))
    ks.copy_((torch.rand(ks.shape) * 0.5 + 0.2).half())
    vs.copy_((torch.rand(vs.shape) * 0.5 + 0.2).half())
    kz.copy_((-torch.rand(kz.shape) - 0.3).half())
    vz.copy_((-torch.rand(vz.shape) - 0.3).half())
    from oscar_b200.kv.oracle import window_row
    req_slot = torch.tensor([(2 * r + 1) % 5 for r in range(R)], dtype=torch.int32)  # state slots 0..4
    sink_pages, ring = 1, 4
    rows = 5 * (sink_pages + ring) if window else 4
    sk = torch.randn(rows * 128, Hk, D)
    sv = torch.randn(rows, Hk, D, 128)
    owner = torch.full((rows * 128,), -1, dtype=torch.int32)
    b0 = int(bt[0, 0])
    if window:
        # request 0's sink page, and a page near the end of every request's history
        owner.view(rows, 128)[window_row(int(req_slot[0]), 0, sink_pages, ring), :50] = b0
        for r in range(R):
            lp = max(0, (seqs[r] - qlens[r] - 1) // 128 - 1)
            owner.view(rows, 128)[window_row(int(req_slot[r]), lp, sink_pages, ring), 30:90] = int(bt[r, lp])
    else:
        # mark a few staged tokens for request 0: its first page
        owner.view(rows, 128)[b0 % rows, :50] = b0
    T = sum(qlens)
    q = (torch.randn(T, Hq, D)).half()
    kf = torch.randn(T, Hk, D).half()
    vf = torch.randn(T, Hk, D).half()
    q_start = [0] + list(np.cumsum(qlens))
    # the store writes the current chunk into the BF16 cache before attention reads it
    for r in range(R):
        for i in range(qlens[r]):
            pos = seqs[r] - qlens[r] + i
            b, o = int(bt[r, pos // 128]), pos % 128
            kc[b, o] = kf[q_start[r] + i].to(torch.bfloat16)
            vc[b, o] = vf[q_start[r] + i].to(torch.bfloat16)
    lay_cpu = (req_slot, sink_pages, ring) if window else None
    stage_cpu = (sk, sv, owner, rows, lay_cpu) if kv_mode == 0 else None
    ref_b, ref_q, ref_s = A.attention(q, kf, vf, Hq=Hq, Hk=Hk, D=D, scale=1 / 16, kv_mode=kv_mode, pool=pool, kc=kc,
                                      vc=vc, stage=stage_cpu, block_tables=bt, q_start_t=None, seq_lens_t=None,
                                      q_start=q_start, seq_lens=seqs, plan=None, tok_req=None, RvT=None, gate=None,
                                      gate_ld=0, gate_hstride=0, want_bf16=True, want_q=False)
    d = lambda t: t.to(DEV)  # noqa: E731
    tok_req = torch.repeat_interleave(torch.arange(R), torch.tensor(qlens)).to(torch.int32)
    plan = A.plan_attention(q_start, seqs, g, Hk, F.num_sms(torch.device(DEV)), DEV)
    lay = (d(req_slot), sink_pages, ring) if window else None
    stage = (d(sk), d(sv), d(owner), rows, lay) if kv_mode == 0 else None
    out_b, _, _ = A.attention(d(q), d(kf), d(vf), Hq=Hq, Hk=Hk, D=D, scale=1 / 16, kv_mode=kv_mode, pool=d(pool),
                              kc=d(kc), vc=d(vc), stage=stage, block_tables=d(bt),
                              q_start_t=d(torch.tensor(q_start, dtype=torch.int32)),
                              seq_lens_t=d(torch.tensor(seqs, dtype=torch.int32)), q_start=q_start, seq_lens=seqs,
                              plan=plan, tok_req=d(tok_req), RvT=None, gate=None, gate_ld=0, gate_hstride=0,
                              want_bf16=True, want_q=False)
    torch.cuda.synchronize()
    assert _rel(out_b.float().cpu(), ref_b.float()) < 1e-2


def test_attention_merge_rotation_gate_quant():
    torch.manual_seed(2)
    Hq, Hk, D = 6, 1, 256
    seqs, qlens = [500, 300], [4, 4]
    T = 8
    nb = 10
    bt = torch.arange(8, dtype=torch.int32).view(2, 4)
    pool = torch.zeros(nb, Hk, fmt.page_head_bytes(D), dtype=torch.uint8)
    kcod, vcod, ks, kz, vs, vz = fmt.page_views(pool, D)
    kcod.copy_(torch.randint(0, 256, kcod.shape, dtype=torch.uint8))
    vcod.copy_(torch.randint(0, 256, vcod.shape, dtype=torch.uint8))
    for t in (ks, vs):
        t.copy_(torch.full(t.shape, 0.3).half())
    for t in (kz, vz):
        t.copy_(torch.full(t.shape, -0.45).half())
    q = torch.randn(T, Hq, D).half()
    kf = torch.randn(T, Hk, D).half()
    vf = torch.randn(T, Hk, D).half()
    Rv = torch.linalg.qr(torch.randn(D, D)).Q
    RvT = Rv.t().contiguous()
    gate_buf = torch.randn(T, Hq * 2 * D).to(torch.bfloat16)
    gate = gate_buf[:, D:]
    q_start = [0, 4, 8]
    kw = dict(Hq=Hq, Hk=Hk, D=D, scale=1 / 16, kv_mode=0, kc=None, vc=None, stage=None, q_start=q_start,
              seq_lens=seqs, gate_ld=gate_buf.stride(0), gate_hstride=2 * D, want_bf16=True, want_q=True)
    rb, rq, rs = A.attention(q, kf, vf, pool=pool, block_tables=bt, q_start_t=None, seq_lens_t=None, plan=None,
                             tok_req=None, RvT=RvT, gate=gate, **kw)
    d = lambda t: t.to(DEV)  # noqa: E731
    plan = A.plan_attention(q_start, seqs, Hq // Hk, Hk, F.num_sms(torch.device(DEV)), DEV)
    gb = d(gate_buf)
    ob, oq, os_ = A.attention(d(q), d(kf), d(vf), pool=d(pool), block_tables=d(bt),
                              q_start_t=d(torch.tensor(q_start, dtype=torch.int32)),
                              seq_lens_t=d(torch.tensor(seqs, dtype=torch.int32)), plan=plan,
                              tok_req=d(torch.tensor([0] * 4 + [1] * 4, dtype=torch.int32)), RvT=d(RvT),
                              gate=gb[:, D:], **kw)
    torch.cuda.synchronize()
    assert _rel(ob.float().cpu(), rb.float()) < 1e-2
    assert torch.allclose(os_.cpu(), rs, rtol=2e-2)


# ---------------------------------------------------------------------------- GDN
def _gdn_inputs(T, Hk, Hv, dk, dv, seed):
    g = torch.Generator().manual_seed(seed)
    r = Hv // Hk
    n_qkvz = Hk * (2 * dk + 2 * r * dv)
    qkvz = (torch.randn(T, n_qkvz, generator=g)).to(torch.bfloat16)
    ba = (torch.randn(T, 2 * Hv, generator=g)).to(torch.bfloat16)
    conv_dim = 2 * Hk * dk + Hv * dv
    w = dict(conv_w=torch.randn(conv_dim, 4, generator=g) * 0.5, A_log=torch.log(torch.rand(Hv, generator=g) * 15 + 1),
             dt_bias=torch.ones(Hv), norm_w=1 + torch.randn(dv, generator=g) * 0.02)
    return qkvz, ba, w, conv_dim


@pytest.mark.parametrize("mode", ["prefill_long", "prefill_mixed", "decode", "verify_commit"])
def test_gdn_step_matches_ref(mode):
    """prefill_long / prefill_mixed exercise the chunked (WY) tensor-core path for
    requests of >= 16 tokens, next to verify and short requests in the same step."""
    Hk, Hv, dk, dv = 2, 6, 128, 128
    slots, P = 4, 4
    conv_dim = 2 * Hk * dk + Hv * dv
    gen = torch.Generator().manual_seed(5)
    state0 = (torch.randn(slots, Hv, dk, dv, generator=gen) * 0.1).to(torch.bfloat16)
    conv0 = torch.randn(2, slots, conv_dim, 3, generator=gen).to(torch.bfloat16)
    px0 = torch.randn(2, slots, P, conv_dim, generator=gen).to(torch.bfloat16)
    pb0 = torch.randn(slots, P, 2 * Hv, generator=gen).to(torch.bfloat16)
    if mode == "prefill_long":
        qlens, ncom, keep = [200, 37], [0, 0], [0, 0]
    elif mode == "prefill_mixed":
        qlens, ncom, keep = [150, 4, 3, 64], [0, 2, 0, 0], [0, 1, 0, 0]
    elif mode == "decode":
        qlens, ncom, keep = [1, 1, 1], [0, 0, 0], [0, 0, 0]
    else:
        qlens, ncom, keep = [4, 4, 4], [2, 4, 0], [1, 1, 1]
    R = len(qlens)
    T = sum(qlens)
    qkvz, ba, w, _ = _gdn_inputs(T, Hk, Hv, dk, dv, 9)
    q_start = torch.tensor([0] + list(np.cumsum(qlens)), dtype=torch.int32)
    meta = dict(parity=torch.tensor([0, 1, 0, 1][:R], dtype=torch.int32), req_slot=torch.tensor([2, 0, 1, 3][:R], dtype=torch.int32),
                q_start=q_start, n_commit=torch.tensor(ncom, dtype=torch.int32),
                keep_pending=torch.tensor(keep, dtype=torch.int32))
    res = {}
    for dev in ("cpu", DEV):
        st, cs, px, pb = (t.clone().to(dev) for t in (state0, conv0, px0, pb0))
        out = torch.zeros(T, Hv * dv, dtype=torch.bfloat16, device=dev)
        gdn_step(qkvz.to(dev), ba.to(dev), Hk=Hk, Hv=Hv, dk=dk, dv=dv, eps=1e-6, state=st, conv_state=cs, pend_x=px,
                 pend_ba=pb, out=out, smem_state=mode.startswith("prefill"), **{k: v.to(dev) for k, v in w.items()},
                 **{k: v.to(dev) for k, v in meta.items()})
        res[dev] = [t.cpu() for t in (out, st, cs, px, pb)]
    c, g = res["cpu"], res[DEV]
    assert _rel(g[0].float(), c[0].float()) < 2e-2
    assert _rel(g[1].float(), c[1].float()) < 2e-2
    assert torch.equal(g[2], c[2])
    assert torch.equal(g[3], c[3])
    assert torch.equal(g[4], c[4])


def test_peer_wait_times_out_into_status():
    """Failure detection on the device without a fault: the consumer's wait on peer
    completion flags that nobody sets gives up after its budget, records the timeout in
    the status word and returns; the context stays usable."""
    dev = torch.device(DEV)
    x = torch.randn(4, 512, device=dev)
    w = torch.zeros(512, device=dev)
    flags = torch.zeros(8, dtype=torch.int32, device=dev)  # no rank ever publishes
    epoch = torch.ones(1, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    F.rmsnorm_quant(x, w, 1e-6, wait=(flags.data_ptr(), epoch, 2, 200), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 5  # kTimeoutPeerFlag
    y = (x * 2).sum()  # the device still works
    assert torch.isfinite(y)
