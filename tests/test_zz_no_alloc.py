"""The allocation-free attention entry point, called through its exported C symbol.

``oscar_paged_attention_noalloc`` is for callers that cannot allocate device memory
when they launch attention (allocator callbacks, runtimes that forbid cudaMalloc on
the serving path, fixed-footprint embedders): it takes the same inputs and outputs
as the regular entry points but keeps its split-KV partials in a fixed device array
inside the library.  This test checks its output against the regular entry points
on two calls in a row (with different inputs, so stale scratch contents would show).
It builds all of its inputs itself, so it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

from oscar_b200.kv import format as fmt
from oscar_b200.ops import attention as A
from oscar_b200.ops import functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"
P = ctypes.c_void_p
I = ctypes.c_int


class AttnParams(ctypes.Structure):
    _fields_ = [("q", P), ("k_fresh", P), ("v_fresh", P), ("Hq", I), ("Hk", I), ("D", I), ("scale", ctypes.c_float),
                ("kv_mode", I), ("pool", P), ("page_bytes", I), ("kc", P), ("vc", P), ("stage_k", P),
                ("stage_v", P), ("owner", P), ("stage_rows", I), ("block_tables", P), ("bt_stride", I),
                ("q_start", P), ("seq_lens", P), ("work", P), ("n_work", I), ("part_o", P), ("part_lse", P),
                ("status", P), ("stage_req_slot", P), ("stage_sink", I), ("stage_ring", I)]


class MergeParams(ctypes.Structure):
    _fields_ = [("part_o", P), ("part_lse", P), ("item_first", P), ("item_count", P), ("max_rb", I),
                ("tok_req", P), ("q_start", P), ("Hq", I), ("Hk", I), ("D", I), ("RvT", P), ("gate", P),
                ("gate_ld", ctypes.c_longlong), ("gate_hstride", I), ("out_bf16", P), ("out_i8", P),
                ("out_scale", P), ("T", I)]


def _so():
    import oscar_b200._C as C

    return ctypes.CDLL(C.__file__)


def _layout(cls):
    return [ctypes.sizeof(cls)] + [getattr(cls, name).offset for name, _ in cls._fields_]


def test_ctypes_mirror_matches_library_layout():
    """The structs above mirror csrc/params.h; the library reports its own compiled
    sizes and field offsets (``oscar_params_layout``), so a field added or moved in the
    header fails here instead of passing misaligned pointers."""
    fn = _so().oscar_params_layout
    fn.argtypes = [ctypes.POINTER(ctypes.c_longlong), I]
    fn.restype = I
    n = fn(None, 0)
    buf = (ctypes.c_longlong * n)()
    assert fn(buf, n) == n
    assert list(buf) == _layout(AttnParams) + _layout(MergeParams)


def _lib():
    fn = _so().oscar_paged_attention_noalloc
    fn.argtypes = [ctypes.POINTER(AttnParams), ctypes.POINTER(MergeParams), P]
    fn.restype = ctypes.c_int
    return fn


def _ptr(t):
    return None if t is None else t.data_ptr()


def _case(seed):
    torch.manual_seed(seed)
    Hq, Hk, D = 6, 1, 256
    seqs, qlens = [2000, 513, 1300], [4, 4, 4]
    nb = sum((s + 127) // 128 for s in seqs) + 2
    perm = torch.randperm(nb)
    bt = torch.zeros(len(seqs), max((s + 127) // 128 for s in seqs), dtype=torch.int32)
    k = 0
    for r, s in enumerate(seqs):
        n = (s + 127) // 128
        bt[r, :n] = perm[k:k + n]
        k += n
    pool = torch.zeros(nb, Hk, fmt.page_head_bytes(D), dtype=torch.uint8)
    kcod, vcod, ks, kz, vs, vz = fmt.page_views(pool, D)
    kcod.copy_(torch.randint(0, 256, kcod.shape, dtype=torch.uint8))
    vcod.copy_(torch.randint(0, 256, vcod.shape, dtype=torch.uint8))
    for t in (ks, vs):
        t.copy_((torch.rand(t.shape) * 0.5 + 0.2).half())
    for t in (kz, vz):
        t.copy_((-torch.rand(t.shape) - 0.3).half())
    T = sum(qlens)
    q = torch.randn(T, Hq, D).half()
    kf = torch.randn(T, Hk, D).half()
    vf = torch.randn(T, Hk, D).half()
    Rv = torch.linalg.qr(torch.randn(D, D)).Q.contiguous()
    gate_buf = torch.randn(T, Hq * 2 * D).to(torch.bfloat16)
    q_start = [0] + list(np.cumsum(qlens))
    return dict(Hq=Hq, Hk=Hk, D=D, seqs=seqs, q_start=q_start, bt=bt, pool=pool, q=q, kf=kf, vf=vf,
                RvT=Rv.t().contiguous(), gate_buf=gate_buf, T=T)


def _regular(c):
    d = lambda t: t.to(DEV)  # noqa: E731
    plan = A.plan_attention(c["q_start"], c["seqs"], c["Hq"] // c["Hk"], c["Hk"], F.num_sms(torch.device(DEV)), DEV)
    gb = d(c["gate_buf"])
    tok_req = torch.repeat_interleave(torch.arange(len(c["seqs"])), torch.tensor(np.diff(c["q_start"]))).to(torch.int32)
    dev_t = dict(q=d(c["q"]), kf=d(c["kf"]), vf=d(c["vf"]), pool=d(c["pool"]), bt=d(c["bt"]),
                 q_start=d(torch.tensor(c["q_start"], dtype=torch.int32)),
                 seqs=d(torch.tensor(c["seqs"], dtype=torch.int32)), tok_req=d(tok_req), RvT=d(c["RvT"]), gb=gb,
                 plan=plan)
    ob, oq, os_ = A.attention(dev_t["q"], dev_t["kf"], dev_t["vf"], Hq=c["Hq"], Hk=c["Hk"], D=c["D"], scale=1 / 16,
                              kv_mode=0, pool=dev_t["pool"], kc=None, vc=None, stage=None,
                              block_tables=dev_t["bt"], q_start_t=dev_t["q_start"], seq_lens_t=dev_t["seqs"],
                              q_start=c["q_start"], seq_lens=c["seqs"], plan=plan, tok_req=dev_t["tok_req"],
                              RvT=dev_t["RvT"], gate=gb[:, c["D"]:], gate_ld=gb.stride(0), gate_hstride=2 * c["D"],
                              want_bf16=True, want_q=True)
    return (ob, oq, os_), dev_t


def _noalloc(fn, c, t):
    T, Hq, D = c["T"], c["Hq"], c["D"]
    ob = torch.empty(T, Hq * D, dtype=torch.bfloat16, device=DEV)
    oq = torch.empty(T, Hq * D, dtype=torch.int8, device=DEV)
    os_ = torch.empty(T, dtype=torch.float32, device=DEV)
    plan = t["plan"]
    a = AttnParams(q=_ptr(t["q"]), k_fresh=_ptr(t["kf"]), v_fresh=_ptr(t["vf"]), Hq=Hq, Hk=c["Hk"], D=D,
                   scale=1 / 16, kv_mode=0, pool=_ptr(t["pool"]), page_bytes=t["pool"].shape[2], kc=None, vc=None,
                   stage_k=None, stage_v=None, owner=None, stage_rows=0, block_tables=_ptr(t["bt"]),
                   bt_stride=t["bt"].stride(0), q_start=_ptr(t["q_start"]), seq_lens=_ptr(t["seqs"]),
                   work=_ptr(plan.work), n_work=plan.n_work, part_o=None, part_lse=None, status=None)
    gb = t["gb"]
    m = MergeParams(part_o=None, part_lse=None, item_first=_ptr(plan.item_first), item_count=_ptr(plan.item_count),
                    max_rb=plan.max_rb, tok_req=_ptr(t["tok_req"]), q_start=_ptr(t["q_start"]), Hq=Hq, Hk=c["Hk"],
                    D=D, RvT=_ptr(t["RvT"]), gate=gb[:, D:].data_ptr(), gate_ld=gb.stride(0), gate_hstride=2 * D,
                    out_bf16=_ptr(ob), out_i8=_ptr(oq), out_scale=_ptr(os_), T=T)
    stream = torch.cuda.current_stream().cuda_stream
    rc = fn(ctypes.byref(a), ctypes.byref(m), ctypes.c_void_p(stream))
    assert rc == 0, f"oscar_paged_attention_noalloc returned {rc}"
    return ob, oq, os_


def _rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm().clamp(min=1e-30)).item()


def test_noalloc_matches_regular_entry_point_twice():
    fn = _lib()
    for seed in (11, 12):  # two calls in a row, different inputs
        c = _case(seed)
        (rb, rq, rs), t = _regular(c)
        nb, nq, ns = _noalloc(fn, c, t)
        torch.cuda.synchronize()
        assert _rel(nb.float(), rb.float()) < 1e-2
        assert (nq.int() - rq.int()).abs().max().item() <= 1
        assert torch.allclose(ns, rs, rtol=1e-2)


def test_noalloc_rejects_oversized_work():
    fn = _lib()
    a = AttnParams(Hq=6, Hk=1, D=256, n_work=100000)
    m = MergeParams(Hq=6, Hk=1, D=256, T=1)
    rc = fn(ctypes.byref(a), ctypes.byref(m), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == -310
