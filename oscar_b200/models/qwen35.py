"""Qwen3.5-shaped hybrid model on the oscar_b200 kernels (random init from a seed).

Layer stack (``config.HybridConfig``): gated DeltaNet layers and, every
``full_attention_interval`` layers, a gated full-attention layer whose KV cache is
OSCAR INT2 (rotated, clipped, 2-bit per-vector codes in 128-token pages with an fp32
sink/recent staging window).  All projections are W8A8 int8 GEMMs with per-channel
weight scales and per-token dynamic activation scales; the residual stream is fp32.
The MTP head (one full-attention layer with a BF16 KV "shadow" pool) drafts tokens
for speculative decoding.

Tensor parallelism: attention/GDN heads, the MLP intermediate dimension and the
vocabulary are split across ranks; o_proj / out_proj / down_proj are row-parallel
and their partial sums are all-reduced (NCCL baseline) before the fused
residual-add + RMSNorm kernel.

Reference parity: the OSCAR attention write/read semantics follow the reference
backend (``oscar_ascend/backend.py:129-189, 239-415``); everything else is the host
framework's model that the reference runs on (``delivery/serve_oscar.sh:76-99``).
"""
from __future__ import annotations

import contextlib
import math
from dataclasses import dataclass, field

import torch

from ..config import OscarConfig
from ..kv import format as fmt
from ..kv.oracle import arena_rows, window_layout
from ..kv.rotation import get_layer_rotation, random_orthogonal
from ..ops import attention as A
from ..ops import functional as F
from ..ops.gdn import gdn_step
from ..ops import sampling as samp
from ..parallel.fused import NcclRowReduce, make_row_reduce
from ..parallel.groups import TPGroup
from .config import HybridConfig
from .selection import AttentionSpec, beat, should_oscar

P_MAX = 4  # pending (uncommitted) tokens per GDN slot: 1 verified + 3 drafts


@dataclass
class QLinear:
    q: torch.Tensor  # int8 [N, K]
    s: torch.Tensor  # fp32 [N]

    def to(self, device):
        return QLinear(self.q.to(device), self.s.to(device))


@dataclass
class StepBatch:
    """Device metadata of one engine step (built on the host, uploaded once)."""

    tokens: torch.Tensor        # [T] int32
    positions: torch.Tensor     # [T] int32
    slots: torch.Tensor         # [T] int32 physical slot (block * 128 + offset), -1 = no write
    q_start: torch.Tensor       # [R + 1] int32
    seq_lens: torch.Tensor      # [R] int32 (including this step's tokens)
    block_tables: torch.Tensor  # [R, max_pages] int32
    tok_req: torch.Tensor       # [T] int32
    q_start_l: list
    seq_lens_l: list
    plan: A.AttnPlan | None
    stage_seat: torch.Tensor | None   # [T] int32
    owner_seat: torch.Tensor | None   # [n] int32
    owner_val: torch.Tensor | None    # [n] int32
    req_slot: torch.Tensor            # [R] int32 (GDN state slot)
    n_commit: torch.Tensor            # [R] int32
    keep_pending: torch.Tensor        # [R] int32
    parity: torch.Tensor              # [R] int32
    logit_rows: torch.Tensor          # [n_sel] int64
    extra: dict = field(default_factory=dict)

    @property
    def T(self) -> int:
        return int(self.tokens.shape[0])


_RANDOM_INIT = [True]


@contextlib.contextmanager
def no_random_init():
    """Inside this context the constructors allocate zero weights (unit scales) of the
    same shapes instead of drawing random ones: the model is about to be overwritten by
    a checkpoint, and drawing the random logical matrices of a 27B model first would
    cost more time than loading it."""
    _RANDOM_INIT.append(False)
    try:
        yield
    finally:
        _RANDOM_INIT.pop()


def _gen(seed: int, device) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _rand_qlinear(N: int, K: int, seed: int, device, rows=None, cols=None) -> QLinear:
    """Random int8 weight of the LOGICAL (unsharded) ``[N, K]`` matrix, then this rank's
    part: ``rows`` = list of ``(begin, end)`` row ranges (column-parallel) or ``cols`` =
    one ``(begin, end)`` column range (row-parallel; the per-row scale stays whole).  Every
    tensor-parallel size therefore holds slices of the same model."""
    if not _RANDOM_INIT[-1]:
        n = N if rows is None else sum(b - a for a, b in rows)
        k = K if cols is None else cols[1] - cols[0]
        return QLinear(torch.zeros(n, k, dtype=torch.int8, device=device),
                       torch.ones(n, dtype=torch.float32, device=device))
    g = _gen(seed, device)
    q = torch.randint(-127, 128, (N, K), dtype=torch.int8, generator=g, device=device)
    s = ((torch.rand(N, generator=g, device=device) * 0.5 + 0.75) / (73.3 * math.sqrt(K))).float()
    if rows is not None:
        q = torch.cat([q[a:b] for a, b in rows]).contiguous()
        s = torch.cat([s[a:b] for a, b in rows]).contiguous()
    if cols is not None:
        q = q[:, cols[0]:cols[1]].contiguous()
    return QLinear(q, s)


def _rand_vec(n: int, seed: int, device, std: float = 0.02, mean: float = 0.0) -> torch.Tensor:
    if not _RANDOM_INIT[-1]:
        return torch.full((n,), float(mean), dtype=torch.float32, device=device)
    g = _gen(seed, device)
    return (torch.randn(n, generator=g, device=device) * std + mean).float()


def _blocks(begin: int, end: int, width: int, offset: int = 0) -> tuple[int, int]:
    return offset + begin * width, offset + end * width


class FullAttentionLayer:
    """Gated full attention with OSCAR INT2 KV (or BF16 KV for the MTP draft layer)."""

    def __init__(self, cfg: HybridConfig, tp: TPGroup, layer_id: int, seed: int, device, oscar: OscarConfig,
                 kv_mode: str = "int2", rotation: str = "random"):
        H, D = cfg.hidden_size, cfg.head_dim
        self.layer_id = layer_id
        self.D = D
        self.Hq = cfg.num_attention_heads // tp.world
        if cfg.num_key_value_heads >= tp.world:
            self.Hk = cfg.num_key_value_heads // tp.world
        else:
            self.Hk = 1  # KV heads replicated across ranks (tp > num_key_value_heads)
        self.kv_mode = 0 if kv_mode == "int2" else 1
        self.scale = 1.0 / math.sqrt(D)
        self.eps = cfg.rms_norm_eps
        self.rot_dim = cfg.rot_dim
        self.q_off = 0
        self.q_head_stride = 2 * D  # per head: [query (D) | gate (D)]
        self.k_off = self.Hq * 2 * D
        self.v_off = self.k_off + self.Hk * D
        self.n_qkv = self.v_off + self.Hk * D
        base = seed * 1000 + layer_id * 17
        nq, nk = cfg.num_attention_heads, cfg.num_key_value_heads
        h0 = tp.rank * self.Hq
        k0 = (tp.rank * nk) // tp.world if nk < tp.world else tp.rank * self.Hk
        self.h0, self.k0 = h0, k0  # first query / KV head of this rank (checkpoint loading)
        kv_base = nq * 2 * D
        self.qkv = _rand_qlinear(nq * 2 * D + 2 * nk * D, H, base + 1, device, rows=[
            _blocks(h0, h0 + self.Hq, 2 * D), _blocks(k0, k0 + self.Hk, D, kv_base),
            _blocks(k0, k0 + self.Hk, D, kv_base + nk * D)])
        self.o = _rand_qlinear(H, nq * D, base + 2, device, cols=_blocks(h0, h0 + self.Hq, D))
        self.q_norm = _rand_vec(D, base + 3, device)
        self.k_norm = _rand_vec(D, base + 4, device)
        self.input_norm = _rand_vec(H, base + 5, device)
        self.post_norm = _rand_vec(H, base + 6, device)
        self.k_clip_idx = oscar.clip_index(oscar.k_clip_ratio) if (self.kv_mode == 0 and oscar.k_clip_ratio > 0) else -1
        self.v_clip_idx = oscar.clip_index(oscar.v_clip_ratio) if (self.kv_mode == 0 and oscar.v_clip_ratio > 0) else -1
        if self.kv_mode == 0:
            if rotation == "identity":
                self.Rk = self.Rv = self.RvT = None
            elif rotation == "random":
                self.Rk = random_orthogonal(D, seed * 7919 + layer_id * 2).to(device)
                self.Rv = random_orthogonal(D, seed * 7919 + layer_id * 2 + 1).to(device)
                self.RvT = self.Rv.t().contiguous()
            else:  # checkpoint path (v2 oscar_rotations.pt)
                self.Rk = get_layer_rotation(oscar.k_rotation_path or rotation, layer_id, D, device, mode="k",
                                             strict=True)
                self.Rv = get_layer_rotation(oscar.v_rotation_path or rotation, layer_id, D, device, mode="v",
                                             strict=True)
                self.RvT = self.Rv.t().contiguous()
        else:
            self.Rk = self.Rv = self.RvT = None
        self._split_rotations()
        self.calib = None  # CalibrationCapture while calibrating rotations
        self.pool = self.kc = self.vc = None
        self.stage_k = self.stage_v = None

    def _split_rotations(self):
        self.rk_split = A.split_rotation(self.Rk)
        self.rv_split = A.split_rotation(self.Rv)
        self.rv_merge_split = A.split_rotation(self.RvT)

    def to(self, device):
        for k, v in list(vars(self).items()):
            if isinstance(v, torch.Tensor):
                setattr(self, k, v.to(device))
            elif isinstance(v, QLinear):
                setattr(self, k, v.to(device))
        self._split_rotations()
        return self

    def allocate_cache(self, num_blocks: int, device, stage_rows: int = 0):
        if self.kv_mode == 0:
            self.pool = torch.zeros(num_blocks, self.Hk, fmt.page_head_bytes(self.D), dtype=torch.uint8,
                                    device=device)
            if stage_rows:
                self.stage_k = torch.zeros(stage_rows * fmt.PAGE, self.Hk, self.D, dtype=torch.float32,
                                           device=device)
                # V staging is dim-major per row (the attention kernels read one dim's
                # 128 tokens contiguously)
                self.stage_v = torch.zeros(stage_rows, self.Hk, self.D, fmt.PAGE, dtype=torch.float32,
                                           device=device)
        else:
            self.kc = torch.zeros(num_blocks, fmt.PAGE, self.Hk, self.D, dtype=torch.bfloat16, device=device)
            self.vc = torch.zeros_like(self.kc)

    def cache_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.pool, self.kc, self.vc, self.stage_k, self.stage_v)
                   if t is not None)

    def attention(self, xq, xs, b: StepBatch, rope, owner, stage_rows, write_owner: bool, status=None,
                  stage_layout=None):
        """qkv GEMM -> fused store -> paged attention -> merge. Returns (o_int8, o_scale)."""
        T = xq.shape[0]
        if self.kv_mode == 0:
            beat()
        dev = xq.device
        qkv = F.linear_i8(xq, xs, self.qkv.q, self.qkv.s, status=status)
        q_out = torch.empty(T, self.Hq, self.D, dtype=torch.float16, device=dev)
        k_fr = torch.empty(T, self.Hk, self.D, dtype=torch.float16, device=dev)
        v_fr = torch.empty_like(k_fr)
        staged = self.kv_mode == 0 and stage_rows > 0 and b.stage_seat is not None
        A.kv_store(qkv, q_off=self.q_off, q_head_stride=self.q_head_stride, k_off=self.k_off, v_off=self.v_off,
                   Hq=self.Hq, Hk=self.Hk, D=self.D, q_norm_w=self.q_norm, k_norm_w=self.k_norm, eps=self.eps,
                   norm_offset=1.0, positions=b.positions, rope_cos=rope[0], rope_sin=rope[1], rot_dim=self.rot_dim,
                   Rk=self.Rk, Rv=self.Rv, k_clip_idx=self.k_clip_idx, v_clip_idx=self.v_clip_idx, q_out=q_out,
                   k_fresh=k_fr, v_fresh=v_fr, kv_mode=self.kv_mode, pool=self.pool, kc=self.kc, vc=self.vc,
                   slots=b.slots, stage_k=self.stage_k if staged else None,
                   stage_v=self.stage_v if staged else None, stage_seat=b.stage_seat if staged else None,
                   owner=owner if staged else None,
                   owner_seat=b.owner_seat if (staged and write_owner) else None,
                   owner_val=b.owner_val if (staged and write_owner) else None, status=status,
                   rk_split=self.rk_split, rv_split=self.rv_split)
        if self.calib is not None:  # rotation calibration: unquantised q / k / v of this layer
            self.calib.record(f"model.layers.{self.layer_id}.self_attn.attn", q_out, k_fr, v_fr, self.Hq, self.Hk,
                              self.D)
        stage = None
        if staged:
            lay = None if stage_layout is None else (b.req_slot, stage_layout[0], stage_layout[1])
            stage = (self.stage_k, self.stage_v, owner, stage_rows, lay)
        gate = qkv[:, self.D:]  # gate of head h at columns h * 2D + D ..
        _, oq, os_ = A.attention(q_out, k_fr, v_fr, Hq=self.Hq, Hk=self.Hk, D=self.D, scale=self.scale,
                                 kv_mode=self.kv_mode, pool=self.pool, kc=self.kc, vc=self.vc, stage=stage,
                                 block_tables=b.block_tables, q_start_t=b.q_start, seq_lens_t=b.seq_lens,
                                 q_start=b.q_start_l, seq_lens=b.seq_lens_l, plan=b.plan, tok_req=b.tok_req,
                                 RvT=self.RvT, gate=gate, gate_ld=qkv.stride(0), gate_hstride=2 * self.D,
                                 want_bf16=False, want_q=True, status=status,
                                 rv_merge_split=self.rv_merge_split)
        return oq, os_


class GDNLayer:
    """Gated DeltaNet mixer (linear attention) with deferred speculative commit."""

    def __init__(self, cfg: HybridConfig, tp: TPGroup, layer_id: int, seed: int, device):
        H = cfg.hidden_size
        self.layer_id = layer_id
        self.Hk = cfg.linear_num_key_heads // tp.world
        self.Hv = cfg.linear_num_value_heads // tp.world
        self.dk, self.dv = cfg.linear_key_head_dim, cfg.linear_value_head_dim
        self.r = self.Hv // self.Hk
        self.eps = cfg.rms_norm_eps
        self.n_qkvz = self.Hk * (2 * self.dk + 2 * self.r * self.dv)
        self.n_ba = 2 * self.Hv
        self.conv_dim = 2 * self.Hk * self.dk + self.Hv * self.dv
        base = seed * 1000 + layer_id * 17
        nk, nv = cfg.linear_num_key_heads, cfg.linear_num_value_heads
        k0, v0 = tp.rank * self.Hk, tp.rank * self.Hv
        self.k0, self.v0 = k0, v0  # first key / value head of this rank (checkpoint loading)
        grp = 2 * self.dk + 2 * self.r * self.dv
        # logical rows: [qkvz grouped per key head | ba grouped per key head]
        self.inp = _rand_qlinear(nk * grp + 2 * nv, H, base + 1, device, rows=[
            _blocks(k0, k0 + self.Hk, grp), _blocks(k0, k0 + self.Hk, 2 * self.r, nk * grp)])
        # zero output rows up to a multiple of 8: the projection's rows stay 16-byte
        # aligned (bf16), which the chunked prefill kernels' vector loads need at every TP size
        pad = -self.inp.q.shape[0] % 8
        if pad:
            self.inp = QLinear(torch.cat([self.inp.q, self.inp.q.new_zeros(pad, H)]).contiguous(),
                               torch.cat([self.inp.s, self.inp.s.new_ones(pad)]).contiguous())
        self.out = _rand_qlinear(H, nv * self.dv, base + 2, device, cols=_blocks(v0, v0 + self.Hv, self.dv))
        g = _gen(base + 3, device)
        Kd = nk * self.dk
        conv_full = torch.randn(2 * Kd + nv * self.dv, cfg.linear_conv_kernel_dim, generator=g, device=device) * 0.5
        # conv channels: [q heads | k heads | v heads]
        self.conv_w = torch.cat([conv_full[k0 * self.dk:(k0 + self.Hk) * self.dk],
                                 conv_full[Kd + k0 * self.dk:Kd + (k0 + self.Hk) * self.dk],
                                 conv_full[2 * Kd + v0 * self.dv:2 * Kd + (v0 + self.Hv) * self.dv]]).float().contiguous()
        self.A_log = torch.log(torch.rand(nv, generator=g, device=device) * 15 + 1)[v0:v0 + self.Hv].float().contiguous()
        self.dt_bias = torch.ones(self.Hv, device=device).float()
        self.norm_w = (1.0 + torch.randn(self.dv, generator=g, device=device) * 0.02).float()
        self.input_norm = _rand_vec(H, base + 5, device)
        self.post_norm = _rand_vec(H, base + 6, device)
        self.state = self.conv_state = self.pend_x = self.pend_ba = None

    def to(self, device):
        for k, v in list(vars(self).items()):
            if isinstance(v, torch.Tensor):
                setattr(self, k, v.to(device))
            elif isinstance(v, QLinear):
                setattr(self, k, v.to(device))
        return self

    def allocate_cache(self, slots: int, device):
        self.state = torch.zeros(slots, self.Hv, self.dk, self.dv, dtype=torch.bfloat16, device=device)
        self.conv_state = torch.zeros(2, slots, self.conv_dim, 3, dtype=torch.bfloat16, device=device)
        self.pend_x = torch.zeros(2, slots, P_MAX, self.conv_dim, dtype=torch.bfloat16, device=device)
        self.pend_ba = torch.zeros(slots, P_MAX, 2 * self.Hv, dtype=torch.bfloat16, device=device)

    def cache_bytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.state, self.conv_state, self.pend_x, self.pend_ba)
                   if t is not None)

    def mixer(self, xq, xs, b: StepBatch, status=None):
        proj = F.linear_i8(xq, xs, self.inp.q, self.inp.s, status=status)
        T = proj.shape[0]
        o = torch.empty(T, self.Hv * self.dv, dtype=torch.bfloat16, device=proj.device)
        gdn_step(proj[:, :self.n_qkvz], proj[:, self.n_qkvz:self.n_qkvz + self.n_ba], Hk=self.Hk, Hv=self.Hv, dk=self.dk, dv=self.dv,
                 conv_w=self.conv_w, A_log=self.A_log, dt_bias=self.dt_bias, norm_w=self.norm_w, eps=self.eps,
                 state=self.state, conv_state=self.conv_state, pend_x=self.pend_x, pend_ba=self.pend_ba,
                 parity=b.parity, req_slot=b.req_slot, q_start=b.q_start, n_commit=b.n_commit,
                 keep_pending=b.keep_pending, out=o, smem_state=b.extra.get("max_qlen", T) > 4, status=status)
        return F.act_quant(o)


class MLP:
    def __init__(self, cfg: HybridConfig, tp: TPGroup, layer_id: int, seed: int, device):
        H = cfg.hidden_size
        self.I = cfg.intermediate_size // tp.world
        base = seed * 1000 + layer_id * 17 + 50
        I_full = cfg.intermediate_size
        i0 = tp.rank * self.I
        self.i0 = i0  # first intermediate column of this rank (checkpoint loading)
        self.gate_up = _rand_qlinear(2 * I_full, H, base + 1, device, rows=[
            (i0, i0 + self.I), (I_full + i0, I_full + i0 + self.I)])
        self.down = _rand_qlinear(H, I_full, base + 2, device, cols=(i0, i0 + self.I))

    def to(self, device):
        self.gate_up = self.gate_up.to(device)
        self.down = self.down.to(device)
        return self


class HybridModel:
    """The full model of one tensor-parallel rank."""

    def __init__(self, cfg: HybridConfig, tp: TPGroup | None = None, device="cpu", seed: int = 0,
                 oscar: OscarConfig | None = None, kv_mode: str = "int2", rotation: str = "random",
                 mtp: bool = True):
        self.cfg = cfg
        self.tp = tp or TPGroup()
        self.device = torch.device(device)
        self.oscar = oscar or OscarConfig().validate()
        self.kv_mode = kv_mode
        H = cfg.hidden_size
        V = cfg.vocab_size
        self.V_local = (V + self.tp.world - 1) // self.tp.world
        self.vocab_begin = self.tp.rank * self.V_local
        dev = self.device
        base = seed * 1000
        g = _gen(base + 999, dev)
        v0, v1 = self.vocab_begin, min(V, self.vocab_begin + self.V_local)
        emb = torch.zeros(self.V_local, H, dtype=torch.bfloat16, device=dev)
        if _RANDOM_INIT[-1]:
            emb[:v1 - v0] = (torch.randn(V, H, generator=g, device=dev) * 0.02)[v0:v1].to(torch.bfloat16)
        self.embed = emb
        self.lm_head = _rand_qlinear(V, H, base + 998, dev, rows=[(v0, v1)])  # only real vocab rows
        self.final_norm = _rand_vec(H, base + 997, dev)
        self.layers = []
        for i, t in enumerate(cfg.layer_types):
            if t == "full_attention":
                lkv = kv_mode if should_oscar(AttentionSpec(i), cfg) else "bf16"
                mixer = FullAttentionLayer(cfg, self.tp, i, seed, dev, self.oscar, lkv, rotation)
            else:
                mixer = GDNLayer(cfg, self.tp, i, seed, dev)
            self.layers.append((mixer, MLP(cfg, self.tp, i, seed, dev)))
        self.mtp = MTPHead(self, seed) if (mtp and cfg.num_mtp_layers > 0) else None
        self.rope = F.rope_tables(cfg.max_position, cfg.rot_dim, cfg.rope_theta, dev, cfg.rope_scaling)
        self.stage_rows = 0
        self.stage_layout = None
        self.owner = None
        self.status = torch.zeros(1, dtype=torch.int32, device=dev) if dev.type == "cuda" else None

    # ------------------------------------------------------------------ setup
    def to(self, device):
        self.device = torch.device(device)
        self.embed = self.embed.to(device)
        self.lm_head = self.lm_head.to(device)
        self.final_norm = self.final_norm.to(device)
        for mixer, mlp in self.layers:
            mixer.to(device)
            mlp.to(device)
        if self.mtp is not None:
            self.mtp.to(device)
        self.rope = (self.rope[0].to(device), self.rope[1].to(device))
        if self.owner is not None:
            self.owner = self.owner.to(device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device) if self.device.type == "cuda" else None
        return self

    @property
    def full_layers(self):
        return [m for m, _ in self.layers if isinstance(m, FullAttentionLayer)]

    @property
    def gdn_layers(self):
        return [m for m, _ in self.layers if isinstance(m, GDNLayer)]

    def allocate_cache(self, num_blocks: int, max_slots: int):
        o = self.oscar
        int2 = any(m.kv_mode == 0 for m in self.full_layers)
        self.stage_rows = arena_rows(o.sink_tokens, o.recent_tokens, o.staging_tokens, o.staging_layout,
                                     max_slots) if (o.window_enabled and int2) else 0
        # (sink_pages, ring) of the per-request window layout, None for the hashed arena
        self.stage_layout = window_layout(o.sink_tokens, o.recent_tokens) if (
            self.stage_rows and o.staging_layout == "window") else None
        if self.stage_rows:
            self.owner = torch.full((self.stage_rows * fmt.PAGE,), -1, dtype=torch.int32, device=self.device)
        for m in self.full_layers:
            m.allocate_cache(num_blocks, self.device, self.stage_rows)
        for m in self.gdn_layers:
            m.allocate_cache(max_slots, self.device)
        if self.mtp is not None:
            self.mtp.layer.allocate_cache(num_blocks, self.device)

    def reset_state_slots(self, slots: list) -> None:
        """Zero the recurrent state and conv window of GDN state slots taken by new
        requests: the kernels start a request from ``state[slot]`` and the conv window of
        the slot, which still hold the previous occupant's."""
        if not slots:
            return
        idx = torch.as_tensor(list(slots), dtype=torch.long).to(self.device)
        for m in self.gdn_layers:
            m.state.index_fill_(0, idx, 0)
            m.conv_state.index_fill_(1, idx, 0)

    def cache_bytes(self) -> dict:
        full = sum(m.cache_bytes() for m in self.full_layers)
        gdn = sum(m.cache_bytes() for m in self.gdn_layers)
        shadow = self.mtp.layer.cache_bytes() if self.mtp is not None else 0
        return {"full_kv": full, "gdn_state": gdn, "mtp_shadow": shadow,
                "owner": 0 if self.owner is None else self.owner.numel() * 4}

    # ------------------------------------------------------------------ forward
    def setup_row_reduce(self, max_rows: int) -> None:
        """Choose the row-parallel reduction: fused GEMM + NVLS all-reduce on CUDA TP
        groups that support multicast, else GEMM + NCCL all-reduce."""
        self.row_reduce = make_row_reduce(self.tp, max_rows, self.cfg.hidden_size, self.device)

    def _reducer(self):
        if getattr(self, "row_reduce", None) is None:
            self.row_reduce = NcclRowReduce(self.tp)
        return self.row_reduce

    def decoder(self, b: StepBatch, residual: torch.Tensor) -> dict:
        """All decoder layers over the residual rows this rank keeps (all rows, or its own
        rows under sequence parallelism); returns the pending reduction of the last MLP,
        which the final norm consumes."""
        red = self._reducer()
        eps = self.cfg.rms_norm_eps
        pending: dict | None = None
        first_full = True
        k = 0
        for mixer, mlp in self.layers:
            xq, xs, _ = red.norm(residual, mixer.input_norm, eps, pending, status=self.status)
            if isinstance(mixer, FullAttentionLayer):
                oq, os_ = mixer.attention(xq, xs, b, self.rope, self.owner, self.stage_rows,
                                          write_owner=first_full, status=self.status,
                                          stage_layout=self.stage_layout)
                first_full = False
                w_o = mixer.o
            else:
                oq, os_ = mixer.mixer(xq, xs, b, status=self.status)
                w_o = mixer.out
            pending = red.gemm(oq, os_, w_o, k, status=self.status)
            xq, xs, _ = red.norm(residual, mixer.post_norm, eps, pending, status=self.status)
            gu = F.linear_i8(xq, xs, mlp.gate_up.q, mlp.gate_up.s, status=self.status)
            hq, hs = F.swiglu_quant(gu, mlp.I)
            pending = red.gemm(hq, hs, mlp.down, k + 1, status=self.status)
            k += 2
        return pending

    def forward(self, b: StepBatch):
        """Main model on a step.  Returns ``(hidden_bf16 [T, H], next_tokens [n_sel])``."""
        T = b.T
        H = self.cfg.hidden_size
        red = self._reducer()
        red.begin(T, H, self.device)
        residual = red.embed_in(b.tokens, self.embed, self.vocab_begin)
        pending = self.decoder(b, residual)
        xq, xs, hid = red.norm(residual, self.final_norm, self.cfg.rms_norm_eps, pending, want_bf16=True,
                               status=self.status)
        rows = b.logit_rows
        tok = self.sample(xq[rows], xs[rows], b.extra.get("sampling"), b.extra.get("logprobs_k"))
        return hid, tok

    def sample(self, xq, xs, rows: "samp.SampleRows | None" = None, logprobs_k: int | None = None) -> torch.Tensor:
        """Tokens over the vocab-parallel lm_head: greedy (global argmax across ranks), or,
        with ``rows``, per-row temperature / top-k / top-p sampling and draft verification.
        With ``logprobs_k`` the chosen tokens' log-probabilities and the ``logprobs_k`` most
        likely tokens of every row are left in ``self.last_logprobs``."""
        logits = F.linear_i8(xq, xs, self.lm_head.q, self.lm_head.s, status=self.status)
        if rows is not None:
            tok = samp.sample(logits, self.vocab_begin, rows, self.tp)
        else:
            tok = self._greedy(logits)
        if logprobs_k is not None:
            self.last_logprobs = samp.logprobs(logits, self.vocab_begin, tok, logprobs_k, self.tp)
        return tok

    def _greedy(self, logits) -> torch.Tensor:
        v, i = F.argmax(logits, self.vocab_begin)
        if self.tp.world > 1:
            vs = self.tp.all_gather(v.unsqueeze(0))      # [world, n]
            ids = self.tp.all_gather(i.unsqueeze(0))
            best = vs.argmax(dim=0)
            i = ids.gather(0, best.unsqueeze(0)).squeeze(0)
        return i


class MTPHead:
    """One-layer multi-token-prediction head (shares the embedding and lm_head)."""

    def __init__(self, model: HybridModel, seed: int):
        cfg = model.cfg
        tp = model.tp
        dev = model.device
        H = cfg.hidden_size
        lid = cfg.num_layers  # layer id after the main stack
        base = seed * 1000 + lid * 17 + 7
        self.model = model
        self.fc = _rand_qlinear(H, 2 * H, base + 1, dev)  # replicated (small)
        self.norm_emb = _rand_vec(H, base + 2, dev)
        self.norm_hid = _rand_vec(H, base + 3, dev)
        self.final_norm = _rand_vec(H, base + 4, dev)
        self.layer = FullAttentionLayer(cfg, tp, lid, seed, dev, model.oscar, kv_mode="bf16")
        self.mlp = MLP(cfg, tp, lid, seed, dev)

    def to(self, device):
        for name in ("fc",):
            setattr(self, name, getattr(self, name).to(device))
        self.norm_emb = self.norm_emb.to(device)
        self.norm_hid = self.norm_hid.to(device)
        self.final_norm = self.final_norm.to(device)
        self.layer.to(device)
        self.mlp.to(device)
        return self

    def forward(self, b: StepBatch, hidden: torch.Tensor, tokens: torch.Tensor | None = None):
        """Draft pass: ``hidden`` [T, H] bf16 (post-norm main or previous draft hidden),
        ``tokens`` (default ``b.tokens``) = the next token of every position, may be a
        device tensor produced by the previous pass.  Returns (hidden_bf16, next_tokens)."""
        m = self.model
        cfg = m.cfg
        T, H = hidden.shape
        eps = cfg.rms_norm_eps
        e = torch.empty(T, H, dtype=torch.float32, device=m.device)
        F.embed(b.tokens if tokens is None else tokens, m.embed, m.vocab_begin, e)
        m.tp.all_reduce_(e)
        _, _, e_n = F.rmsnorm_quant(e, self.norm_emb, eps, want_q=False, want_bf16=True)
        hf = hidden.float().contiguous()
        _, _, h_n = F.rmsnorm_quant(hf, self.norm_hid, eps, want_q=False, want_bf16=True)
        cat = torch.cat([e_n, h_n], dim=1)
        cq, cs = F.act_quant(cat)
        red = m._reducer()
        red.begin(T, H, m.device)
        # the fc projection is replicated: each rank computes the residual rows it keeps
        residual = red.fc_rows(cq, cs, self.fc, m.status)
        xq, xs, _ = red.norm(residual, self.layer.input_norm, eps, None, status=m.status)
        oq, os_ = self.layer.attention(xq, xs, b, m.rope, None, 0, write_owner=False, status=m.status)
        pending = red.gemm(oq, os_, self.layer.o, 0, status=m.status)
        xq, xs, _ = red.norm(residual, self.layer.post_norm, eps, pending, status=m.status)
        gu = F.linear_i8(xq, xs, self.mlp.gate_up.q, self.mlp.gate_up.s, status=m.status)
        hq, hs = F.swiglu_quant(gu, self.mlp.I)
        pending = red.gemm(hq, hs, self.mlp.down, 1, status=m.status)
        xq, xs, hid = red.norm(residual, self.final_norm, eps, pending, want_bf16=True, status=m.status)
        rows = b.logit_rows
        tok = m.sample(xq[rows], xs[rows])
        return hid, tok
