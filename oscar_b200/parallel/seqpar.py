"""Sequence-parallel tensor parallelism: reduce-scatter fused into the row-parallel
GEMMs, all-gather fused into the RMSNorm that feeds the column-parallel GEMMs.

The baseline (:class:`oscar_b200.parallel.fused.NcclRowReduce`) keeps the whole fp32
residual stream ``[T, H]`` on every rank: each row-parallel projection (attention
``o_proj``, GDN ``out_proj``, MLP ``down_proj``) writes a partial sum that NCCL
all-reduces (``2 x 4`` bytes per element over NVLink), and every rank then normalises
all ``T`` rows.  The reference runs the same projections under vLLM-Ascend's
row-parallel linear layers with HCCL all-reduces (``delivery/serve_oscar.sh:81``).

Here rank ``r`` owns the token rows ``[r * Tl, (r + 1) * Tl)`` (``Tl = ceil(T / W)``)
of the residual stream:

* **reduce-scatter in the GEMM epilogue** (``gemm_i8_rs``, epilogue mode 5): each
  output tile's split-K slices are summed through the thread-block cluster's
  distributed shared memory, then every fp32 row of token ``t`` is stored with 16-byte
  stores straight into this rank's slot of the owner's receive buffer over NVLink (peer
  pointers of one symmetric-memory allocation), while other tiles are still on the
  tensor cores; the last CTA publishes an epoch into slot ``rank`` of every rank's
  signal pad;
* **RMSNorm + all-gather** (``rmsnorm_ag``): the owner waits (bounded) for all ranks'
  reduce-scatter epochs, adds the ``W`` slots of its rows in rank order (the same sum
  on every run) into its residual rows, normalises and quantises them and stores the
  int8 rows + scales (and
  the bf16 rows of the final norm) into the same rows of every rank's full-height
  activation buffer - the all-gather, pushed as rows are produced - then publishes its
  all-gather epoch;
* the consuming column-parallel GEMM (qkv, GDN in-projection, gate_up, lm_head) is
  launched as a programmatic dependent of a one-warp ``wait_flags`` kernel: its CTAs
  set up TMEM and stream their first weight tiles while the gather is in flight and
  read the gathered activations only after every rank's epoch arrived.

Bytes over NVLink per projection and rank: ``(W-1)/W * T * H * 4`` (reduce-scatter)
plus ``(W-1)/W * T * H`` (int8 all-gather), against ``2 (W-1)/W * T * H * 4`` for the
fp32 all-reduce; RMSNorm work is divided by ``W``.

Buffer reuse needs no double buffering: a rank stores into a peer's receive slot for
projection ``k+1`` only after its own column GEMM consumed all-gather ``k``, which
every rank publishes after reading its receive slots for ``k``; a rank overwrites a
peer's activation rows for norm ``k+1`` only after all ranks' reduce-scatter ``k+1``
arrived, which each rank issues after its GEMM read the rows of norm ``k``.  The first
norm of a pass has no reduce-scatter before it; the NCCL collective that starts every
pass (embedding reduce-scatter / all-reduce) and the one that ends it (the greedy
sampler's all-gather) order those.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import functional as F
from ..ops._ext import ext
from .groups import TPGroup

WAIT_BUDGET_NS = 5_000_000_000


def _round_up(x: int, m: int) -> int:
    return (x + m - 1) // m * m


class SeqParallelTP:
    """Residual stream sharded by token rows over the TP group (see module docstring)."""

    fused = True
    seq_parallel = True

    def __init__(self, tp: TPGroup, max_rows: int, H: int, device):
        import torch.distributed._symmetric_memory as symm

        if tp.world < 2 or tp.world > 8:
            raise ValueError("sequence-parallel TP needs 2..8 ranks")
        self.tp = tp
        self.W = W = tp.world
        self.H = H
        self.device = torch.device(device)
        self.Tp_max = _round_up(max(max_rows, W), W)
        self.Tl_max = self.Tp_max // W
        # one symmetric allocation: [recv fp32 W slots x Tl_max x H | xq int8 Tp_max x H | xs fp32 Tp_max |
        #                            hid bf16 Tp_max x H]
        self.off_delta = 0
        self.slot_stride = self.Tl_max * H
        self.off_xq = _round_up(W * self.Tl_max * H * 4, 256)
        self.off_xs = _round_up(self.off_xq + self.Tp_max * H, 256)
        self.off_hid = _round_up(self.off_xs + self.Tp_max * 4, 256)
        total = _round_up(self.off_hid + self.Tp_max * H * 2, 256)
        group = tp.group if tp.group is not None else dist.group.WORLD
        self.buf = symm.empty(total, dtype=torch.uint8, device=self.device)
        self.hdl = symm.rendezvous(self.buf, group)
        self.buf.zero_()
        me = self.hdl.rank
        self.delta = self.buf[self.off_delta:self.off_delta + W * self.Tl_max * H * 4].view(torch.float32).view(
            W * self.Tl_max, H)
        self.xq = self.buf[self.off_xq:self.off_xq + self.Tp_max * H].view(torch.int8).view(self.Tp_max, H)
        self.xs = self.buf[self.off_xs:self.off_xs + self.Tp_max * 4].view(torch.float32)
        self.hid = self.buf[self.off_hid:self.off_hid + self.Tp_max * H * 2].view(torch.bfloat16).view(self.Tp_max, H)
        ptrs = [int(p) for p in self.hdl.buffer_ptrs]
        pads = [int(p) for p in self.hdl.signal_pad_ptrs]
        pad = self.hdl.get_signal_pad(me, (2 * W,), dtype=torch.int32)
        pad.zero_()
        self.rs_wait_ptr = pads[me]                    # slots [0, W): reduce-scatter epochs
        self.ag_wait_ptr = pads[me] + 4 * W            # slots [W, 2W): all-gather epochs
        self.xq_ptrs = [p + self.off_xq for p in ptrs]
        self.xs_ptrs = [p + self.off_xs for p in ptrs]
        self.hid_ptrs = [p + self.off_hid for p in ptrs]
        self.ag_slots = [p + 4 * (W + me) for p in pads]
        self.peer_delta = torch.tensor([p + self.off_delta for p in ptrs], dtype=torch.int64, device=self.device)
        self.peer_rs_pads = torch.tensor(pads, dtype=torch.int64, device=self.device)
        # local state
        self.residual = torch.zeros(self.Tl_max, H, dtype=torch.float32, device=self.device)
        self.ws = torch.zeros(self.Tp_max, H, dtype=torch.float32, device=self.device)
        self.tile_cnt = torch.zeros(1 << 16, dtype=torch.int32, device=self.device)
        self.rs_done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.rs_epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.ag_done = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.ag_epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._embed = torch.zeros(self.Tp_max, H, dtype=torch.float32, device=self.device)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)
        self.T = 0

    # ------------------------------------------------------------------ rows
    def begin(self, T: int, H: int, device) -> None:
        if T > self.Tp_max or H != self.H:
            raise ValueError(f"sequence-parallel buffers hold {self.Tp_max}x{self.H} rows, step needs {T}x{H}")
        self.T = T
        self.Tl = max(1, (T + self.W - 1) // self.W)
        r = self.tp.rank
        self.row0 = min(T, r * self.Tl)
        self.own = max(0, min(T, (r + 1) * self.Tl) - self.row0)

    def embed_in(self, tokens: torch.Tensor, table: torch.Tensor, vocab_begin: int) -> torch.Tensor:
        """Vocab-parallel embedding rows, reduce-scattered (NCCL) into this rank's rows."""
        Tp = self.Tl * self.W
        e = self._embed[:Tp]
        if Tp > self.T:
            e[self.T:].zero_()
        F.embed(tokens, table, vocab_begin, e[:self.T])
        res = self.residual[:self.Tl]
        dist.reduce_scatter_tensor(res, e, group=self.tp.group)
        return res

    def from_replicated(self, full: torch.Tensor) -> torch.Tensor:
        """This rank's rows of a residual every rank computed in full."""
        res = self.residual[:self.Tl]
        if self.own:
            res[:self.own].copy_(full[self.row0:self.row0 + self.own])
        return res

    def fc_rows(self, xq, xs, w, status=None) -> torch.Tensor:
        """A replicated projection (the MTP head's fc) computed for this rank's rows only."""
        res = self.residual[:self.Tl]
        res.zero_()
        if self.own:
            F.linear_i8(xq[self.row0:self.row0 + self.own], xs[self.row0:self.row0 + self.own], w.q, w.s,
                        out=res[:self.own], accumulate=True, status=status)
        return res

    # ------------------------------------------------------------------ fused collectives
    def norm(self, residual: torch.Tensor, w: torch.Tensor, eps: float, pending: dict | None = None,
             want_bf16: bool = False, status=None):
        """RMSNorm of the owned rows (after adding the reduce-scattered delta when
        ``pending``) with the all-gather; returns full-height ``(xq [T,H], xs [T],
        hid [T,H] bf16 or None)`` once every rank's rows are in."""
        e = ext()
        rs = bool(pending)
        e.rmsnorm_ag(residual, self.delta if rs else None, self.W, self.slot_stride, w, 1.0, float(eps), self.own,
                     self.row0, self.xq_ptrs,
                     self.xs_ptrs, self.hid_ptrs if want_bf16 else [], self.ag_slots, self.ag_done, self.ag_epoch,
                     self.rs_wait_ptr if rs else 0, self.rs_epoch if rs else None, status, WAIT_BUDGET_NS)
        e.wait_flags(self.ag_wait_ptr, self.ag_epoch, self.W, status, WAIT_BUDGET_NS)
        T = self.T
        return self.xq[:T], self.xs[:T], (self.hid[:T] if want_bf16 else None)

    def gemm(self, xq, xs, w, k: int = 0, status=None) -> dict:
        """Row-parallel projection; its result is reduce-scattered into the owners' rows."""
        M, K = xq.shape
        N = w.q.shape[0]
        plan = F.plan_gemm(M, N, K, F.num_sms(xq.device), allow_split=True)
        e = ext()
        if plan.swap:
            e.gemm_i8_rs(w.q, xq, w.s, xs, 1, plan.bn, plan.splits, int(self.peer_delta.data_ptr()), self.Tl, self.H,
                         self.slot_stride, self.rs_done, self.rs_epoch, int(self.peer_rs_pads.data_ptr()), self.tp.rank, self.W, self.ws,
                         self.tile_cnt, status)
        else:
            e.gemm_i8_rs(xq, w.q, xs, w.s, 0, plan.bn, plan.splits, int(self.peer_delta.data_ptr()), self.Tl, self.H,
                         self.slot_stride, self.rs_done, self.rs_epoch, int(self.peer_rs_pads.data_ptr()), self.tp.rank, self.W, self.ws,
                         self.tile_cnt, status)
        return {"rs": True}
