"""Row-parallel projection + all-reduce, fused into one GEMM over NVSwitch.

Every row-parallel projection of the decoder (attention ``o_proj``, GDN ``out_proj``,
MLP ``down_proj``) produces a partial sum that the tensor-parallel ranks must add
before the next RMSNorm.  The reference issues a GEMM followed by a separate
all-reduce collective per projection (vLLM's row-parallel linear under
``oscar/vllm_plugin`` serving).  Here the two are one kernel:

* the residual-delta buffers live in symmetric memory (``torch`` ``_symmetric_memory``
  is only the allocator/rendezvous: it gives each rank's unicast pointer, the NVLS
  multicast address of the whole allocation and per-rank signal pads);
* the int8 tcgen05 GEMM epilogue writes its fp32 tile with
  ``multimem.red.add`` to the multicast address, so the switch adds it into the same
  element of every rank's buffer while the next tiles are still on the tensor cores;
* the last CTA of the GEMM bumps a device-resident epoch and stores it with release
  semantics into every peer's signal pad slot ``[rank]``;
* the consuming RMSNorm kernel waits (bounded, acquire) until all ``world`` slots of its
  own pad reach its epoch, adds the buffer into the fp32 residual and zeroes the
  buffer for the reduction after next.

Two buffers alternate: a rank can only start reduction ``i+2`` after it consumed
reduction ``i+1``, which needs every peer's GEMM ``i+1`` done, which in each peer's
stream order follows that peer's read-and-zero of reduction ``i``.  Every forward
starts on buffer 0 and issues an even number of fused reductions, so captured CUDA
graphs keep the alternation on replay.

This path needs NVLS multicast (``has_multicast_support``); :class:`NcclRowReduce`
(GEMM into a local delta + ``dist.all_reduce``) is the fallback and the default (see
:func:`make_row_reduce`).
"""
from __future__ import annotations

import os

import torch
import torch.distributed as dist

from ..ops import functional as F
from ..ops._ext import ext
from .groups import TPGroup


class FullRows:
    """Every rank keeps all ``T`` rows of the residual stream (the all-reduce designs):
    the embedding is all-reduced, a replicated projection fills every row, and each
    norm runs over all rows, consuming the pending reduction's keyword arguments."""

    seq_parallel = False

    def embed_in(self, tokens: torch.Tensor, table: torch.Tensor, vocab_begin: int) -> torch.Tensor:
        T = tokens.shape[0]
        residual = torch.empty(T, table.shape[1], dtype=torch.float32, device=table.device)
        F.embed(tokens, table, vocab_begin, residual)
        self.tp.all_reduce_(residual)
        return residual

    def fc_rows(self, xq, xs, w, status=None) -> torch.Tensor:
        residual = torch.zeros(xq.shape[0], w.q.shape[0], dtype=torch.float32, device=xq.device)
        F.linear_i8(xq, xs, w.q, w.s, out=residual, accumulate=True, status=status)
        return residual

    def norm(self, residual, w, eps: float, pending: dict | None = None, want_bf16: bool = False, status=None):
        return F.rmsnorm_quant(residual, w, eps, want_bf16=want_bf16, status=status, **(pending or {}))


class NcclRowReduce(FullRows):
    """Baseline: local fp32 delta, GEMM accumulate, NCCL all-reduce.  The delta buffer is
    zero between reductions: the consuming RMSNorm adds it into the residual and clears
    it, so no separate fill precedes each GEMM."""

    fused = False

    def __init__(self, tp: TPGroup, max_rows: int = 0, H: int = 0, device=None):
        self.tp = tp
        self.delta = None
        if max_rows > 0 and H > 0 and device is not None:
            self.delta = torch.zeros(max_rows, H, dtype=torch.float32, device=device)

    def begin(self, T: int, H: int, device) -> None:
        if self.delta is None or self.delta.shape[0] < T or self.delta.shape[1] != H or self.delta.device != device:
            self.delta = torch.zeros(max(T, 1), H, dtype=torch.float32, device=device)
        self._T = T

    def gemm(self, xq, xs, w, k: int, status=None) -> dict:
        """``delta = all_reduce(xq @ w^T)``; returns the kwargs of the consuming RMSNorm."""
        d = self.delta[:self._T]
        F.linear_i8(xq, xs, w.q, w.s, out=d, accumulate=True, status=status)
        self.tp.all_reduce_(d)
        return {"delta": d, "zero_delta": True}


class FusedRowReduce(FullRows):
    """GEMM epilogue reduces through NVLS multicast; the RMSNorm waits on peer flags."""

    fused = True

    def __init__(self, tp: TPGroup, max_rows: int, H: int, device):
        import torch.distributed._symmetric_memory as symm

        self.tp = tp
        self.H = H
        self.max_rows = max_rows
        group = tp.group if tp.group is not None else dist.group.WORLD
        idx = device.index if device.index is not None else torch.cuda.current_device()
        if not symm._SymmetricMemory.has_multicast_support(symm.DeviceType.CUDA, idx):
            raise RuntimeError("NVLS multicast is not supported on this device")
        self.bufs = symm.empty((2, max_rows, H), dtype=torch.float32, device=device)
        self.hdl = symm.rendezvous(self.bufs, group)
        if not int(self.hdl.multicast_ptr):
            raise RuntimeError("NVLS multicast is not available for this group")
        self.bufs.zero_()
        self.mc = int(self.hdl.multicast_ptr)
        self.peer_signals = int(self.hdl.signal_pad_ptrs_dev)
        self.my_signals = int(self.hdl.signal_pad_ptrs[self.hdl.rank])
        # zero our own signal slots (others' stores only ever raise them)
        pad = self.hdl.get_signal_pad(self.hdl.rank, (tp.world,), dtype=torch.int32)
        pad.zero_()
        self.epoch = torch.zeros(1, dtype=torch.int32, device=device)
        self.done = torch.zeros(1, dtype=torch.int32, device=device)
        # split-K partials are summed locally first (one NVLink crossing per element)
        self.ws = torch.zeros(max_rows, H, dtype=torch.float32, device=device)
        self.tile_cnt = torch.zeros(1 << 16, dtype=torch.int32, device=device)
        torch.cuda.synchronize(device)
        dist.barrier(group=group)
        self._T = 0

    def begin(self, T: int, H: int, device) -> None:
        if T > self.max_rows or H != self.H:
            raise ValueError(f"fused all-reduce buffer holds {self.max_rows}x{self.H}, step needs {T}x{H}")
        self._T = T

    def gemm(self, xq, xs, w, k: int, status=None) -> dict:
        M, K = xq.shape
        N = w.q.shape[0]
        plan = F.plan_gemm(M, N, K, F.num_sms(xq.device), allow_split=True)
        b = k & 1
        mc = self.mc + b * self.max_rows * self.H * 4
        if plan.swap:
            ext().gemm_i8_allreduce(w.q, xq, w.s, xs, mc, self.H, 1, plan.bn, plan.splits, self.done, self.epoch,
                                    self.peer_signals, self.tp.rank, self.tp.world, self.ws, self.tile_cnt, status)
        else:
            ext().gemm_i8_allreduce(xq, w.q, xs, w.s, mc, self.H, 0, plan.bn, plan.splits, self.done, self.epoch,
                                    self.peer_signals, self.tp.rank, self.tp.world, self.ws, self.tile_cnt, status)
        return {"delta": self.bufs[b, :self._T], "wait": (self.my_signals, self.epoch, self.tp.world),
                "zero_delta": True}


def tp_comm_mode() -> str:
    """``OSCAR_TP_COMM``: ``sp`` (default: sequence-parallel residual with the
    reduce-scatter in the row-parallel GEMM epilogue and the all-gather pushed by the
    RMSNorm, :mod:`oscar_b200.parallel.seqpar`), ``nvls`` (GEMM epilogue all-reduce
    through NVLS multicast, :class:`FusedRowReduce`; also ``OSCAR_FUSED_AR=1``) or
    ``nccl`` (GEMM + NCCL all-reduce, the baseline)."""
    mode = os.environ.get("OSCAR_TP_COMM", "").strip().lower()
    if not mode:
        mode = "nvls" if os.environ.get("OSCAR_FUSED_AR", "0") in ("1", "auto") else "sp"
    if mode not in ("sp", "nvls", "nccl"):
        raise ValueError(f"OSCAR_TP_COMM={mode!r}: expected sp, nvls or nccl")
    return mode


def make_row_reduce(tp: TPGroup, max_rows: int, H: int, device):
    """Row-parallel reduction of a TP group (:func:`tp_comm_mode`).  CPU groups (gloo)
    and single ranks use :class:`NcclRowReduce`; a fused mode that cannot be set up
    (no symmetric memory / NVLS on the system) falls back to it with a message, unless
    it was asked for explicitly."""
    dev = torch.device(device)
    if tp.world == 1 or dev.type != "cuda":
        return NcclRowReduce(tp, max_rows, H, dev)
    mode = tp_comm_mode()
    explicit = bool(os.environ.get("OSCAR_TP_COMM")) or os.environ.get("OSCAR_FUSED_AR") == "1"
    try:
        if mode == "sp":
            from .seqpar import SeqParallelTP
            return SeqParallelTP(tp, max_rows, H, dev)
        if mode == "nvls":
            return FusedRowReduce(tp, max_rows, H, dev)
    except (RuntimeError, ImportError, ValueError) as exc:
        if explicit:
            raise
        print(f"[oscar_b200] {mode} tensor-parallel path unavailable ({exc}); using NCCL all-reduce")
    return NcclRowReduce(tp, max_rows, H, dev)
