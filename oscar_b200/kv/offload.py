"""Host KV offload: swap a request's cache out to pinned host memory and back.

The reference does not offload KV (``README.md:111``); BASELINE config 5 asks for host
offload of cold INT2 pages.  At the target shapes the INT2 cache of every running
request fits in HBM, so offload serves preemption: when the block pool runs dry the
scheduler swaps the most recently admitted request out - every FULL layer's INT2 pages,
the MTP layer's BF16 shadow pages, the request's staged sink/recent values and its GDN
recurrent state - frees its blocks and slot, and swaps it back in (new physical blocks,
new slot) when room returns.  Outputs are identical to an uninterrupted run.

Why whole requests and not cold pages: a FULL-attention decode step reads every
history page of every running request (the INT2 page *is* the cold storage - 136 B per
token and head), so a page kept on the host would cross PCIe on every step; the
capacity that offload buys is for requests that are not running.

Host memory comes from one pinned pool (:class:`PinnedPool`), sized when the engine
starts (``OSCAR_OFFLOAD_HOST_GIB``, default 4 GiB) and grown only in whole chunks when a
swap does not fit; a swap takes byte ranges from it and returns them when the request
comes back, so the serving path does not pin memory per swap.

The request's pages are gathered (``index_select``) on the compute stream, and the
copies to pinned host memory run on a side stream; the blocks return to the free list
once the copies' event has completed (:meth:`HostKVStore.poll` / ``drain``).  Swap-in
copies host -> device on the side stream, the compute stream waits on its event and
scatters the pages into the new blocks.  Staging owner tags change with the blocks, so
both directions report the tag updates for the engine's host mirror of the table.  On
the CPU reference path the same code runs without streams.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

import torch

PAGE = 128
_ALIGN = 256


class PinnedPool:
    """Byte ranges of a few large pinned host buffers (first fit, coalescing frees).

    Buffers are allocated at construction (``initial_bytes``) and then only when a
    request does not fit, ``chunk_bytes`` or more at a time; they are never returned to
    the system while the pool lives."""

    def __init__(self, initial_bytes: int = 0, chunk_bytes: int = 1 << 30, pin: bool = True):
        self.chunk_bytes = chunk_bytes
        self.pin = pin
        self.chunks: list[torch.Tensor] = []
        self.free: list[list[int]] = []  # [chunk, offset, size], sorted by (chunk, offset)
        self.allocations = 0             # buffers allocated from the system (not per request)
        if initial_bytes > 0:
            self._grow(initial_bytes)

    @property
    def capacity(self) -> int:
        return sum(c.numel() - _ALIGN for c in self.chunks)

    def _grow(self, need: int) -> None:
        size = max(self.chunk_bytes, (need + (1 << 20) - 1) // (1 << 20) * (1 << 20))
        buf = torch.empty(size + _ALIGN, dtype=torch.uint8, pin_memory=self.pin)
        pad = (-buf.data_ptr()) % _ALIGN  # ranges start on 256-byte boundaries
        self.chunks.append(buf)
        self.free.append([len(self.chunks) - 1, pad, size])
        self.allocations += 1

    def alloc(self, nbytes: int):
        """Returns ``(uint8 view, handle)``."""
        n = max(_ALIGN, (nbytes + _ALIGN - 1) // _ALIGN * _ALIGN)
        for attempt in range(2):
            for i, (c, off, size) in enumerate(self.free):
                if size >= n:
                    if size == n:
                        self.free.pop(i)
                    else:
                        self.free[i] = [c, off + n, size - n]
                    return self.chunks[c][off:off + nbytes], (c, off, n)
            if attempt == 0:
                self._grow(n)
        raise MemoryError(f"pinned pool cannot hold {nbytes} bytes")

    def release(self, handle) -> None:
        c, off, n = handle
        self.free.append([c, off, n])
        self.free.sort()
        merged: list[list[int]] = []
        for e in self.free:
            if merged and merged[-1][0] == e[0] and merged[-1][1] + merged[-1][2] == e[1]:
                merged[-1][2] += e[2]
            else:
                merged.append(list(e))
        self.free = merged

    def used(self) -> int:
        return self.capacity - sum(e[2] for e in self.free)


@dataclass
class Swapped:
    """Host copy of one request's device state."""

    rid: int
    n_blocks: int
    pages: list            # per FULL layer: [n_blocks, Hk, page_bytes] uint8 (host)
    shadow: tuple | None   # MTP layer (kc, vc): [n_blocks, 128, Hk, D] bf16 (host)
    staged_mask: torch.Tensor | None   # [n_blocks, 128] bool: seat held this block's token
    staged: list           # per FULL layer: (k, v) [n_staged, Hk, D] fp32 (host)
    gdn: list              # per GDN layer: tuple of host tensors
    parity: int = 0
    event: object = None   # completion of the device->host copies
    nbytes: int = 0
    owner_cleared: object = None  # staging seats whose tags were reset (numpy)
    handles: list = field(default_factory=list)  # pinned-pool ranges of the host tensors


@dataclass
class OffloadStats:
    swapped_out: int = 0
    swapped_in: int = 0
    bytes_out: int = 0
    bytes_in: int = 0
    host_bytes_peak: int = 0
    _host_now: int = 0


class HostKVStore:
    def __init__(self, model, pin: bool | None = None, host_bytes: int | None = None):
        self.model = model
        dev = model.device
        self.cuda = dev.type == "cuda"
        self.pin = self.cuda if pin is None else pin
        self.stream = torch.cuda.Stream(device=dev) if self.cuda else None
        self.swapped: dict[int, Swapped] = {}
        self.stats = OffloadStats()
        self._pending_free: list = []  # (event, callback)
        if host_bytes is None:
            host_bytes = int(float(os.environ.get("OSCAR_OFFLOAD_HOST_GIB", "4")) * (1 << 30)) if self.cuda else 0
        self.pool = PinnedPool(host_bytes, pin=self.pin)
        self._handles: list = []  # ranges taken by the current _to_host call

    # ------------------------------------------------------------ helpers
    def _to_host(self, dev_tensors: list) -> list:
        """Device temporaries -> pinned host copies on the side stream."""
        if not self.cuda:
            return [t.clone() for t in dev_tensors]
        main = torch.cuda.current_stream(self.model.device)
        self.stream.wait_stream(main)
        out = []
        self._handles = []
        with torch.cuda.stream(self.stream):
            for t in dev_tensors:
                raw, hd = self.pool.alloc(t.numel() * t.element_size())
                self._handles.append(hd)
                h = raw.view(t.dtype).view(t.shape)
                h.copy_(t, non_blocking=True)
                t.record_stream(self.stream)
                out.append(h)
        return out

    def _to_device(self, host_tensors: list) -> list:
        if not self.cuda:
            return list(host_tensors)
        dev = self.model.device
        out = []
        with torch.cuda.stream(self.stream):
            for h in host_tensors:
                out.append(h.to(dev, non_blocking=True))
            ev = torch.cuda.Event()
            ev.record(self.stream)
        main = torch.cuda.current_stream(dev)
        main.wait_event(ev)
        for t in out:
            t.record_stream(main)
        ev.synchronize()  # the pinned sources may be released after this
        return out

    def poll(self) -> None:
        """Run the deferred frees whose device->host copies have completed."""
        keep = []
        for ev, cb in self._pending_free:
            if ev is None or ev.query():
                cb()
            else:
                keep.append((ev, cb))
        self._pending_free = keep

    def drain(self) -> None:
        for ev, cb in self._pending_free:
            if ev is not None:
                ev.synchronize()
            cb()
        self._pending_free = []

    # ------------------------------------------------------------ layout
    def _stage_rows_of(self, idx: torch.Tensor, slot: int) -> torch.Tensor:
        """Staging row of each of a request's blocks (in logical page order)."""
        m = self.model
        lay = getattr(m, "stage_layout", None)
        if lay is None:
            return idx % m.stage_rows
        from .oracle import window_row
        return window_row(slot, torch.arange(idx.numel(), device=idx.device), lay[0], lay[1])

    def _gdn_views(self, g):
        return ((g.state, 0), (g.conv_state, 1), (g.pend_x, 1), (g.pend_ba, 0))

    # ------------------------------------------------------------ swap out
    def swap_out(self, rid: int, blocks: list[int], slot: int, parity: int, on_freed) -> Swapped:
        """Gather on the compute stream, copy to host on the side stream; ``on_freed`` runs
        (from :meth:`poll`) once the copies are done and the blocks may be reused."""
        m = self.model
        dev = m.device
        idx = torch.tensor(blocks, dtype=torch.long, device=dev)
        dev_t, kinds = [], []
        for layer in m.full_layers:
            if layer.pool is not None:
                dev_t.append(layer.pool.index_select(0, idx))
                kinds.append(("pool", 1))
            else:
                dev_t += [layer.kc.index_select(0, idx), layer.vc.index_select(0, idx)]
                kinds.append(("bf16", 2))
        n_shadow = 0
        if getattr(m, "mtp", None) is not None and m.mtp.layer.kc is not None:
            L = m.mtp.layer
            dev_t += [L.kc.index_select(0, idx), L.vc.index_select(0, idx)]
            n_shadow = 2
        maskd = None
        n_staged = 0
        owner_cleared = None
        if m.stage_rows:
            seats = (self._stage_rows_of(idx, slot) * PAGE).unsqueeze(1) + torch.arange(PAGE, device=dev)  # [nb, 128]
            own = m.owner[seats.view(-1)].view(len(blocks), PAGE)
            maskd = own == idx.unsqueeze(1).to(own.dtype)
            sel = seats[maskd]
            for layer in m.full_layers:
                if layer.stage_k is not None:
                    # V staging is dim-major per row: gather [n, Hk, D] at (row, :, :, off)
                    dev_t += [layer.stage_k.index_select(0, sel),
                              layer.stage_v[sel // PAGE, :, :, sel % PAGE].contiguous()]
                    n_staged += 1
            m.owner[sel] = -1  # these seats stop belonging to blocks that are about to be reused
            dev_t.append(maskd)
            owner_cleared = sel
        s = torch.tensor([slot], dtype=torch.long, device=dev)
        for g in m.gdn_layers:
            dev_t += [t.index_select(dim, s) for t, dim in self._gdn_views(g)]
        host = self._to_host(dev_t)
        ev = None
        if self.cuda:
            ev = torch.cuda.Event()
            ev.record(self.stream)
        # unpack
        it = iter(host)
        pages = [next(it) if k == "pool" else (next(it), next(it)) for k, _ in kinds]
        shadow = (next(it), next(it)) if n_shadow else None
        staged = [(next(it), next(it)) for _ in range(n_staged)]
        mask = next(it) if maskd is not None else None
        gdn = [tuple(next(it) for _ in range(4)) for _ in m.gdn_layers]
        nbytes = sum(t.numel() * t.element_size() for t in host)
        sw = Swapped(rid, len(blocks), pages, shadow, mask, staged, gdn, parity, ev, nbytes)
        sw.handles, self._handles = self._handles, []
        sw.owner_cleared = owner_cleared.cpu().numpy() if owner_cleared is not None else None
        self.swapped[rid] = sw
        self._pending_free.append((ev, on_freed))
        st = self.stats
        st.swapped_out += 1
        st.bytes_out += nbytes
        st._host_now += nbytes
        st.host_bytes_peak = max(st.host_bytes_peak, st._host_now)
        return sw

    # ------------------------------------------------------------ swap in
    def discard(self, rid: int) -> None:
        """Drop the host copy of a swapped-out request that will not come back (aborted)."""
        sw = self.swapped.pop(rid, None)
        if sw is not None:
            if sw.event is not None:
                sw.event.synchronize()  # no copy into the host buffers is still in flight
            for hd in sw.handles:
                self.pool.release(hd)
            self.stats._host_now -= sw.nbytes

    def swap_in(self, rid: int, blocks: list[int], slot: int):
        """Restore ``rid`` into new ``blocks`` / ``slot``.  Returns ``(parity, seats, tags)``:
        the saved slot parity and the staging owner-tag updates (numpy, or None)."""
        m = self.model
        sw = self.swapped.pop(rid)
        if sw.event is not None:
            sw.event.synchronize()  # the host copy is complete before it is read back
        dev = m.device
        assert len(blocks) == sw.n_blocks
        idx = torch.tensor(blocks, dtype=torch.long, device=dev)
        flat = list(_tensors(sw.pages, sw.shadow, sw.staged, []))
        if sw.staged_mask is not None:
            flat.append(sw.staged_mask)
        for g in sw.gdn:
            flat += list(g)
        d = iter(self._to_device(flat))
        for layer, hp in zip(m.full_layers, sw.pages):
            if layer.pool is not None:
                layer.pool.index_copy_(0, idx, next(d))
            else:
                layer.kc.index_copy_(0, idx, next(d))
                layer.vc.index_copy_(0, idx, next(d))
        if sw.shadow is not None:
            L = m.mtp.layer
            L.kc.index_copy_(0, idx, next(d))
            L.vc.index_copy_(0, idx, next(d))
        staged = [(next(d), next(d)) for _ in sw.staged]
        owner_upd = (None, None)
        if sw.staged_mask is not None:
            maskd = next(d)
            seats = (self._stage_rows_of(idx, slot) * PAGE).unsqueeze(1) + torch.arange(PAGE, device=dev)
            lay = getattr(m, "stage_layout", None)
            if lay is None:
                # no stale tag may claim the new blocks; restored tokens get their tags back
                tags = torch.where(maskd, idx.unsqueeze(1), torch.full_like(seats, -1)).view(-1).to(m.owner.dtype)
                m.owner[seats.view(-1)] = tags
                owner_upd = (seats.view(-1).cpu().numpy(), tags.cpu().numpy())
            else:
                # the slot's rows are the request's own: clear them all, then restore the
                # staged tokens' tags (pages sharing a ring row must not race on a seat)
                per = lay[0] + lay[1]
                own_seats = ((slot * per + torch.arange(per, device=dev)) * PAGE).unsqueeze(1) + torch.arange(
                    PAGE, device=dev)
                own_seats = own_seats.view(-1)
                claimed = seats[maskd]
                ctags = idx.unsqueeze(1).expand_as(seats)[maskd].to(m.owner.dtype)
                reset = own_seats[~torch.isin(own_seats, claimed)]
                m.owner[reset] = -1
                m.owner[claimed] = ctags
                owner_upd = (torch.cat([reset, claimed]).cpu().numpy(),
                             torch.cat([torch.full_like(reset, -1).to(m.owner.dtype), ctags]).cpu().numpy())
            sel = seats[maskd]
            it = iter(staged)
            for layer in m.full_layers:
                if layer.stage_k is not None:
                    k, v = next(it)
                    layer.stage_k.index_copy_(0, sel, k)
                    layer.stage_v[sel // PAGE, :, :, sel % PAGE] = v
        s = torch.tensor([slot], dtype=torch.long, device=dev)
        for g in m.gdn_layers:
            for t, dim in self._gdn_views(g):
                t.index_copy_(dim, s, next(d))
        for hd in sw.handles:  # _to_device waited for the copies out of these ranges
            self.pool.release(hd)
        st = self.stats
        st.swapped_in += 1
        st.bytes_in += sw.nbytes
        st._host_now -= sw.nbytes
        return sw.parity, owner_upd[0], owner_upd[1]


def _tensors(pages, shadow, staged, gdn):
    for p in pages:
        if isinstance(p, tuple):
            yield from p
        else:
            yield p
    if shadow is not None:
        yield from shadow
    for kv in staged:
        yield from kv
    for g in gdn:
        yield from g
