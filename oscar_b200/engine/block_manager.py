"""Paged KV block manager (128-token kernel pages) and recurrent-state slot manager.

Every FULL-attention layer's INT2 pool and the MTP layer's BF16 shadow pool share one
physical block-id space, so a request's block table and slot mapping are computed
once per step: ``slot = block * 128 + offset`` (the reference's slot convention with
a 128-token kernel page, ``plan/ANALYSIS-20260904-C-...md:124-127``).
"""
from __future__ import annotations

PAGE = 128


class OutOfBlocks(RuntimeError):
    pass


class BlockManager:
    def __init__(self, num_blocks: int, page: int = PAGE):
        self.num_blocks = num_blocks
        self.page = page
        # LIFO free list: recently freed blocks are reused first (they are L2-warm)
        self._free = list(range(num_blocks - 1, -1, -1))
        self.tables: dict[int, list[int]] = {}

    @property
    def free_blocks(self) -> int:
        return len(self._free)

    def blocks_needed(self, rid: int, total_tokens: int) -> int:
        have = len(self.tables.get(rid, ()))
        return max(0, (total_tokens + self.page - 1) // self.page - have)

    def can_allocate(self, rid: int, total_tokens: int) -> bool:
        return self.blocks_needed(rid, total_tokens) <= len(self._free)

    def ensure(self, rid: int, total_tokens: int) -> list[int]:
        """Grow ``rid``'s table to cover ``total_tokens`` positions."""
        need = self.blocks_needed(rid, total_tokens)
        if need > len(self._free):
            raise OutOfBlocks(f"request {rid} needs {need} blocks, {len(self._free)} free")
        t = self.tables.setdefault(rid, [])
        for _ in range(need):
            t.append(self._free.pop())
        return t

    def slot(self, rid: int, pos: int) -> int:
        t = self.tables[rid]
        return t[pos // self.page] * self.page + pos % self.page

    def free(self, rid: int) -> None:
        for b in reversed(self.tables.pop(rid, [])):
            self._free.append(b)

    def table(self, rid: int) -> list[int]:
        return self.tables.get(rid, [])


class SlotManager:
    """Fixed pool of recurrent-state slots (GDN state, conv window, pending inputs)."""

    def __init__(self, n: int):
        self.n = n
        self._free = list(range(n - 1, -1, -1))
        self.owner: dict[int, int] = {}
        self.parity = [0] * n

    def acquire(self, rid: int) -> int:
        if rid in self.owner:
            return self.owner[rid]
        if not self._free:
            raise OutOfBlocks("no free recurrent-state slot")
        s = self._free.pop()
        self.owner[rid] = s
        self.parity[s] = 0
        return s

    def release(self, rid: int) -> None:
        s = self.owner.pop(rid, None)
        if s is not None:
            self._free.append(s)

    @property
    def free_slots(self) -> int:
        return len(self._free)
