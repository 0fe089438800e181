"""LFUDA: LFU with dynamic aging, the shipped default (bigrig_engine/policies/lfuda.py:67-173).

Every use re-anchors an expert's key to the cache age: ``key = L + count``,
with ``count`` saturating at ``fcap`` (12).  The victim is the resident expert
with the smallest key, ties to the least recently used.  An eviction raises
``L`` to the victim's key (never lowers it) and, with ``keep_ghost``, keeps the
victim's count multiplied by ``ghost_decay`` (0.5) so a returning expert is not
a stranger.  ``rank_weight`` > 0 credits a use at router rank r with
1 + rank_weight / (1 + r) instead of 1.  ``victim(exclude=...)`` skips experts
the caller is still using, so the pool never has to report a false eviction.
"""
from __future__ import annotations

from ..pool import Policy


class LFUDA(Policy):
    name = "lfuda"

    def __init__(self, capacity, n_experts, rank_weight: float = 0.0, keep_ghost: bool = True,
                 fcap: float | None = 12.0, ghost_decay: float = 0.5):
        super().__init__(capacity, n_experts)
        self.rank_weight = float(rank_weight)
        self.keep_ghost = bool(keep_ghost)
        self.fcap = fcap
        self.ghost_decay = float(ghost_decay)
        self.L = 0.0          # cache age: the largest key evicted so far
        self.cnt: dict = {}   # expert -> frequency credit (kept across evictions as a ghost)
        self.key: dict = {}   # resident expert -> L at last use + credit
        self.last: dict = {}  # expert -> tick of last use (tie-break)
        self.resident: set = set()
        self.tick = 0

    def _use(self, e: int, rank: int) -> None:
        self.tick += 1
        self.last[e] = self.tick
        credit = 1.0 if self.rank_weight == 0.0 else 1.0 + self.rank_weight / (1.0 + rank)
        c = self.cnt.get(e, 0.0) + credit
        if self.fcap is not None and c > self.fcap:
            c = self.fcap
        self.cnt[e] = c
        self.key[e] = self.L + c

    def admit(self, e, rank=0):
        self.resident.add(e)
        if not self.keep_ghost:
            self.cnt.pop(e, None)
        self._use(e, rank)

    def touch(self, e, rank=0):
        self._use(e, rank)

    def victim(self, exclude=()):
        cands = self.resident if not exclude else self.resident.difference(exclude)
        if not cands:
            return -1
        return min(cands, key=lambda x: (self.key.get(x, 0.0), self.last.get(x, 0)))

    def evicted(self, e):
        k = self.key.pop(e, self.L)
        if k > self.L:
            self.L = k
        self.resident.discard(e)
        if not self.keep_ghost:
            self.cnt.pop(e, None)
            self.last.pop(e, None)
        elif self.ghost_decay != 1.0:
            self.cnt[e] = self.cnt.get(e, 0.0) * self.ghost_decay


class TextbookLFUDA(LFUDA):
    """Uncapped count dropped on eviction: aging alone (kept for comparison)."""
    name = "lfuda_textbook"

    def __init__(self, capacity, n_experts):
        super().__init__(capacity, n_experts, keep_ghost=False, fcap=None, ghost_decay=1.0)


def factory(**kw):
    """``factory(**params)`` -> ``f(capacity, n_experts)`` with LFUDA's parameters bound."""
    return lambda capacity, n_experts: LFUDA(capacity, n_experts, **kw)
