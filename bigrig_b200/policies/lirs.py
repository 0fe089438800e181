"""LIRS: evict by inter-reference recency (bigrig_engine/policies/lirs.py:53-227).

A recency stack S (oldest at the bottom) holds LIR experts, resident HIR
experts and a bounded history of non-resident HIR ids; a queue Q holds the
resident HIR experts, the eviction candidates.  ``capacity - L_hirs`` experts
are LIR, with ``L_hirs = max(min_hir, round(hir_ratio * capacity))`` clamped to
[1, capacity - 1].  Referencing an expert found in S makes it LIR (it was
re-used within the LIR set's recency); LIR overflow demotes the bottom LIR
expert to HIR (to the back of Q if resident).  S is pruned so its bottom is
always LIR; the non-resident history is held to ``round(hist_ratio *
capacity)`` entries, oldest first.  The victim is Q's front, else the lowest
resident entry of S, else any resident expert.

The decisions, and the order of operations on S, Q and the resident set, are
kept identical to the reference so that miss counts replay exactly.
"""
from __future__ import annotations

from collections import OrderedDict

from ..pool import Policy

LIR = 0
HIR = 1


class LIRS(Policy):
    name = "lirs"

    def __init__(self, capacity: int, n_experts: int, hir_ratio: float = 0.05,
                 min_hir: int = 1, hist_ratio: float | None = 0.25):
        super().__init__(capacity, n_experts)
        h = max(min_hir, int(round(hir_ratio * capacity)))
        self.L_hirs = max(1, min(h, capacity - 1))
        self.L_lirs = capacity - self.L_hirs
        self.hist_limit = None if hist_ratio is None else max(1, int(round(hist_ratio * capacity)))
        self.S: OrderedDict = OrderedDict()   # bottom (oldest) first
        self.Q: OrderedDict = OrderedDict()   # front first
        self.status: dict = {}
        self.resident: set = set()
        self.n_lir = 0
        self.n_nonres = 0

    @staticmethod
    def _bottom(od):
        for e in od:
            return e
        return None

    def _prune(self) -> None:
        while self.S:
            b = self._bottom(self.S)
            if self.status.get(b) == LIR:
                return
            del self.S[b]
            if b not in self.resident:
                self.status.pop(b, None)
                self.n_nonres -= 1

    def _trim_history(self) -> None:
        if self.hist_limit is None:
            return
        while self.n_nonres > self.hist_limit:
            oldest = next((b for b in self.S if b not in self.resident), None)
            if oldest is None:
                self.n_nonres = 0
                return
            del self.S[oldest]
            self.status.pop(oldest, None)
            self.n_nonres -= 1

    def _demote_bottom(self) -> None:
        self._prune()
        if not self.S:
            return
        b = self._bottom(self.S)
        del self.S[b]
        self.status[b] = HIR
        self.n_lir -= 1
        if b in self.resident:
            self.Q.pop(b, None)
            self.Q[b] = None
        self._prune()

    def _make_lir(self, e: int) -> None:
        self.status[e] = LIR
        self.n_lir += 1
        self.S.pop(e, None)
        self.S[e] = None
        self.Q.pop(e, None)
        while self.n_lir > self.L_lirs:
            before = self.n_lir
            self._demote_bottom()
            if self.n_lir == before:
                break
        self._prune()

    def admit(self, e, rank=0):
        in_s = e in self.S
        if in_s and e not in self.resident:
            self.n_nonres -= 1
        self.resident.add(e)
        if in_s:
            self._make_lir(e)
            return
        if self.n_lir < self.L_lirs:
            self.status[e] = LIR
            self.n_lir += 1
            self.S[e] = None
        else:
            self.status[e] = HIR
            self.S[e] = None
            self.Q.pop(e, None)
            self.Q[e] = None

    def touch(self, e, rank=0):
        if self.status.get(e) == LIR:
            was_bottom = self._bottom(self.S) == e
            self.S.pop(e, None)
            self.S[e] = None
            if was_bottom:
                self._prune()
            return
        if e in self.S:
            self._make_lir(e)
        else:
            self.S[e] = None
            self.Q.pop(e, None)
            self.Q[e] = None

    def victim(self):
        if self.Q:
            return self._bottom(self.Q)
        self._prune()
        for b in self.S:
            if b in self.resident:
                return b
        for e in self.resident:
            return e
        return -1

    def evicted(self, e):
        self.resident.discard(e)
        self.Q.pop(e, None)
        if self.status.get(e) == LIR:
            self.status[e] = HIR
            self.n_lir -= 1
            self.S.pop(e, None)
            self.status.pop(e, None)
        elif e in self.S:
            self.n_nonres += 1
        self._prune()
        self._trim_history()


def make(capacity: int, n_experts: int) -> LIRS:
    return LIRS(capacity, n_experts)
