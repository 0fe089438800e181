"""ARC, adaptive replacement cache (bigrig_engine/policies/arc.py:52-129).

Two resident lists, T1 (seen once) and T2 (seen again), each least recent
first, and their ghost lists B1/B2 of evicted ids.  A hit promotes T1 -> T2 or
refreshes T2.  A miss that finds its id in B1 grows the target size ``p`` of
T1 by max(1, |B2|/|B1|) (capped at c) and lands in T2; one in B2 shrinks ``p``
by max(1, |B1|/|B2|) (floored at 0) and lands in T2; a new id lands in T1.
The victim is the oldest of T1 when T1 exceeds ``p`` (or T2 is empty), else the
oldest of T2.  Ghosts keep |T1|+|B1| <= c and the four lists <= 2c, oldest ghost
dropped first (B2 before B1 for the second bound).
"""
from __future__ import annotations

from collections import OrderedDict

from ..pool import Policy


class ARC(Policy):
    name = "arc"

    def __init__(self, capacity: int, n_experts: int):
        super().__init__(capacity, n_experts)
        self.c = capacity
        self.p = 0.0
        self.t1: OrderedDict = OrderedDict()
        self.t2: OrderedDict = OrderedDict()
        self.b1: OrderedDict = OrderedDict()
        self.b2: OrderedDict = OrderedDict()

    def _bound_ghosts(self) -> None:
        while self.b1 and len(self.t1) + len(self.b1) > self.c:
            self.b1.popitem(last=False)
        while len(self.t1) + len(self.t2) + len(self.b1) + len(self.b2) > 2 * self.c:
            if self.b2:
                self.b2.popitem(last=False)
            elif self.b1:
                self.b1.popitem(last=False)
            else:
                break

    def admit(self, e, rank=0):
        if e in self.b1:
            self.p = min(float(self.c), self.p + max(1.0, len(self.b2) / max(1, len(self.b1))))
            del self.b1[e]
            self.t2[e] = None
        elif e in self.b2:
            self.p = max(0.0, self.p - max(1.0, len(self.b1) / max(1, len(self.b2))))
            del self.b2[e]
            self.t2[e] = None
        else:
            self.t1.pop(e, None)
            self.t2.pop(e, None)
            self.t1[e] = None
        self._bound_ghosts()

    def touch(self, e, rank=0):
        if e in self.t1:
            del self.t1[e]
            self.t2[e] = None
        elif e in self.t2:
            self.t2.move_to_end(e)
        else:
            self.t2[e] = None

    @staticmethod
    def _oldest(od) -> int:
        for e in od:
            return e
        return -1

    def victim(self):
        if self.t1 and (len(self.t1) > self.p or not self.t2):
            return self._oldest(self.t1)
        if self.t2:
            return self._oldest(self.t2)
        return self._oldest(self.t1)

    def evicted(self, e):
        if e in self.t1:
            del self.t1[e]
            self.b1[e] = None
        elif e in self.t2:
            del self.t2[e]
            self.b2[e] = None
        self._bound_ghosts()
