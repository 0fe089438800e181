"""ARC, adaptive replacement: a recency list, a frequency list and their ghost lists.

Decision rule (bigrig_engine/policies/arc.py:52-129).  Lists, each ordered from its
least recent entry: T1 (held, used once), T2 (held, used again), B1 and B2 (ids
evicted from T1 and T2).  ``p`` is T1's target length, between 0 and the capacity c.

* admission of a B1 ghost raises ``p`` by max(1, |B2| / max(1, |B1|)) (at most c)
  and puts the expert at T2's tail; of a B2 ghost lowers ``p`` by
  max(1, |B1| / max(1, |B2|)) (at least 0) and puts it at T2's tail; any other
  expert goes to T1's tail;
* a use moves the expert to T2's tail (from T1, from within T2, or from nowhere);
* the victim is T1's oldest when T1 is longer than ``p`` or T2 is empty, else T2's
  oldest;
* an eviction moves the expert from T1 to B1's tail or from T2 to B2's tail;
* after admissions and evictions the ghosts are trimmed, oldest first: B1 while
  |T1| + |B1| > c, then B2 (or B1 when B2 is empty) while all four exceed 2c.

State: per expert a list code and the clock value at which it entered that list,
plus each list's member set; a list's oldest entry is its member with the smallest
entry clock.
"""
from __future__ import annotations

from ..pool import Policy
from ._columns import Columns, first_by

OUT, T1, T2, B1, B2 = 0, 1, 2, 3, 4


class ARC(Policy):
    name = "arc"

    def __init__(self, capacity: int, n_experts: int):
        super().__init__(capacity, n_experts)
        self.c = capacity
        self.p = 0.0
        self.clock = 0
        self.members = [set() for _ in range(5)]     # per list code (OUT unused)
        self.col = Columns(n_experts, where=OUT, entered=0)

    def _put(self, e: int, lst: int) -> None:
        """Move e to the tail of ``lst`` (OUT removes it from every list)."""
        c = self.col
        self.members[c.where[e]].discard(e)
        if lst != OUT:
            self.members[lst].add(e)
        c.where[e] = lst
        self.clock += 1
        c.entered[e] = self.clock

    def _oldest(self, lst: int) -> int:
        return first_by(self.members[lst], self.col.entered)

    def _trim_ghosts(self) -> None:
        t1, t2, b1, b2 = (self.members[i] for i in (T1, T2, B1, B2))
        while b1 and len(t1) + len(b1) > self.c:
            self._put(self._oldest(B1), OUT)
        while len(t1) + len(t2) + len(b1) + len(b2) > 2 * self.c:
            if b2:
                self._put(self._oldest(B2), OUT)
            elif b1:
                self._put(self._oldest(B1), OUT)
            else:
                break

    def admit(self, e, rank=0):
        e = int(e)
        self.col.fit(e)
        w = self.col.where[e]
        n_b1, n_b2 = len(self.members[B1]), len(self.members[B2])
        if w == B1:
            self.p = min(float(self.c), self.p + max(1.0, n_b2 / max(1, n_b1)))
            self._put(e, T2)
        elif w == B2:
            self.p = max(0.0, self.p - max(1.0, n_b1 / max(1, n_b2)))
            self._put(e, T2)
        else:
            self._put(e, T1)
        self._trim_ghosts()

    def touch(self, e, rank=0):
        e = int(e)
        self.col.fit(e)
        self._put(e, T2)

    def victim(self):
        t1, t2 = self.members[T1], self.members[T2]
        if t1 and (len(t1) > self.p or not t2):
            return self._oldest(T1)
        if t2:
            return self._oldest(T2)
        return -1

    def evicted(self, e):
        e = int(e)
        self.col.fit(e)
        w = self.col.where[e]
        if w == T1:
            self._put(e, B1)
        elif w == T2:
            self._put(e, B2)
        self._trim_ghosts()


def factory(capacity, n_experts):
    return ARC(capacity, n_experts)
