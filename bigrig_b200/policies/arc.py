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

State: per expert a list code and the clock value at which it entered that list;
a list's oldest entry is its member with the smallest entry clock.
"""
from __future__ import annotations

import numpy as np

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
        self.size = [0, 0, 0, 0, 0]          # entries per list code
        self.col = Columns(n_experts, where=(np.int8, OUT), entered=(np.int64, 0))

    def _put(self, e: int, lst: int) -> None:
        """Move e to the tail of ``lst`` (OUT removes it from every list)."""
        c = self.col
        self.size[int(c.where[e])] -= 1
        self.size[lst] += 1
        c.where[e] = lst
        self.clock += 1
        c.entered[e] = self.clock

    def _oldest(self, lst: int) -> int:
        return first_by(self.col.where == lst, self.col.entered)

    def _trim_ghosts(self) -> None:
        s = self.size
        while s[B1] and s[T1] + s[B1] > self.c:
            self._put(self._oldest(B1), OUT)
        while s[T1] + s[T2] + s[B1] + s[B2] > 2 * self.c:
            if s[B2]:
                self._put(self._oldest(B2), OUT)
            elif s[B1]:
                self._put(self._oldest(B1), OUT)
            else:
                break

    def admit(self, e, rank=0):
        e = int(e)
        self.col.fit(e)
        w = int(self.col.where[e])
        s = self.size
        if w == B1:
            self.p = min(float(self.c), self.p + max(1.0, s[B2] / max(1, s[B1])))
            self._put(e, T2)
        elif w == B2:
            self.p = max(0.0, self.p - max(1.0, s[B1] / max(1, s[B2])))
            self._put(e, T2)
        else:
            self._put(e, T1)
        self._trim_ghosts()

    def touch(self, e, rank=0):
        e = int(e)
        self.col.fit(e)
        self._put(e, T2)

    def victim(self):
        s = self.size
        if s[T1] and (s[T1] > self.p or not s[T2]):
            return self._oldest(T1)
        if s[T2]:
            return self._oldest(T2)
        return -1

    def evicted(self, e):
        e = int(e)
        self.col.fit(e)
        w = int(self.col.where[e])
        if w == T1:
            self._put(e, B1)
        elif w == T2:
            self._put(e, B2)
        self._trim_ghosts()


def factory(capacity, n_experts):
    return ARC(capacity, n_experts)
