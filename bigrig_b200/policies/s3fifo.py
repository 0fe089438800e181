"""S3-FIFO (bigrig_engine/policies/s3fifo.py:42-144).

A small FIFO S (target 10% of capacity) quarantines new experts, a main FIFO M
holds proven ones, and a ghost FIFO (capacity entries) remembers ids evicted
from S.  A hit bumps a frequency capped at 3.  Admission puts a ghost id
straight into M, anything else into S.  Eviction: while S holds at least its
target, pop S's head -- promoted to M's tail (frequency reset) if it was hit more
than once, else evicted and remembered as a ghost; otherwise pop M's head --
re-queued with frequency - 1 if it was hit, else evicted.
"""
from __future__ import annotations

from collections import OrderedDict, deque

from ..pool import Policy


class S3FIFO(Policy):
    name = "s3fifo"

    S_RATIO = 0.10
    FREQ_MAX = 3
    PROMOTE_THRESHOLD = 1
    GHOST_RATIO = 1.0

    def __init__(self, capacity, n_experts):
        super().__init__(capacity, n_experts)
        self.s_target = max(1, int(round(self.S_RATIO * capacity)))
        self.ghost_max = max(1, int(round(self.GHOST_RATIO * capacity)))
        self.small: deque = deque()
        self.main: deque = deque()
        self.in_small: set = set()
        self.in_main: set = set()
        self.freq: dict = {}
        self.ghost: OrderedDict = OrderedDict()

    def admit(self, e, rank=0):
        if e in self.in_small or e in self.in_main:
            return
        self.freq[e] = 0
        if e in self.ghost:
            del self.ghost[e]
            self.main.append(e)
            self.in_main.add(e)
        else:
            self.small.append(e)
            self.in_small.add(e)

    def touch(self, e, rank=0):
        f = self.freq.get(e, 0)
        if f < self.FREQ_MAX:
            self.freq[e] = f + 1

    def _from_small(self):
        e = self.small.popleft()
        self.in_small.discard(e)
        if self.freq.get(e, 0) > self.PROMOTE_THRESHOLD:
            self.freq[e] = 0
            self.main.append(e)
            self.in_main.add(e)
            return None
        self.freq.pop(e, None)
        self.ghost[e] = None
        self.ghost.move_to_end(e)
        while len(self.ghost) > self.ghost_max:
            self.ghost.popitem(last=False)
        return e

    def _from_main(self):
        e = self.main.popleft()
        f = self.freq.get(e, 0)
        if f > 0:
            self.freq[e] = f - 1
            self.main.append(e)
            return None
        self.in_main.discard(e)
        self.freq.pop(e, None)
        return e

    def victim(self):
        while self.small or self.main:
            if self.small and len(self.small) >= self.s_target:
                v = self._from_small()
            elif self.main:
                v = self._from_main()
            else:
                v = self._from_small()
            if v is not None:
                return v
        return -1

    def evicted(self, e):
        self.in_small.discard(e)
        self.in_main.discard(e)
        self.freq.pop(e, None)
        for q in (self.small, self.main):
            try:
                q.remove(e)
            except ValueError:
                pass


def factory(capacity, n_experts):
    return S3FIFO(capacity, n_experts)
