"""GateRank: recency plus a bonus for the router's rank (bigrig_engine/policies/gaterank.py:102-165).

Each use sets an expert's priority to ``tick + boost * w(rank)`` (kept at least
its previous priority when ``monotone``); the victim is the resident expert with
the lowest priority, ties to the lower id.  ``w`` is one of ``linear`` (k-1-r)/(k-1)
with k = ``param`` (default 8), ``inv`` 1/(1+r), or ``geom`` param**r.  Priorities
live in a lazily invalidated heap, rebuilt when stale entries pile up.
"""
from __future__ import annotations

import heapq

from ..pool import Policy


def _w_inv(r: int) -> float:
    return 1.0 / (1.0 + r)


def _w_geom(gamma: float):
    return lambda r: gamma ** r


def _w_linear(k: int):
    def f(r: int) -> float:
        if k <= 1:
            return 1.0
        return max(0.0, (k - 1 - r) / (k - 1))
    return f


SHAPES = {"inv": lambda p: _w_inv, "geom": lambda p: _w_geom(p), "linear": lambda p: _w_linear(int(p))}


class GateRank(Policy):
    name = "gaterank"

    def __init__(self, capacity, n_experts, boost: float = 16.0, shape: str = "linear",
                 param: float = 8, monotone: bool = True):
        super().__init__(capacity, n_experts)
        self.boost = float(boost)
        self.monotone = bool(monotone)
        self.w = SHAPES[shape](param)
        self.tick = 0
        self.key: dict = {}
        self.heap: list = []
        self._limit = 4 * max(1, capacity) + 16

    def _use(self, e: int, rank: int) -> None:
        self.tick += 1
        k = self.tick + self.boost * self.w(rank)
        if self.monotone:
            old = self.key.get(e)
            if old is not None and old > k:
                k = old
        self.key[e] = k
        heapq.heappush(self.heap, (k, e))
        if len(self.heap) > self._limit:
            self.heap = [(v, x) for x, v in self.key.items()]
            heapq.heapify(self.heap)

    def admit(self, e, rank=0):
        self._use(e, rank)

    def touch(self, e, rank=0):
        self._use(e, rank)

    def victim(self):
        while self.heap:
            k, e = self.heap[0]
            if self.key.get(e) != k:
                heapq.heappop(self.heap)
                continue
            return e
        return -1

    def evicted(self, e):
        self.key.pop(e, None)


def make(boost: float = 16.0, shape: str = "linear", param: float = 8, monotone: bool = True):
    """A ``factory(capacity, n_experts)`` with GateRank's parameters bound."""
    return lambda capacity, n_experts: GateRank(capacity, n_experts, boost=boost, shape=shape,
                                                param=param, monotone=monotone)


gaterank = make()
