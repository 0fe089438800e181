"""GateRank: recency with a bonus for a high router rank.

Decision rule (bigrig_engine/policies/gaterank.py:102-165, defaults ``boost=16``,
``shape="linear"``, ``param=8``, ``monotone=True``): the n-th use of the cache
gives the used expert the priority ``n + boost * w(rank)``, or its previous
priority if that is higher and ``monotone`` is set; the victim is the tracked
expert of lowest priority, ties to the lowest expert id; an evicted expert is
forgotten.  Rank weights ``w``:

* ``linear``: (k - 1 - r) / (k - 1) with k = ``param`` (1 when k <= 1), at least 0;
* ``inv``: 1 / (1 + r);
* ``geom``: ``param`` ** r.

State: a priority column and the set of tracked experts; the victim is the
tracked expert of smallest priority.
"""
from __future__ import annotations

from ..pool import Policy
from ._columns import Columns, first_by


def rank_weight(shape: str, param: float):
    """The rank-weight function ``w(r)`` for ``shape`` and its parameter."""
    if shape == "inv":
        return lambda r: 1.0 / (1.0 + r)
    if shape == "geom":
        g = param
        return lambda r: g ** r
    if shape == "linear":
        k = int(param)
        if k <= 1:
            return lambda r: 1.0
        return lambda r: max(0.0, (k - 1 - r) / (k - 1))
    raise ValueError(f"rank-weight shape must be linear, inv or geom, got {shape!r}")


class GateRank(Policy):
    name = "gaterank"

    def __init__(self, capacity, n_experts, boost: float = 16.0, shape: str = "linear",
                 param: float = 8, monotone: bool = True):
        super().__init__(capacity, n_experts)
        self.boost = float(boost)
        self.monotone = bool(monotone)
        self.weight = rank_weight(shape, param)
        self.clock = 0
        self.col = Columns(n_experts, prio=0.0)
        self.tracked: set = set()

    def _use(self, e: int, rank: int) -> None:
        c = self.col
        c.fit(e)
        self.clock += 1
        p = self.clock + self.boost * self.weight(rank)
        if self.monotone and e in self.tracked and c.prio[e] > p:
            p = c.prio[e]
        c.prio[e] = p
        self.tracked.add(e)

    def admit(self, e, rank=0):
        self._use(int(e), rank)

    def touch(self, e, rank=0):
        self._use(int(e), rank)

    def victim(self):
        return first_by(self.tracked, self.col.prio)

    def evicted(self, e):
        self.tracked.discard(int(e))


def make(boost: float = 16.0, shape: str = "linear", param: float = 8, monotone: bool = True):
    """A ``factory(capacity, n_experts)`` building GateRank with these parameters."""
    return lambda capacity, n_experts: GateRank(capacity, n_experts, boost=boost, shape=shape,
                                                param=param, monotone=monotone)


def gaterank(capacity, n_experts):
    """The shipped configuration."""
    return GateRank(capacity, n_experts)
