"""LFUDA, frequency with dynamic aging: the engine's default expert-cache policy.

Decision rule (bigrig_engine/policies/lfuda.py:67-173, defaults ``rank_weight=0``,
``keep_ghost=True``, ``fcap=12``, ``ghost_decay=0.5``):

* a use of expert e adds a credit (1, or 1 + rank_weight / (1 + rank) when rank
  weighting is on) to e's frequency, saturating at ``fcap``, and sets e's priority
  to ``age + frequency``;
* the victim is the held expert of lowest priority, ties to the one used longest
  ago; ``victim(exclude=...)`` never names an excluded expert;
* an eviction raises ``age`` to the victim's priority if that is higher, and
  keeps the victim's frequency scaled by ``ghost_decay`` (``keep_ghost``) or
  forgets it.

State: per-expert columns (frequency, priority, use clock), the set of held
experts and the scalar age.  Priorities and frequencies are float64 and updated with the
same operations in the same order as the rule above states, so the victims, and
the miss counts on a replayed trace, are the reference's.
"""
from __future__ import annotations

from ..pool import Policy
from ._columns import Columns, first_by


class LFUDA(Policy):
    name = "lfuda"

    def __init__(self, capacity, n_experts, rank_weight: float = 0.0, keep_ghost: bool = True,
                 fcap: float | None = 12.0, ghost_decay: float = 0.5):
        super().__init__(capacity, n_experts)
        self.rank_weight = float(rank_weight)
        self.keep_ghost = bool(keep_ghost)
        self.fcap = None if fcap is None else float(fcap)
        self.ghost_decay = float(ghost_decay)
        self.age = 0.0
        self.clock = 0
        self.col = Columns(n_experts, freq=0.0, prio=0.0, used_at=0, has_prio=False)
        self.held: set = set()

    def _credit(self, rank: int) -> float:
        if self.rank_weight == 0.0:
            return 1.0
        return 1.0 + self.rank_weight / (1.0 + rank)

    def _use(self, e: int, rank: int) -> None:
        c = self.col
        c.fit(e)
        self.clock += 1
        c.used_at[e] = self.clock
        f = c.freq[e] + self._credit(rank)
        if self.fcap is not None and f > self.fcap:
            f = self.fcap
        c.freq[e] = f
        c.prio[e] = self.age + f
        c.has_prio[e] = True

    def admit(self, e, rank=0):
        e = int(e)
        self.col.fit(e)
        self.held.add(e)
        if not self.keep_ghost:
            self.col.freq[e] = 0.0
        self._use(e, rank)

    def touch(self, e, rank=0):
        self._use(int(e), rank)

    def victim(self, exclude=()):
        c = self.col
        cands = self.held.difference(exclude) if exclude else self.held
        return first_by(cands, c.prio, c.used_at)

    def evicted(self, e):
        e = int(e)
        c = self.col
        c.fit(e)
        p = c.prio[e] if c.has_prio[e] else self.age
        c.has_prio[e] = False
        if p > self.age:
            self.age = p
        self.held.discard(e)
        if not self.keep_ghost:
            c.freq[e] = 0.0
            c.used_at[e] = 0
        elif self.ghost_decay != 1.0:
            c.freq[e] = c.freq[e] * self.ghost_decay

    @property
    def L(self) -> float:
        """The cache age under its conventional name."""
        return self.age


def factory(**params):
    """``factory(**params)`` -> ``f(capacity, n_experts)`` building LFUDA with those parameters."""
    return lambda capacity, n_experts: LFUDA(capacity, n_experts, **params)
