"""Residency bookkeeping of one layer's expert pool: which expert holds which slot.

``SlotTable`` is the host half of ``stream.ExpertPool``: the expert<->slot tables,
the request counters and the conversation with the eviction policy.  It moves no
bytes; the pool subclass owns the HBM slab and the copies.

The order of decisions is the reference pool's (bigrig_engine/stream.py:622-780),
because the slot ids it hands out are compared with the reference's on a replayed
decode stream:

* a request batch is looked up in the order given; every hit is reported to the
  policy (``touch``) in that order and the misses are returned in that order;
* a slot is freed from the free list while it has any (last freed first out),
  else the policy names a victim (passing the protected experts when its
  ``victim`` accepts ``exclude``); a victim that is protected, absent or not an
  expert is refused and the slot admitted longest ago among unprotected ones is
  taken instead; the policy hears ``evicted`` only for the expert really evicted;
* an admission stamps its slot with the admission clock and tells the policy
  ``admit`` with the rank the expert was requested at.
"""
from __future__ import annotations

import inspect

import numpy as np

from .policies._columns import first_by
from .pool import _policy_factory


class SlotTable:
    """Expert<->slot tables and counters for ``capacity`` slots over ``n_experts`` experts."""

    def __init__(self, layer: int, n_experts: int, capacity: int, policy="lfuda"):
        if not 1 <= capacity <= n_experts:
            raise ValueError(
                f"capacity must be in [1, {n_experts}] for layer {layer}, got {capacity}: a "
                f"pool can hold no more experts than the layer has, and an empty one cannot "
                f"serve a token.")
        self.layer, self.n_experts, self.capacity = layer, n_experts, capacity
        self.policy = (_policy_factory(policy, capacity, n_experts)(capacity, n_experts)
                       if isinstance(policy, str) else policy)
        try:
            params = inspect.signature(self.policy.victim).parameters
            self._victim_takes_exclude = "exclude" in params
        except (TypeError, ValueError):
            self._victim_takes_exclude = False
        self._tells_evictions = hasattr(self.policy, "evicted")
        self.g2s = np.full(n_experts, -1, dtype=np.int32)     # expert -> slot, -1 absent
        self.s2g = np.full(capacity, -1, dtype=np.int32)      # slot -> expert, -1 free
        self._admitted_at = np.zeros(capacity, dtype=np.int64)
        self._admit_clock = 0
        self._free = list(range(capacity))
        self._n_resident = 0
        self._miss_rank: dict = {}
        self._g2s_dirty = True
        self.uses = np.zeros(n_experts, dtype=np.int64)
        self.hits = self.misses = self.admits = self.evicts = 0

    # -- lookups ---------------------------------------------------------------
    def slot_of(self, e: int) -> int:
        return int(self.g2s[e])

    @property
    def full(self) -> bool:
        """Every expert resident: no request can miss (stream.py:782-789)."""
        return self.capacity == self.n_experts and self._n_resident == self.n_experts

    # -- requests --------------------------------------------------------------
    def touch(self, experts, ranks=None) -> list:
        """Count a request for each expert (router rank ``ranks``, default 0), tell the
        policy about the resident ones and return the rest, in request order."""
        ex = experts.tolist() if isinstance(experts, np.ndarray) else [int(e) for e in experts]
        if ranks is None:
            rk = [0] * len(ex)
        else:
            rk = ranks.tolist() if isinstance(ranks, np.ndarray) else [int(r) for r in ranks]
        slots = self.g2s[ex].tolist() if ex else []
        uses, note = self.uses, self.policy.touch
        need, miss_rank = [], {}
        for e, r, slot in zip(ex, rk, slots):
            uses[e] += 1
            if slot < 0:
                need.append(e)
                miss_rank[e] = r
            else:
                note(e, r)
        self.hits += len(ex) - len(need)
        self.misses += len(need)
        self._miss_rank = miss_rank
        return need

    # -- slot turnover ---------------------------------------------------------
    def _policy_choice(self, protect: set) -> int:
        v = self.policy.victim(exclude=protect) if self._victim_takes_exclude else self.policy.victim()
        if v is None:
            return -1
        v = int(v)
        ok = 0 <= v < self.n_experts and v not in protect and self.g2s[v] >= 0
        return v if ok else -1

    def _oldest_unprotected(self, protect: set) -> int:
        s2g = self.s2g.tolist()
        slots = [j for j, e in enumerate(s2g) if e >= 0 and e not in protect]
        slot = first_by(slots, self._admitted_at.tolist())
        return -1 if slot < 0 else s2g[slot]

    def _victim(self, protect=()) -> int:
        """A slot for the next admission: a free one, else the policy's victim's."""
        if self._free:
            return self._free.pop()
        if not isinstance(protect, (set, frozenset)):
            protect = {int(x) for x in protect}
        ev = self._policy_choice(protect)
        if ev < 0:
            ev = self._oldest_unprotected(protect)
        if ev < 0:
            raise RuntimeError(
                f"layer {self.layer}: all {self.capacity} slots hold experts this step still "
                f"uses, so none can be evicted; the capacity must be at least top-k.")
        slot = int(self.g2s[ev])
        if self._tells_evictions:
            self.policy.evicted(ev)
        self.g2s[ev] = -1
        self.s2g[slot] = -1
        self._n_resident -= 1
        self._g2s_dirty = True
        self.evicts += 1
        return slot

    def _placed(self, e: int, slot: int) -> None:
        """Record that expert ``e`` now occupies ``slot`` (its bytes are on their way)."""
        self._n_resident += int(self.s2g[slot] < 0)
        self.g2s[e] = slot
        self.s2g[slot] = e
        self._g2s_dirty = True
        self._admit_clock += 1
        self._admitted_at[slot] = self._admit_clock
        self.policy.admit(e, int(self._miss_rank.get(e, 0)))
        self.admits += 1

    def stats(self) -> dict:
        n = self.hits + self.misses
        return dict(layer=self.layer, capacity=self.capacity, n_experts=self.n_experts,
                    hits=self.hits, misses=self.misses, miss_rate=(self.misses / n) if n else 0.0,
                    admits=self.admits, evicts=self.evicts)
