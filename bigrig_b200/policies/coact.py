"""CoAct: co-activation aware eviction (bigrig_engine/policies/coact.py:52-232).

score(x) = S(x) + beta * A(x): S is x's own use count decayed with a half-life
in requests, A is x's affinity to the last ``window`` requests,
``A(x) = sum over recent requests y != x of decay^(t - t_y) * P(x | y)``, with
P(x | y) the share of tokens holding y that also held x (denominator at least
``min_support``).  Token boundaries are recovered from the rank stream: a rank
not above the previous one opens a new token.  Decay is carried by one growing
factor ``g`` (values are stored multiplied by it), renormalised before it
overflows.  The victim is the resident expert with the lowest score, ties to the
least recently used; A is dropped on eviction, S survives as a ghost.

Every floating-point update happens in the same order as the reference so the
scores, and therefore the victims, are bit-for-bit the same.
"""
from __future__ import annotations

from collections import defaultdict, deque

from ..pool import Policy


class CoAct(Policy):
    name = "coact"

    def __init__(self, capacity, n_experts, half_life: float = 128.0, beta: float = 0.8,
                 window: int = 12, max_nb: int = 64, min_support: int = 4,
                 ghost: bool = True, rank_w: float = 0.0):
        super().__init__(capacity, n_experts)
        self.decay = 0.5 ** (1.0 / float(half_life))
        self.beta = float(beta)
        self.W = int(window)
        self.max_nb = int(max_nb)
        self.min_support = int(min_support)
        self.ghost = bool(ghost)
        self.rank_w = float(rank_w)
        self.S: dict = {}
        self.A: dict = {}
        self.resident: set = set()
        self.g = 1.0
        self.t = 0
        self.last: dict = {}
        self.co: dict = defaultdict(dict)   # e -> {partner: tokens holding both}
        self.tok: dict = defaultdict(int)   # e -> tokens holding e
        self.cur: list = []
        self.last_rank = 1 << 30
        self.win: deque = deque()           # [expert, g at request, {x: credit given}]

    def _support(self, y: int) -> int:
        d = self.tok[y]
        return d if d > self.min_support else self.min_support

    def _close_token(self) -> None:
        cur = self.cur
        for i, a in enumerate(cur):
            self.tok[a] += 1
            row = self.co[a]
            for b in cur[i + 1:]:
                row[b] = row.get(b, 0) + 1
                other = self.co[b]
                other[a] = other.get(a, 0) + 1
            if len(row) > 2 * self.max_nb:
                self.co[a] = dict(sorted(row.items(), key=lambda kv: -kv[1])[:self.max_nb])
        self.cur = []

    def _enter(self, e: int) -> None:
        g = self.g
        given: dict = {}
        if self.beta:
            gd = g / self._support(e)
            for x, c in self.co[e].items():
                if x != e and x in self.resident:
                    v = c * gd
                    self.A[x] = self.A.get(x, 0.0) + v
                    given[x] = v
        self.win.append([e, g, given])
        while len(self.win) > self.W:
            _y, _gy, gv = self.win.popleft()
            for x, v in gv.items():
                if x in self.resident:
                    self.A[x] -= v

    def _seed(self, e: int) -> float:
        if not self.beta:
            return 0.0
        total = 0.0
        for entry in self.win:
            y, gy, gv = entry
            if y == e:
                continue
            v = gv.get(e)
            if v is None:
                c = self.co[y].get(e)
                if not c:
                    continue
                v = (c / self._support(y)) * gy
                gv[e] = v
            total += v
        return total

    def _tick(self, e: int, rank: int) -> None:
        if rank <= self.last_rank and self.cur:
            self._close_token()
        self.last_rank = rank
        self.cur.append(e)
        self.t += 1
        self.g /= self.decay
        if self.g > 1e120:
            gg = self.g
            for d in (self.S, self.A):
                for key in d:
                    d[key] /= gg
            for entry in self.win:
                entry[1] /= gg
                for key in entry[2]:
                    entry[2][key] /= gg
            self.g = 1.0

    def _credit(self, rank: int) -> float:
        return self.g * (1.0 + self.rank_w / (1.0 + rank))

    def admit(self, e, rank=0):
        self._tick(e, rank)
        self.resident.add(e)
        self.A[e] = self._seed(e)
        if not self.ghost:
            self.S[e] = 0.0
        self.S[e] = self.S.get(e, 0.0) + self._credit(rank)
        self.last[e] = self.t
        self._enter(e)

    def touch(self, e, rank=0):
        self._tick(e, rank)
        self.S[e] = self.S.get(e, 0.0) + self._credit(rank)
        self.last[e] = self.t
        self._enter(e)

    def victim(self):
        if not self.resident:
            return -1
        b = self.beta
        return min(self.resident,
                   key=lambda x: (self.S.get(x, 0.0) + b * self.A.get(x, 0.0), self.last.get(x, 0)))

    def evicted(self, e):
        self.resident.discard(e)
        self.A.pop(e, None)
        if not self.ghost:
            self.S.pop(e, None)


def factory(**kw):
    """``factory(**params)`` -> ``f(capacity, n_experts)`` with CoAct's parameters bound."""
    return lambda capacity, n_experts: CoAct(capacity, n_experts, **kw)
