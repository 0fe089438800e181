"""Expert-cache policies: the contract, the baselines, the resolver and the replay tools.

Drop-in for bigrig_engine/pool.py.  The contract is the reference's
(bigrig_engine/pool.py:29-50): a policy for one layer's cache of ``capacity``
experts out of ``n_experts`` answers

* ``admit(e, rank)``  -- expert ``e`` missed and was just placed,
* ``touch(e, rank)``  -- ``e`` was requested and already resident,
* ``victim()``        -- which resident expert to evict (-1: none), optionally
  ``victim(exclude=...)`` so the pool can protect the experts a step still needs,
* ``evicted(e)``      -- optional notice that ``e`` actually left.

``rank`` is the expert's position in the router's top-k (0 = highest score).

Policies stay host-side Python objects so any module under ``policies/`` plugs
in unchanged; the HBM slab in ``stream.ExpertPool`` follows whatever they decide.
The replay tools (``simulate``, ``belady``, ``evaluate``, ``select_policy``)
reproduce the reference's miss counts exactly on the same request streams; the
golden fixtures under tests/golden/ pin that.
"""
from __future__ import annotations

import heapq
import importlib
import os
from collections import OrderedDict, defaultdict


class Policy:
    """Eviction policy for a single layer's expert cache (bigrig_engine/pool.py:29-50)."""

    name = "policy"

    def __init__(self, capacity: int, n_experts: int):
        self.capacity, self.n_experts = capacity, n_experts

    def admit(self, e: int, rank: int = 0) -> None: ...

    def touch(self, e: int, rank: int = 0) -> None: ...

    def victim(self) -> int:
        raise NotImplementedError


class LRU(Policy):
    """Least recently used (bigrig_engine/pool.py:53-72): evict the oldest use."""

    name = "lru"

    def __init__(self, capacity, n_experts):
        super().__init__(capacity, n_experts)
        self._order: OrderedDict = OrderedDict()     # oldest use first

    def admit(self, e, rank=0):
        self._order[e] = None
        self._order.move_to_end(e)

    def touch(self, e, rank=0):
        self._order.move_to_end(e)

    def victim(self):
        for e in self._order:
            return e
        return -1

    def evicted(self, e):
        self._order.pop(e, None)


class WindowedLFU(Policy):
    """Fewest uses inside a sliding window of requests, ties to the least recent
    (bigrig_engine/pool.py:75-118)."""

    name = "wlfu"

    def __init__(self, capacity, n_experts, window: int = 128):
        super().__init__(capacity, n_experts)
        self.window = window
        self._recent: list = []
        self._uses: dict = defaultdict(int)
        self._held: set = set()
        self._clock = 0
        self._seen: dict = {}

    def _note(self, e):
        self._clock += 1
        self._seen[e] = self._clock
        self._recent.append(e)
        self._uses[e] += 1
        if len(self._recent) > self.window:
            gone = self._recent.pop(0)
            self._uses[gone] -= 1
            if self._uses[gone] <= 0:
                del self._uses[gone]

    def admit(self, e, rank=0):
        self._held.add(e)
        self._note(e)

    def touch(self, e, rank=0):
        self._note(e)

    def victim(self):
        if not self._held:
            return -1
        return min(self._held, key=lambda x: (self._uses.get(x, 0), self._seen.get(x, 0)))

    def evicted(self, e):
        self._held.discard(e)


class BeladyOracle:
    """Marker for the offline optimum; see ``belady``."""
    name = "belady"


def recommended(capacity: int = 0, n_experts: int = 0):
    """The default policy, LFUDA with its tuned parameters (bigrig_engine/pool.py:126-167).

    With a capacity, an instance; without one, the factory ``f(capacity, n_experts)``.
    """
    from .policies.lfuda import factory
    f = factory()
    return f(capacity, n_experts) if capacity else f


_BUILTIN = {"lru": LRU, "windowed_lfu": WindowedLFU, "wlfu": WindowedLFU}


def available_policies() -> list:
    import pkgutil
    from . import policies as _pk
    mods = {m.name for m in pkgutil.iter_modules(_pk.__path__) if not m.name.startswith("_")}
    return sorted(mods | set(_BUILTIN))


def _policy_factory(name: str, capacity: int, n_experts: int):
    """Resolve a policy name to ``factory(capacity, n_experts)`` (bigrig_engine/pool.py:170-216).

    Baselines resolve here.  A module under ``policies/`` may expose its tuned
    configuration three ways, tried in this order: a module-level callable named
    like the module, a ``factory`` that is either ``factory(capacity, n_experts)``
    or ``factory(**kw) -> factory``, or failing both its own policy class.
    A dotted name (``package.module``) resolves the same way from that module, so
    any policy module written against the contract plugs in without living here.
    Unknown names raise ImportError listing what exists.
    """
    if name in _BUILTIN:
        return _BUILTIN[name]
    if name.startswith("_"):
        raise ImportError(f"no policy named {name!r}. Available: "
                          f"{', '.join(available_policies())}")
    path = name if "." in name else f"{__package__}.policies.{name}"
    try:
        mod = importlib.import_module(path)
    except ModuleNotFoundError:
        raise ImportError(f"no policy named {name!r}. Available: "
                          f"{', '.join(available_policies())}") from None
    name = name.rsplit(".", 1)[-1]

    def works(f) -> bool:
        try:
            return hasattr(f(capacity, n_experts), "victim")
        except Exception:
            return False

    named = getattr(mod, name, None)
    if callable(named) and not isinstance(named, type) and works(named):
        return named
    fac = getattr(mod, "factory", None)
    if callable(fac):
        if works(fac):
            return fac
        try:
            inner = fac()
            if works(inner):
                return inner
        except Exception:
            pass
    for attr in dir(mod):
        obj = getattr(mod, attr)
        if isinstance(obj, type) and hasattr(obj, "victim") and obj.__module__ == mod.__name__:
            if works(obj):
                return obj
    raise ImportError(f"no usable policy factory in {mod.__name__}")


def simulate(seq, capacity: int, n_experts: int, policy_factory, ranks=None) -> dict:
    """Replay one layer's request stream through a cache (bigrig_engine/pool.py:252-279).

    A request for a non-resident expert is a miss; when the cache is full the
    policy's victim leaves first (a victim < 0 leaves nothing).
    """
    pol = policy_factory(capacity, n_experts)
    held: set = set()
    hits = misses = 0
    if ranks is None:
        ranks = [0] * len(seq)
    for e, r in zip(seq, ranks):
        e = int(e)
        if e in held:
            hits += 1
            pol.touch(e, r)
            continue
        misses += 1
        if len(held) >= capacity:
            v = pol.victim()
            if v >= 0:
                held.discard(v)
                if hasattr(pol, "evicted"):
                    pol.evicted(v)
        held.add(e)
        pol.admit(e, r)
    n = max(1, hits + misses)
    return {"policy": getattr(pol, "name", "?"), "misses": misses, "hits": hits, "requests": n,
            "miss_rate": misses / n}


def belady(seq, capacity: int) -> dict:
    """Exact offline optimum: evict the resident expert whose next use is furthest away
    (bigrig_engine/pool.py:282-314).  Next uses are precomputed, the resident set is a
    max-heap of next-use positions, so each request costs O(log capacity)."""
    seq = [int(x) for x in seq]
    n = len(seq)
    nxt = [n] * n                       # position of the next request for seq[i], n = never
    last_pos: dict = {}
    for i in range(n - 1, -1, -1):
        nxt[i] = last_pos.get(seq[i], n)
        last_pos[seq[i]] = i
    INF = float("inf")
    held: dict = {}                     # expert -> its current next-use position
    heap: list = []                     # (-next_use, expert), lazily invalidated
    hits = misses = 0
    for i, e in enumerate(seq):
        nu = nxt[i] if nxt[i] < n else INF
        if e in held:
            hits += 1
        else:
            misses += 1
            if len(held) >= capacity:
                while True:
                    neg, v = heapq.heappop(heap)
                    if held.get(v) == -neg:
                        del held[v]
                        break
        held[e] = nu
        heapq.heappush(heap, (-nu, e))
    total = max(1, hits + misses)
    return {"policy": "belady", "misses": misses, "hits": hits, "requests": total,
            "miss_rate": misses / total}


def home() -> str:
    """Where data lives: $BIGRIG_HOME, else the repository root."""
    return os.environ.get("BIGRIG_HOME") or os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def load_trace(tag: str):
    """(idx [layers, tokens, k], seq_bounds) of ``<home>/data/traces/<tag>_full.npz``, or of
    ``tag`` itself when it is a path to an .npz (bigrig_engine/pool.py:317-334)."""
    import numpy as np
    p = tag if tag.endswith(".npz") else os.path.join(home(), "data", "traces", f"{tag}_full.npz")
    d = np.load(p)
    if "idx" in d:
        idx = d["idx"].astype(int)
    else:
        idx = np.argsort(-d["logits"].astype("float32"), axis=-1)[:, :, :8].astype(int)
    return idx, d["seq_bounds"]


def requests(idx, layer: int):
    """One layer's requests flattened in router-rank order within each token, with ranks."""
    L, T, k = idx.shape
    seq = [int(idx[layer, t, r]) for t in range(T) for r in range(k)]
    return seq, [r for _t in range(T) for r in range(k)]


def evaluate(policy_factory, tag: str, capacities, layers=None) -> dict:
    """Mean miss rate per capacity over layers (bigrig_engine/pool.py:337-358)."""
    idx, _ = load_trace(tag)
    E = int(idx.max()) + 1
    layers = range(idx.shape[0]) if layers is None else layers
    out = {}
    for C in capacities:
        rates = []
        for l in layers:
            seq, ranks = requests(idx, l)
            rates.append(simulate(seq, C, E, policy_factory, ranks)["miss_rate"])
        out[C] = sum(rates) / len(rates)
    return out


def select_policy(tag: str, capacity: int, candidates=None, layers: int = 2,
                  n_experts: int | None = None) -> dict:
    """Score candidate policies on a trace against the LRU and Belady bounds and pick the
    one that closes most of the gap (bigrig_engine/pool.py:219-249)."""
    import numpy as np
    names = candidates or [n for n in available_policies() if n not in _BUILTIN]
    idx, _ = load_trace(tag)
    E = n_experts or int(idx.max()) + 1
    streams = [requests(idx, l) for l in range(min(layers, idx.shape[0]))]
    lru = float(np.mean([simulate(s, capacity, E, LRU, r)["miss_rate"] for s, r in streams]))
    bel = float(np.mean([belady(s, capacity)["miss_rate"] for s, _ in streams]))
    out = {"lru": lru, "belady": bel, "policies": {}}
    for n in names:
        try:
            fac = _policy_factory(n, capacity, E)
            v = float(np.mean([simulate(s, capacity, E, fac, r)["miss_rate"] for s, r in streams]))
            out["policies"][n] = {"miss_rate": v,
                                  "gap_pct": (lru - v) / (lru - bel) * 100 if lru > bel else 0.0}
        except Exception as e:  # a broken candidate must not hide a good one
            out["policies"][n] = {"error": str(e)[:120]}
    ok = {n: d for n, d in out["policies"].items() if "gap_pct" in d}
    out["best"] = max(ok, key=lambda n: ok[n]["gap_pct"]) if ok else "lru"
    out["best_gap_pct"] = ok[out["best"]]["gap_pct"] if ok else 0.0
    return out
