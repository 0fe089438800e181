"""Per-expert state held as columns indexed by expert id.

The policies in this package keep no linked lists, ordered dicts or heaps.  Every
piece of per-expert state (a frequency, a priority, the clock value of a queue
entry, a membership code) is one numpy column of length ``n_experts``; an ordered
list of experts is a membership code plus a monotonically increasing entry clock,
so "the head of queue Q" is the member with the smallest clock and "move to the
tail" is a fresh clock value.  With at most a few hundred experts per layer a
masked ``argmin`` over a column costs about as much as one step through a Python
container, and the state of a whole layer is a handful of flat arrays.
"""
from __future__ import annotations

import numpy as np


class Columns:
    """Named per-expert columns that grow when an id beyond the current length shows up."""

    def __init__(self, n: int, **columns):
        self._n = max(1, int(n))
        self._spec = {}
        for name, (dtype, fill) in columns.items():
            self._spec[name] = (dtype, fill)
            setattr(self, name, np.full(self._n, fill, dtype=dtype))

    def fit(self, e: int) -> None:
        """Make every column long enough to index expert ``e``."""
        if e < self._n:
            return
        n = max(e + 1, 2 * self._n)
        for name, (dtype, fill) in self._spec.items():
            old = getattr(self, name)
            new = np.full(n, fill, dtype=dtype)
            new[:old.shape[0]] = old
            setattr(self, name, new)
        self._n = n


def first_by(mask: np.ndarray, *keys: np.ndarray) -> int:
    """The expert id that is smallest under the keys, compared in order, among ``mask``.

    Ties after the last key go to the lowest id.  Returns -1 when ``mask`` is empty."""
    ids = np.flatnonzero(mask)
    for key in keys:
        if ids.size <= 1:
            break
        vals = key[ids]
        ids = ids[vals == vals.min()]
    return int(ids[0]) if ids.size else -1
