"""Per-expert state held as columns indexed by expert id.

The policies in this package keep no linked lists, ordered dicts or heaps.  Every
piece of per-expert state (a frequency, a priority, the clock value of a queue
entry, a membership code) is one column -- a flat list indexed by expert id -- and
an ordered list of experts is a member set plus a monotonically increasing entry
clock, so "the head of queue Q" is the member with the smallest clock and "move to
the tail" is a fresh clock value.  With at most a few hundred experts per layer and
a resident set of tens, a scan of the members costs about as much as one step
through a linked structure, and the state of a layer is a handful of flat columns.
"""
from __future__ import annotations


class Columns:
    """Named per-expert columns (lists) that grow when an id beyond their length shows up."""

    def __init__(self, n: int, **columns):
        self._n = max(1, int(n))
        self._fill = dict(columns)
        for name, fill in columns.items():
            setattr(self, name, [fill] * self._n)

    def fit(self, e: int) -> None:
        """Make every column long enough to index expert ``e``."""
        if e < self._n:
            return
        grow = max(e + 1, 2 * self._n) - self._n
        for name, fill in self._fill.items():
            getattr(self, name).extend([fill] * grow)
        self._n += grow


def first_by(ids, first, second=None) -> int:
    """The expert id in ``ids`` smallest under the column ``first``, then ``second``, then
    its own id; -1 when ``ids`` is empty."""
    if not ids:
        return -1
    if second is None:
        return min(ids, key=lambda e: (first[e], e))
    return min(ids, key=lambda e: (first[e], second[e], e))
