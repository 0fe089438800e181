"""S3-FIFO: a small probationary FIFO, a main FIFO and a ghost FIFO of recent rejects.

Decision rule (bigrig_engine/policies/s3fifo.py:42-144; small queue target 10 %
of capacity, frequency capped at 3, promotion above 1 use, ghost length equal to
the capacity):

* admission places a ghost straight into the main queue, anything else into the
  small queue, with frequency 0 (an expert already queued is left alone);
* a use raises the frequency by one, up to the cap;
* ``victim()`` works the queues until it frees someone.  While the small queue
  holds at least its target (or the main queue is empty) its head leaves it: with
  frequency above 1 it moves to the main queue's tail with frequency 0, otherwise
  it is the victim and becomes the newest ghost (the oldest ghost is forgotten
  once the ghosts exceed their length).  Otherwise the main queue's head leaves
  it: with a positive frequency it re-enters at the tail one lower, otherwise it
  is the victim;
* ``evicted(e)`` drops e from whichever queue still holds it.

State: per expert the clock value at which it entered its queue, a frequency and a
ghost clock (0 = not a ghost); the member sets of the small queue, the main queue
and the ghosts.  A queue's head is its member with the smallest entry clock.
"""
from __future__ import annotations

from ..pool import Policy
from ._columns import Columns, first_by

NONE, SMALL, MAIN = 0, 1, 2


class S3FIFO(Policy):
    name = "s3fifo"

    SMALL_SHARE = 0.10
    FREQ_CAP = 3
    PROMOTE_ABOVE = 1
    GHOST_SHARE = 1.0

    def __init__(self, capacity, n_experts):
        super().__init__(capacity, n_experts)
        self.small_target = max(1, int(round(self.SMALL_SHARE * capacity)))
        self.ghost_len = max(1, int(round(self.GHOST_SHARE * capacity)))
        self.clock = 0
        self.queues = {SMALL: set(), MAIN: set()}
        self.ghosts: set = set()
        self.col = Columns(n_experts, queue=NONE, entered=0, freq=0, ghost_at=0)

    def _enqueue(self, e: int, q: int) -> None:
        self.clock += 1
        self.col.queue[e] = q
        self.col.entered[e] = self.clock
        self.queues[q].add(e)

    def _dequeue(self, e: int) -> None:
        q = self.col.queue[e]
        if q != NONE:
            self.queues[q].discard(e)
        self.col.queue[e] = NONE

    def _head(self, q: int) -> int:
        return first_by(self.queues[q], self.col.entered)

    def _remember(self, e: int) -> None:
        c = self.col
        self.clock += 1
        c.ghost_at[e] = self.clock
        self.ghosts.add(e)
        while len(self.ghosts) > self.ghost_len:
            g = first_by(self.ghosts, c.ghost_at)
            c.ghost_at[g] = 0
            self.ghosts.discard(g)

    def admit(self, e, rank=0):
        e = int(e)
        c = self.col
        c.fit(e)
        if c.queue[e] != NONE:
            return
        c.freq[e] = 0
        if c.ghost_at[e] > 0:
            c.ghost_at[e] = 0
            self.ghosts.discard(e)
            self._enqueue(e, MAIN)
        else:
            self._enqueue(e, SMALL)

    def touch(self, e, rank=0):
        e = int(e)
        c = self.col
        c.fit(e)
        if c.freq[e] < self.FREQ_CAP:
            c.freq[e] += 1

    def _leave_small(self) -> int:
        """Move the small queue's head on; return it if it is the victim, else -1."""
        c = self.col
        e = self._head(SMALL)
        self._dequeue(e)
        if c.freq[e] > self.PROMOTE_ABOVE:
            c.freq[e] = 0
            self._enqueue(e, MAIN)
            return -1
        c.freq[e] = 0
        self._remember(e)
        return e

    def _leave_main(self) -> int:
        """Move the main queue's head on; return it if it is the victim, else -1."""
        c = self.col
        e = self._head(MAIN)
        self._dequeue(e)
        if c.freq[e] > 0:
            c.freq[e] -= 1
            self._enqueue(e, MAIN)
            return -1
        c.freq[e] = 0
        return e

    def victim(self):
        small, main = self.queues[SMALL], self.queues[MAIN]
        while small or main:
            if small and (len(small) >= self.small_target or not main):
                v = self._leave_small()
            else:
                v = self._leave_main()
            if v >= 0:
                return v
        return -1

    def evicted(self, e):
        e = int(e)
        c = self.col
        c.fit(e)
        if c.queue[e] != NONE:
            self._dequeue(e)
        c.freq[e] = 0


def factory(capacity, n_experts):
    return S3FIFO(capacity, n_experts)
