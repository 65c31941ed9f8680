"""Host-side failure detection between steps for multi-rank runs.

A rank that fails leaves only between steps (no kernel or collective of its own in flight) and says so in the
process group's key-value store; the others check the store before their next launch, so nobody waits inside a
collective for a rank that is gone. A rank that dies without a word stops its heartbeat: a peer whose last beat
is older than `stale` seconds counts as lost. Collectives themselves run under a short process-group timeout as
the last bound.

    hb = Heartbeat(store, rank, world)
    for step in ...:
        hb.check()          # raises PeerLost naming the rank and its reason
        ... launch the step ...
        hb.beat()
"""
from __future__ import annotations

import time


class PeerLost(RuntimeError):
    pass


class Heartbeat:
    def __init__(self, store, rank, world, stale=30.0, prefix="rf"):
        self.store, self.rank, self.world, self.stale, self.prefix = store, rank, world, stale, prefix
        self.beat()

    def _key(self, kind, r):
        return f"{self.prefix}/{kind}/{r}"

    def beat(self):
        self.store.set(self._key("hb", self.rank), repr(time.time()))

    def fail(self, reason):
        """Announce this rank's failure (call before leaving, between steps)."""
        self.store.set(self._key("failed", self.rank), str(reason)[:500])

    def check(self, now=None):
        now = time.time() if now is None else now
        for r in range(self.world):
            if r == self.rank:
                continue
            if self.store.check([self._key("failed", r)]):
                raise PeerLost(f"rank {r} failed: {self.store.get(self._key('failed', r)).decode()}")
            if not self.store.check([self._key("hb", r)]):
                continue                                    # not started yet: the collective timeout bounds it
            last = float(self.store.get(self._key("hb", r)).decode())
            if now - last > self.stale:
                raise PeerLost(f"rank {r}: no heartbeat for {now - last:.1f} s")
