"""Host-side failure detection for multi-process jobs.

A ``Heartbeat`` posts ``hb/<rank>`` = wall time into the job's
``torch.distributed`` store from a daemon thread; ``check()`` raises
``RankFailure`` naming the ranks whose heartbeat is older than ``timeout``
or that posted ``fail/<rank>`` (``report_failure``, e.g. from an exception
handler). Ranks call ``check()`` between steps - before launching the next
collective - so a dead or failed peer ends the job with an error instead of a
collective that waits until its process-group timeout. Device-side waits are
bounded separately (kernels record a status word after 2 s).

Reference: rlx-tune src/distributed.rs (TCP rendezvous, heartbeats, rank
failure surfaced as an error on the surviving ranks) and the fault-injection
knobs of its trainer; here faults are only ever made on the host.
"""
from __future__ import annotations

import threading
import time


class RankFailure(RuntimeError):
    def __init__(self, ranks, why):
        self.ranks = sorted(ranks)
        super().__init__(f"ranks {self.ranks} failed: {why}")


class Heartbeat:
    def __init__(self, store, rank: int, world: int, interval: float = 0.2, timeout: float = 2.0,
                 prefix: str = "b200health"):
        self.store, self.rank, self.world = store, rank, world
        self.interval, self.timeout, self.prefix = interval, timeout, prefix
        self._stop = threading.Event()
        self._beat()
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()

    def _key(self, kind, r):
        return f"{self.prefix}/{kind}/{r}"

    def _beat(self):
        self.store.set(self._key("hb", self.rank), repr(time.time()))

    def _run(self):
        while not self._stop.wait(self.interval):
            try:
                self._beat()
            except Exception:
                return

    def report_failure(self, why: str = "error"):
        self.store.set(self._key("fail", self.rank), why)

    def stop(self):
        self._stop.set()
        self._t.join(timeout=2 * self.interval + 1)

    def check(self, wait_for_first: float = 10.0):
        """Raise RankFailure if any peer is stale or reported a failure."""
        now = time.time()
        failed, why = set(), []
        for r in range(self.world):
            if r == self.rank:
                continue
            fk = self._key("fail", r)
            if self.store.check([fk]):
                failed.add(r)
                why.append(f"{r}: {self.store.get(fk).decode()}")
                continue
            hk = self._key("hb", r)
            deadline = time.time() + wait_for_first
            while not self.store.check([hk]):
                if time.time() > deadline:
                    failed.add(r)
                    why.append(f"{r}: never joined")
                    break
                time.sleep(0.05)
            else:
                age = now - float(self.store.get(hk).decode())
                if age > self.timeout:
                    failed.add(r)
                    why.append(f"{r}: heartbeat {age:.1f}s old")
        if failed:
            raise RankFailure(failed, "; ".join(why))
