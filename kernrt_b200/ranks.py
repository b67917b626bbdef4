"""Host-side failure detection between steps for multi-rank runs.

Ranks run the chain on their own row shards with no exchange on the data path,
so a rank that dies between steps would only show up at the next timing
collective (or never, if the others stop waiting).  StepWatch makes it visible
on the host first: before a step each rank announces it in the process group's
key-value store and waits, for a bounded time, for every other rank's
announcement of the same step.  A rank that does not arrive raises RankFailure
naming it, before any kernel or collective of that step is launched, so no
device work is left waiting on a dead peer.
"""
from __future__ import annotations

import datetime


class RankFailure(RuntimeError):
    """One or more ranks did not reach a step within the watch's timeout."""

    def __init__(self, step: str, missing: list[int]):
        super().__init__(f"rank{'s' if len(missing) > 1 else ''} {', '.join(map(str, missing))} "
                         f"did not reach step {step!r}")
        self.step = step
        self.missing = missing


class StepWatch:
    def __init__(self, store, rank: int, world: int, timeout_s: float = 30.0, prefix: str = "kernrt/step"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout = datetime.timedelta(seconds=timeout_s)
        self.prefix = prefix

    def _key(self, step: str, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def enter(self, step: str) -> None:
        """Announce `step`, then wait for every other rank to announce it."""
        self.store.set(self._key(step, self.rank), "1")
        missing = []
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                self.store.wait([self._key(step, r)], self.timeout)
            except Exception:  # the store's timeout (or its connection closed)
                missing.append(r)
        if missing:
            raise RankFailure(step, missing)
