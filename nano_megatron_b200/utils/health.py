"""Host-side failure detection between training steps.

Every rank publishes, through the key-value store of the default process
group (the ``torchrun`` TCP store, or the file store of a test), how many
steps it has entered and, when it stops on purpose or on an exception, that
it left and why. Before launching step ``k`` a rank announces it and waits
until every peer has announced step ``k`` too. A peer that left instead, or
that announced nothing new within ``timeout`` seconds, raises
:class:`PeerLost` on every survivor before any of them enqueues a kernel or a
collective of step ``k`` that would wait for the lost rank.

This covers the failures a shared GPU pool allows us to provoke: a rank that
raises, exits, or stops making progress between steps. A rank that dies in
the middle of a step is caught by the process group's own timeout (the
collective in flight ends with an error) or, inside the fused kernels, by
their bounded device-side waits (reported through the CUDA status word).

Store keys (all under ``nmb/peers/<job>``): ``entered/<rank>`` is an integer
counter (``store.add``), ``left/<rank>`` an integer flag and ``why/<rank>``
the reason text. ``store.add(key, 0)`` reads a counter without blocking.
"""

from __future__ import annotations

import time

import torch.distributed as dist


class PeerLost(RuntimeError):
    """Another rank of the job left or stopped making progress."""

    def __init__(self, rank: int, kind: str, detail: str):
        super().__init__(f"rank {rank} {kind}: {detail}")
        self.rank, self.kind, self.detail = rank, kind, detail


class PeerWatch:
    """Step-granular liveness of all ranks of a job.

    ``kind`` of a :class:`PeerLost` is ``"left"`` (the peer announced that it
    stopped; ``detail`` is its reason) or ``"silent"`` (no announcement for
    ``timeout`` seconds: hung, killed, or never started).
    """

    def __init__(self, rank: int, world_size: int, *, store=None, timeout: float = 300.0,
                 job: str = "default", poll_interval: float = 0.005):
        if timeout <= 0:
            raise ValueError(f"PeerWatch timeout must be positive, got {timeout}")
        if store is None:
            store = dist.distributed_c10d._get_default_store()
        self.store, self.rank, self.world = store, rank, world_size
        self.timeout, self.poll = timeout, poll_interval
        self.prefix = f"nmb/peers/{job}"
        self.entered = 0
        self._left = False

    def _key(self, what: str, rank: int) -> str:
        return f"{self.prefix}/{what}/{rank}"

    def leave(self, reason: str) -> None:
        """Announce that this rank stops (idempotent); waiting peers raise ``PeerLost``."""
        if self._left:
            return
        self._left = True
        self.store.set(self._key("why", self.rank), reason[:500])
        self.store.add(self._key("left", self.rank), 1)

    def enter_step(self) -> None:
        """Announce the next step, then block until every peer announced it, or raise."""
        target = self.entered = self.store.add(self._key("entered", self.rank), 1)
        waiting = [r for r in range(self.world) if r != self.rank]
        seen = {r: -1 for r in waiting}
        last_news = time.monotonic()
        while True:
            still = []
            for r in waiting:
                count = self.store.add(self._key("entered", r), 0)
                if count >= target:  # already in this step (or past it): not lost
                    continue
                if self.store.add(self._key("left", r), 0):
                    why = self.store.get(self._key("why", r)).decode(errors="replace")
                    raise PeerLost(r, "left", why)
                if count != seen[r]:
                    seen[r], last_news = count, time.monotonic()
                still.append(r)
            waiting = still
            if not waiting:
                return
            if time.monotonic() - last_news > self.timeout:
                r = waiting[0]
                raise PeerLost(r, "silent", f"no announcement for {self.timeout:g} s "
                                            f"(it entered {seen[r]} steps, this rank {target})")
            time.sleep(self.poll)
