"""Host-side failure detection for tensor-parallel decoding.

Every rank publishes a heartbeat (a wall-clock stamp) in the process group's
key-value store between decode steps, and checks its peers' before launching
the next step.  A peer whose heartbeat is older than `timeout` seconds (it
raised, exited or hangs) is reported before this rank issues a collective
that would wait for it; the caller then aborts the communicator
(Decoder.tp_abort) and leaves or rebuilds the group.  A rank leaves only
between steps, with none of its kernels or collectives in flight.

The device side bounds its own waits (the NVLink all-reduce gives up after
about two seconds and sets AXQ8_ERR_WAIT_TIMEOUT, read by Decoder.tp_health
without a device synchronize), so a peer that fails inside a step ends that
step with an error status instead of a hang.
"""
from __future__ import annotations

import struct
import time


class PeerFailure(RuntimeError):
    """A tensor-parallel peer stopped publishing heartbeats."""

    def __init__(self, ranks: list[int]):
        super().__init__(f"tensor-parallel peer(s) {ranks} stopped answering")
        self.ranks = ranks


class Heartbeat:
    def __init__(self, store, rank: int, world: int, timeout: float = 2.0,
                 prefix: str = "axdec/hb"):
        self.store, self.rank, self.world = store, rank, world
        self.timeout, self.prefix = timeout, prefix
        self.started = time.time()

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self) -> None:
        self.store.set(self._key(self.rank), struct.pack("<d", time.time()))

    def stamps(self) -> dict[int, float | None]:
        out = {}
        for r in range(self.world):
            if r == self.rank:
                continue
            try:
                out[r] = struct.unpack("<d", self.store.get(self._key(r)) if
                                       self.store.check([self._key(r)]) else b"")[0]
            except (struct.error, RuntimeError):
                out[r] = None
        return out

    def dead_peers(self) -> list[int]:
        now = time.time()
        dead = []
        for r, t in self.stamps().items():
            last = t if t is not None else self.started
            if now - last > self.timeout:
                dead.append(r)
        return dead

    def check(self) -> None:
        """Publish this rank's beat and raise PeerFailure if a peer is stale."""
        self.beat()
        dead = self.dead_peers()
        if dead:
            raise PeerFailure(dead)


def guarded_step(decoder, heartbeat: Heartbeat, step):
    """Run `step()` (one decode step of `decoder`) after a heartbeat check; on
    a failed peer abort the decoder's communicator and re-raise.  After the
    step, a non-zero NCCL asynchronous error or device status word (a bounded
    wait that gave up) also aborts and raises."""
    try:
        heartbeat.check()
    except PeerFailure:
        decoder.tp_abort()
        raise
    result = step()
    nccl_err, status = decoder.tp_health()
    if nccl_err or status:
        decoder.tp_abort()
        raise RuntimeError(f"tensor-parallel step failed: nccl error {nccl_err}, "
                           f"device status {status}")
    return result
