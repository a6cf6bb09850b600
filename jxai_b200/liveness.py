"""Host-side liveness of the ranks of a sequence-sharded step.

A rank that leaves between sharded steps (its process ended, it stopped
decoding) would leave the others waiting inside the next step's all-gather
until a timeout -- with their kernels and NCCL's already queued.  A
``Heartbeat`` makes every rank announce each step in a shared key-value store
(``torch.distributed.Store``: TCPStore, FileStore, ...) and, before the step
queues any GPU or NCCL work, wait with a deadline until every rank has
announced it.  A missing rank shows as ``JxError`` with code JX_ERR_TIMEOUT
naming the ranks, on every live rank, with nothing in flight -- the caller then
decides whether to abort the communicator and rebuild.

The reference has no multi-GPU path (it serves one engine process); this is
the failure detection of the sharded extension of src/transformer.cpp:2497-2567.

    hb = Heartbeat(store, rank, world)
    for step in range(n):
        hb.check(step, timeout_s=5.0)        # raises before any work is queued
        jx.attn_step_sharded(...)
"""
from __future__ import annotations

import time
from typing import List

from ._lib import JX_ERR_TIMEOUT, JxError


class Heartbeat:
    """Per-step liveness announcements of `world` ranks in a shared store."""

    def __init__(self, store, rank: int, world: int, prefix: str = "jx/alive",
                 poll_s: float = 0.002):
        self.store, self.rank, self.world = store, rank, world
        self.prefix, self.poll_s = prefix, poll_s

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def beat(self, step: int) -> None:
        """Announces that this rank is about to run `step`."""
        self.store.set(self._key(step, self.rank), b"1")
        if step >= 2:
            # keys two steps back are no longer read by anyone
            try:
                self.store.delete_key(self._key(step - 2, self.rank))
            except Exception:
                pass

    def missing(self, step: int, timeout_s: float) -> List[int]:
        """Ranks that have not announced `step` within timeout_s (empty: all alive)."""
        deadline = time.monotonic() + timeout_s
        waiting = [r for r in range(self.world) if r != self.rank]
        while waiting:
            waiting = [r for r in waiting if not self.store.check([self._key(step, r)])]
            if not waiting or time.monotonic() > deadline:
                break
            time.sleep(self.poll_s)
        return waiting

    def check(self, step: int, timeout_s: float) -> None:
        """beat(step), then wait for every other rank's; JxError(JX_ERR_TIMEOUT)
        names the ranks that did not announce the step in time."""
        self.beat(step)
        gone = self.missing(step, timeout_s)
        if gone:
            raise JxError(JX_ERR_TIMEOUT,
                          f"ranks {gone} did not reach step {step} within {timeout_s} s; "
                          "nothing of the step was queued")
