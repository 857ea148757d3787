"""Host-side liveness for ring ranks.

The reference aborts the whole MPI job on any CUDA/NCCL error and has no
timeouts, so a dead peer hangs every other rank (ring/attention/bench/
ring_attention_nccl_gpu_bench.cu:28-45). Here a rank that stops taking part is
detected on the host before the next launch: every rank publishes a heartbeat
(its call counter, or "left") in the process group's key-value store, and
`check(step)` waits a bounded time for every peer to reach `step`. A peer that
left, or that stays silent past the timeout, raises PeerLostError, so no
kernel is ever launched that would wait on a missing neighbour. Kernels
themselves also bound every wait (see KernelStatusError)."""
from __future__ import annotations

import time

import torch.distributed as dist


class PeerLostError(RuntimeError):
    """A ring peer left or stopped publishing heartbeats."""


class RingHealth:
    def __init__(self, group=None, store=None, prefix: str = "mgfa/health"):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.store = store if store is not None else dist.distributed_c10d._get_default_store()
        self.prefix = prefix
        self._last = -1  # last call this rank announced

    def _key(self, r: int) -> str:
        return f"{self.prefix}/{r}"

    def beat(self, step: int) -> None:
        """Announce that this rank is about to run call `step`."""
        self._last = step
        self.store.set(self._key(self.rank), str(step))

    def leave(self) -> None:
        """Announce a clean departure (call between steps, with no kernel in flight).
        The value keeps the last call this rank took part in, so a peer still
        checking that call is not told the rank is gone."""
        self.store.set(self._key(self.rank), f"left:{self._last}")

    def check(self, step: int, timeout_s: float = 10.0, poll_s: float = 0.01) -> None:
        """Return once every peer has announced `step` (or later); raise
        PeerLostError when one left or stays behind for `timeout_s`."""
        deadline = time.monotonic() + timeout_s
        pending = [r for r in range(self.world) if r != self.rank]
        while pending:
            still = []
            for r in pending:
                if not self.store.check([self._key(r)]):
                    still.append(r)
                    continue
                v = self.store.get(self._key(r)).decode()
                if v.startswith("left"):
                    if int(v.split(":", 1)[1]) >= step:
                        continue  # it took part in this call before leaving
                    raise PeerLostError(f"rank {r} left the ring")
                if int(v) < step:
                    still.append(r)
            pending = still
            if pending:
                if time.monotonic() > deadline:
                    raise PeerLostError(f"rank(s) {pending} did not reach call {step} within "
                                        f"{timeout_s:.1f} s")
                time.sleep(poll_s)

    def step(self, step: int, timeout_s: float = 10.0) -> None:
        self.beat(step)
        self.check(step, timeout_s)

    def gate(self, timeout_s: float = 10.0) -> int:
        """Before a ring call: announce the next call and wait (bounded) until
        every peer announced it too. Raises PeerLostError -- before anything is
        launched -- when a peer left or stays silent. Returns the call index."""
        call = self._last + 1
        self.step(call, timeout_s)
        return call
