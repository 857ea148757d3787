"""Executable model of the ring transports' flag protocols, for race checks.

The native engines move KV shards between ranks through receive slots in each
rank's symmetric buffer, ordered only by flag words (arrival counters written by
the sender, credit words written back by the receiver) and by CUDA stream
order on each rank. This module restates those rules as small state machines,
one per concurrent activity (the consumer and producer sides of an attention
kernel, a standalone push kernel, a release kernel), and lets a seeded random
scheduler interleave the activities of all ranks. The checker fails when

  * a store into a slot begins while a reader of that slot is still reading, or
  * a reader finds in its slot anything but the shard it expects (owner, call).

Models:
  fused      RingEngine forward, transport in the attention kernel: step t
             reads slot t % 3 (own buffers at t = 0), pushes into the right
             neighbour's slot (t + 1) % 3 once the credit allows, and the last
             CTA releases slot t % 3 to the left neighbour after every read
             (including the push's) is done. Step t + 1 may start while step t
             runs (dependent launch), but its epilogue waits for step t's grid
             (griddepcontrol.wait), so it releases and finishes after step t;
             the first step of a call starts after the previous call's last
             step has finished. `small_grid=True` lets dependent launches chain
             more than one step deep (grids smaller than the GPU);
             `chain_guard=False` drops the engine's rule that turns dependent
             launch off for those grids at P >= 5, which races;
             `cumulative=True` models arrival counters that are never reset,
             with the host's cumulative targets (dependent launch always on).
  push, ce   RingEngine forward with the transport on a second stream (the
             standalone push kernel or the copy engine): the attention kernel
             only waits; the transfer of step t starts after the compute
             stream's earlier work; a release kernel frees the slot after both.
  backward   RingBwdEngine: per step the dK/dV kernel consumes slot t % 3 (K, V
             and the incoming fp32 accumulators), pushes K/V and the updated
             accumulators into the right neighbour's slot (t + 1) % 3 -- at the
             last step into its home buffer -- and the dQ kernel releases slot
             t % 3; each call ends by waiting for, reading and releasing the
             rank's own home buffer (csrc/comm/ring_bwd_engine.hpp).
  exchange   RingExchange (two slots, the rank's own shard starts in slot 0):
             step t forwards slot t % 2 into the right neighbour's slot
             (t + 1) % 2 and releases slot t % 2 after reading it; the caller
             reads the received slot between steps (sequential order).
             `release_slot0=False` drops the step-0 release of slot 0 (the
             protocol before that fix) and races for P >= 3;
             `wait_received=False` reads the received slot as soon as the
             rank's own step is done, without waiting for its arrivals (a race
             at any P).

The flag arithmetic (slot indices, the host's per-slot use counters, credit
targets and published credit values) follows csrc/comm/ring_engine.hpp,
csrc/comm/ring_bwd_engine.hpp and csrc/comm/ring_exchange.hpp.
"""
from __future__ import annotations

import random
from dataclasses import dataclass, field
from typing import Callable, Dict, Generator, List, Optional, Tuple


class ProtocolViolation(AssertionError):
    """A slot was overwritten while being read, or held the wrong shard."""


@dataclass
class Slot:
    content: Optional[Tuple[int, int]] = None   # (owner, call) of the last completed store
    readers: int = 0                            # reads in progress
    writing: bool = False


@dataclass
class Rank:
    slots: List[Slot]
    arrivals: List[int]
    credit: List[int]                 # credit words this rank holds (written by its right)
    uses: List[int]                   # host-side use counters of its own slots
    started: Dict[Tuple[int, int], bool] = field(default_factory=dict)
    finished: Dict[Tuple[int, int], bool] = field(default_factory=dict)
    pushed: Dict[Tuple[int, int], bool] = field(default_factory=dict)


Wait = Callable[[], bool]
Proc = Generator[Wait, None, None]


class Model:
    def __init__(self, world: int, kind: str, calls: int = 2, seed: int = 0,
                 release_slot0: bool = True, wait_received: bool = True,
                 small_grid: bool = False, chain_guard: bool = True, cumulative: bool = False,
                 mutation: Optional[str] = None):
        if kind not in ("fused", "push", "ce", "exchange", "backward"):
            raise ValueError(kind)
        self.P, self.kind, self.calls = world, kind, calls
        self.release_slot0 = release_slot0
        self.wait_received = wait_received
        # fused engine: with grids larger than the GPU holds at once, step t+2
        # cannot start before step t completed (step t+1's CTAs must all have
        # started, and its first ones wait for step t); small grids let the
        # chain run deeper. The engine turns dependent launch off for small
        # grids when P >= 5 (chain_guard).
        self.small_grid = small_grid
        self.pdl = not (chain_guard and small_grid and world >= 5)
        # fused engine with arrival counters that are never reset: the host
        # keeps each slot's cumulative expected arrivals and the consumer waits
        # for that total (the design that keeps dependent launch on everywhere)
        self.cumulative = cumulative
        if cumulative:
            self.pdl = True
        self.expected = [[0] * (2 if kind == "exchange" else 3) for _ in range(world)]
        # deliberately broken variants, to show the checker catches them:
        # "credit"  credit targets one lower (a push may overwrite one use early)
        # "release" the fused kernel hands its slot back before its reads end
        self.mutation = mutation
        self.rng = random.Random(seed)
        n_slots = 2 if kind == "exchange" else 3
        self.nslots = n_slots
        self.ranks = [Rank([Slot() for _ in range(n_slots)], [0] * n_slots, [0] * n_slots,
                           [0] * n_slots) for _ in range(world)]
        # backward engine: each rank's home buffer (its finished dK/dV)
        self.home = [Slot() for _ in range(world)]
        self.home_arrivals = [0] * world
        self.home_credit = [0] * world
        self.home_uses = [0] * world
        self.procs: List[Proc] = []
        self.waits: List[Optional[Wait]] = []

    # ------------------------------------------------------------ slot access
    def _begin_read(self, r: int, s: int, expect: Tuple[int, int]) -> None:
        slot = self.ranks[r].slots[s]
        if slot.writing:
            raise ProtocolViolation(f"rank {r} slot {s}: read began during a store")
        if slot.content != expect:
            raise ProtocolViolation(f"rank {r} slot {s}: holds {slot.content}, expected {expect}")
        slot.readers += 1

    def _end_read(self, r: int, s: int) -> None:
        self.ranks[r].slots[s].readers -= 1

    def _begin_write(self, r: int, s: int) -> None:
        slot = self.ranks[r].slots[s]
        if slot.readers:
            raise ProtocolViolation(f"rank {r} slot {s}: store began while {slot.readers} "
                                    "reader(s) still read it")
        slot.writing = True

    def _end_write(self, r: int, s: int, data: Tuple[int, int]) -> None:
        slot = self.ranks[r].slots[s]
        slot.writing = False
        slot.content = data

    # ------------------------------------------------------------ engine (forward)
    def _engine_call(self, r: int, c: int) -> Proc:
        """Host loop of one forward() call on rank r: enqueues the step kernels."""
        P, R = self.P, self.ranks[r]
        right, left = (r + 1) % P, (r - 1) % P
        for t in range(P):
            s, sn = t % 3, (t + 1) % 3
            owner = (r - t) % P
            # parameters fixed at enqueue time (host counters)
            credit_target = R.uses[sn] - (1 if self.mutation == "credit" else 0)
            credit_value = R.uses[s] + 1
            key = (c, t)
            prev = (c, t - 1) if t > 0 else ((c - 1, P - 1) if c > 0 else None)
            if self.kind == "fused":
                need = 1
                if self.cumulative and t > 0:
                    self.expected[r][s] += 1
                    need = self.expected[r][s]
                self._spawn(self._fused_kernel(r, c, t, s, sn, owner, credit_target,
                                               credit_value, prev, right, left, need))
            else:
                self._spawn(self._unfused_compute(r, c, t, s, owner, credit_value, prev, left))
                if t < P - 1:
                    self._spawn(self._unfused_transfer(r, c, t, s, sn, owner, credit_target,
                                                       prev, right))
            if t > 0:
                R.uses[s] += 1
            yield lambda: True
        return

    def _fused_kernel(self, r, c, t, s, sn, owner, credit_target, credit_value, prev, right,
                      left, need=1) -> Proc:
        R = self.ranks[r]
        key = (c, t)
        if prev is not None:
            if t == 0 or not self.pdl:   # fully ordered after the previous step
                yield lambda: R.finished.get(prev, False)
            else:        # dependent launch: may start once the previous step started
                yield lambda: R.started.get(prev, False)
                if not self.small_grid and t >= 2:
                    yield lambda: R.finished.get((c, t - 2), False)
        R.started[key] = True
        reading = False
        if t > 0:
            yield lambda: R.arrivals[s] >= need
            self._begin_read(r, s, (owner, c))
            reading = True
            if self.mutation == "release":
                self.ranks[left].credit[s] = credit_value
        if t < self.P - 1:
            yield lambda: R.credit[sn] >= credit_target
            self._begin_write(right, sn)
            yield lambda: True
            self._end_write(right, sn, (owner, c))
            self.ranks[right].arrivals[sn] += 1
        yield lambda: True                   # the rest of the attention work
        if t > 0 and prev is not None:
            # the epilogue's griddepcontrol.wait: the previous step's grid has
            # completed before any CTA merges, releases or exits
            yield lambda: R.finished.get(prev, False)
        if reading:
            self._end_read(r, s)
            # last CTA: rearm the counter (unless counts accumulate), then hand
            # the slot back
            if not self.cumulative:
                R.arrivals[s] = 0
            self.ranks[left].credit[s] = credit_value
        R.finished[key] = True

    def _unfused_compute(self, r, c, t, s, owner, credit_value, prev, left) -> Proc:
        R = self.ranks[r]
        key = (c, t)
        if prev is not None:   # stream order: the previous step, its transfer and release
            yield lambda: R.finished.get(prev, False) and R.pushed.get(prev, True)
        R.started[key] = True
        if t > 0:
            yield lambda: R.arrivals[s] >= 1
            self._begin_read(r, s, (owner, c))
            yield lambda: True
            self._end_read(r, s)
            # release kernel: after the attention and this step's transfer
            yield lambda: R.pushed.get(key, True)
            R.arrivals[s] = 0
            self.ranks[left].credit[s] = credit_value
        else:
            yield lambda: True
        R.finished[key] = True

    def _unfused_transfer(self, r, c, t, s, sn, owner, credit_target, prev, right) -> Proc:
        R = self.ranks[r]
        key = (c, t)
        R.pushed[key] = False
        if prev is not None:  # starts after the compute stream's earlier work
            yield lambda: R.finished.get(prev, False) and R.pushed.get(prev, True)
        reading = False
        if t > 0:
            yield lambda: R.arrivals[s] >= 1
            self._begin_read(r, s, (owner, c))
            reading = True
        yield lambda: R.credit[sn] >= credit_target
        self._begin_write(right, sn)
        yield lambda: True
        self._end_write(right, sn, (owner, c))
        if reading:
            self._end_read(r, s)
        self.ranks[right].arrivals[sn] += 1
        R.pushed[key] = True

    # ------------------------------------------------------------ backward engine
    def _backward_call(self, r: int, c: int) -> Proc:
        """One backward() on rank r: per step the dK/dV kernel then the dQ kernel
        (stream order, no dependent launch), then the wait for the home buffer,
        its copy-out and its release."""
        P, R = self.P, self.ranks[r]
        right, left = (r + 1) % P, (r - 1) % P
        for t in range(P):
            s, sn = t % 3, (t + 1) % 3
            owner = (r - t) % P
            credit_target, credit_value = R.uses[sn], R.uses[s] + 1
            home_target = self.home_uses[r]
            # dK/dV kernel: consume slot s (K, V and the incoming accumulators),
            # push K/V and the updated accumulators into the right neighbour's
            # slot sn -- or, at the last step, its home buffer
            if t > 0:
                yield lambda s=s: R.arrivals[s] >= 1
                self._begin_read(r, s, (owner, c))
            if t < P - 1:
                yield lambda sn=sn, ct=credit_target: R.credit[sn] >= ct
                self._begin_write(right, sn)
                yield lambda: True
                self._end_write(right, sn, (owner, c))
                self.ranks[right].arrivals[sn] += 1
            else:
                yield lambda ht=home_target: self.home_credit[r] >= ht
                h = self.home[right]
                if h.readers:
                    raise ProtocolViolation(f"rank {right} home: store began while it was read")
                h.writing = True
                yield lambda: True
                h.writing = False
                h.content = (owner, c)
                self.home_arrivals[right] += 1
            if t > 0:
                self._end_read(r, s)
            # dQ kernel: reads slot s again, then its last CTA releases it
            if t > 0:
                self._begin_read(r, s, (owner, c))
                yield lambda: True
                self._end_read(r, s)
                R.arrivals[s] = 0
                self.ranks[left].credit[s] = credit_value
                R.uses[s] += 1
        # the finished dK/dV of this rank arrive in its home buffer
        yield lambda: self.home_arrivals[r] >= 1
        h = self.home[r]
        if h.writing or h.content != (r, c):
            raise ProtocolViolation(f"rank {r} home: holds {h.content}, expected {(r, c)}")
        h.readers += 1
        yield lambda: True
        h.readers -= 1
        self.home_arrivals[r] = 0
        self.home_credit[left] = self.home_uses[r] + 1
        self.home_uses[r] += 1

    # ------------------------------------------------------------ RingExchange
    def _exchange_call(self, r: int, c: int) -> Proc:
        """One rotation on rank r in the sequential order: own shard into slot 0,
        then per step a transfer and a read of the received slot."""
        P, R = self.P, self.ranks[r]
        right, left = (r + 1) % P, (r - 1) % P
        if c > 0:  # rotations are separated by a barrier
            yield lambda: all(x.finished.get((c - 1, "rot"), False) for x in self.ranks)
        self._begin_write(r, 0)
        self._end_write(r, 0, (r, c))
        for t in range(P - 1):
            s, sn = t % 2, (t + 1) % 2
            owner = (r - t) % P
            credit_target = R.uses[sn]
            consume = t > 0 or self.release_slot0
            credit_value = R.uses[s] + 1
            if t > 0:
                yield lambda s=s: R.arrivals[s] >= 1
            self._begin_read(r, s, (owner, c))
            yield lambda sn=sn, ct=credit_target: R.credit[sn] >= ct
            self._begin_write(right, sn)
            yield lambda: True
            self._end_write(right, sn, (owner, c))
            self._end_read(r, s)
            self.ranks[right].arrivals[sn] += 1
            if consume:
                R.arrivals[s] = 0
                self.ranks[left].credit[s] = credit_value
                R.uses[s] += 1
            # the caller reads the received slot before the next step: after
            # waiting for its arrivals (wait_received), or -- the race -- as soon
            # as its own step is done
            if self.wait_received:
                yield lambda sn=sn: R.arrivals[sn] >= 1
            else:
                yield lambda: True
            self._begin_read(r, sn, ((owner - 1) % P, c))
            yield lambda: True
            self._end_read(r, sn)
        # release of the last slot
        s = (P - 1) % 2
        yield lambda s=s: R.arrivals[s] >= 1
        R.arrivals[s] = 0
        self.ranks[left].credit[s] = R.uses[s] + 1
        R.uses[s] += 1
        R.finished[(c, "rot")] = True

    # ------------------------------------------------------------ scheduler
    def _spawn(self, proc: Proc) -> None:
        self.procs.append(proc)
        self.waits.append(None)
        self._advance(len(self.procs) - 1)

    def _advance(self, i: int) -> None:
        try:
            self.waits[i] = next(self.procs[i])
        except StopIteration:
            self.waits[i] = None
            self.procs[i] = None

    def run(self, max_events: int = 200000) -> int:
        """Interleaves every activity at random until all finish; returns the
        number of scheduling events. Raises ProtocolViolation on a race and
        RuntimeError on a deadlock."""
        for r in range(self.P):
            if self.kind == "exchange":
                calls = [self._exchange_call(r, c) for c in range(self.calls)]
            elif self.kind == "backward":
                calls = [self._backward_call(r, c) for c in range(self.calls)]
            else:
                calls = [self._engine_call(r, c) for c in range(self.calls)]
            self._spawn(_chain(calls))
        events = 0
        while any(p is not None for p in self.procs):
            ready = [i for i, (p, w) in enumerate(zip(self.procs, self.waits))
                     if p is not None and w is not None and w()]
            if not ready:
                raise RuntimeError("deadlock: no activity can proceed")
            self._advance(self.rng.choice(ready))
            events += 1
            if events > max_events:
                raise RuntimeError("event budget exhausted")
        return events


def engine_plan(world: int, rank: int, calls: int) -> List[List[int]]:
    """The forward engine's flag values as this model derives them (the
    arithmetic of `_engine_call`): one row per step of `calls` consecutive
    calls, [call, t, slot, next_slot, credit_target, credit_value, tag]. The
    native engine's RingEngine.plan() must produce the same rows."""
    uses = [0, 0, 0]
    rows = []
    for c in range(calls):
        for t in range(world):
            s, sn = t % 3, (t + 1) % 3
            owner = (rank - t) % world
            rows.append([c, t, s, sn, uses[sn], uses[s] + 1, (owner + 1) | (c << 8)])
            if t > 0:
                uses[s] += 1
    return rows


def backward_plan(world: int, rank: int, calls: int) -> List[List[int]]:
    """The backward engine's flag values as `_backward_call` derives them: rows
    [call, t, slot, next_slot, credit_target, credit_value, tag,
    home_credit_target]; RingBwdEngine.plan() must produce the same rows."""
    rows = []
    for r in engine_plan(world, rank, calls):
        r = list(r)
        r[6] |= 0x80000000  # backward tags carry the top bit
        rows.append(r + [r[0]])  # one home use per earlier call
    return rows


def _chain(gens: List[Proc]) -> Proc:
    for g in gens:
        yield from g


def check(world: int, kind: str, calls: int = 2, seeds: int = 50, release_slot0: bool = True,
          wait_received: bool = True, small_grid: bool = False, chain_guard: bool = True,
          cumulative: bool = False, mutation: Optional[str] = None) -> None:
    """Runs `seeds` random interleavings; raises on the first violation."""
    for seed in range(seeds):
        Model(world, kind, calls, seed, release_slot0, wait_received, small_grid,
              chain_guard, cumulative, mutation).run()


# ---------------------------------------------------------------- one-launch ring
class OneLaunchModel:
    """The one-launch ring (csrc/comm/ring_engine_p.hpp, kernels/attn_fwd_persistent.cu).

    Every rank has one receive slot per ring step s = 1..P-1 and kv-head chunk
    c; the shard in slot (s, c) belongs to owner (rank - s) mod P. One kernel per
    call and rank, launched after the rank's previous call finished (stream
    order), runs concurrently:
      * `workers` push workers (the push warps): wait until the right neighbour
        finished the previous call (credit >= call), then for every chunk c and
        step s < P-1, in that order, wait for unit (s, c) to have arrived (s >= 1),
        store their part of it into the right neighbour's slot (s + 1, c) and add
        one arrival there;
      * compute workers (the CTAs' producers): read each unit after all its
        parts arrived, chunks in order, a random subset of them (causal
        visibility decides which a rank needs);
      * the last CTA: after every worker finished, wait until every unit of the
        call arrived, re-arm the arrival counts to 0 and publish call + 1 to the
        left neighbour's credit word.
    Violations: a store into a slot whose previous contents the right neighbour
    may still read (it has not finished the call they belong to), or a read
    that finds another (owner, call) than expected.
    Mutations: "no_credit" (pushes skip the credit wait), "no_final_wait" (the
    last CTA re-arms the counts without waiting for late arrivals)."""

    def __init__(self, world: int, chunks: int = 2, workers: int = 2, calls: int = 3,
                 seed: int = 0, mutation: Optional[str] = None):
        self.P, self.C, self.W, self.calls = world, chunks, workers, calls
        self.rng = random.Random(seed)
        self.mutation = mutation
        P, C = world, chunks
        # slot[r][s][c] = (owner, call) of the last completed store; readers
        self.content = [[[None] * C for _ in range(P)] for _ in range(P)]
        self.readers = [[[0] * C for _ in range(P)] for _ in range(P)]
        self.arrivals = [[[0] * C for _ in range(P)] for _ in range(P)]
        self.credit = [0] * P
        self.finished = [0] * P          # calls each rank's kernel completed
        self.procs: List[Proc] = []
        self.waits: List[Optional[Wait]] = []

    def _spawn(self, proc: Proc) -> None:
        self.procs.append(proc)
        self.waits.append(None)
        try:
            self.waits[-1] = next(proc)
        except StopIteration:
            self.procs[-1] = None

    def _call(self, r: int, k: int) -> Proc:
        """Rank r's call k: launched once call k - 1 finished on this rank."""
        yield lambda: self.finished[r] >= k
        done = [0]
        n_workers = 2 * self.W
        for w in range(self.W):
            self._spawn(self._push(r, k, w, done))
            self._spawn(self._compute(r, k, done))
        yield lambda: done[0] == n_workers
        # last CTA
        P, C = self.P, self.C
        if self.mutation != "no_final_wait":
            yield lambda: all(self.arrivals[r][s][c] == self.W
                              for s in range(1, P) for c in range(C))
        for s in range(1, P):
            for c in range(C):
                self.arrivals[r][s][c] = 0
        self.credit[(r - 1) % P] = k + 1
        self.finished[r] = k + 1

    def _push(self, r: int, k: int, w: int, done: List[int]) -> Proc:
        P, C = self.P, self.C
        right = (r + 1) % P
        if self.mutation != "no_credit":
            yield lambda: self.credit[r] >= k
        for c in range(C):
            for s in range(P - 1):
                if s >= 1:
                    yield lambda s=s, c=c: self.arrivals[r][s][c] >= self.W
                    self._read(r, s, c, k)
                owner = (r - s) % P
                # the store: the right neighbour must be done with what it holds
                old = self.content[right][s + 1][c]
                stale = old is not None and old[1] != k and self.finished[right] <= old[1]
                if (self.readers[right][s + 1][c] and old is not None and old[1] != k) or stale:
                    raise ProtocolViolation(
                        f"rank {right} slot ({s + 1}, {c}): store of call {k} while call "
                        f"{old[1] if old else None} may still read it")
                yield lambda: True
                if w == 0:
                    self.content[right][s + 1][c] = (owner, k)
                self.arrivals[right][s + 1][c] += 1
                if s >= 1:
                    self.readers[r][s][c] -= 1
        done[0] += 1

    def _read(self, r: int, s: int, c: int, k: int) -> None:
        expect = ((r - s) % self.P, k)
        if self.content[r][s][c] != expect:
            raise ProtocolViolation(f"rank {r} slot ({s}, {c}): holds "
                                    f"{self.content[r][s][c]}, expected {expect}")
        self.readers[r][s][c] += 1

    def _compute(self, r: int, k: int, done: List[int]) -> Proc:
        for c in range(self.C):
            for s in range(1, self.P):
                if self.rng.random() < 0.3:
                    continue  # a unit nobody on this rank needs (causal visibility)
                yield lambda s=s, c=c: self.arrivals[r][s][c] >= self.W
                self._read(r, s, c, k)
                yield lambda: True
                self.readers[r][s][c] -= 1
        done[0] += 1

    def run(self, max_events: int = 500000) -> int:
        for r in range(self.P):
            self._spawn(_chain([self._call(r, k) for k in range(self.calls)]))
        events = 0
        while any(p is not None for p in self.procs):
            ready = [i for i, (p, w) in enumerate(zip(self.procs, self.waits))
                     if p is not None and w is not None and w()]
            if not ready:
                raise RuntimeError("deadlock: no activity can proceed")
            i = self.rng.choice(ready)
            try:
                self.waits[i] = next(self.procs[i])
            except StopIteration:
                self.waits[i] = None
                self.procs[i] = None
            events += 1
            if events > max_events:
                raise RuntimeError("event budget exhausted")
        return events


def one_launch_plan(world: int, rank: int, calls: int) -> List[List[int]]:
    """The one-launch engine's flag values as the model uses them: one row per
    call, [call, credit the pushes wait for, credit published at the end, tag of
    segment 0, ..., tag of segment world-1] with tag (owner + 1) | call << 8;
    RingEngineP.plan() must produce the same rows."""
    rows = []
    for k in range(calls):
        rows.append([k, k, k + 1] + [((rank - s) % world + 1) | (k << 8)
                                     for s in range(world)])
    return rows


def check_one_launch(world: int, chunks: int = 2, workers: int = 2, calls: int = 3,
                     seeds: int = 50, mutation: Optional[str] = None) -> None:
    """Runs `seeds` random interleavings of the one-launch ring; raises on the
    first violation."""
    for seed in range(seeds):
        OneLaunchModel(world, chunks, workers, calls, seed, mutation).run()
