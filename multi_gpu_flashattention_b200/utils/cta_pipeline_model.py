"""Executable model of one CTA of the persistent attention forward
(csrc/kernels/attn_fwd_persistent.cu), for race checks of its on-chip pipeline.

Inside a CTA the warps hand tiles to each other only through mbarriers, and
two engines run asynchronously to the warps: the TMA unit (loads that complete
in any order, each signalling the barrier it was armed on) and the tensor core
(MMAs executed in issue order; `tcgen05.commit` arrives on a barrier once
every MMA issued before it has finished). This module restates the kernel's
roles as generators -- the scheduler/TMA producer warp, the MMA-issuing
thread, the eight softmax warps (two query tiles x four 32-lane groups of
TMEM) -- plus the two engines, and lets a seeded random scheduler interleave
them. Every buffer carries a tag naming the tile it holds, and the checker
fails when

  * an MMA reads a Q, K or V buffer, or a P lane group, that does not hold the
    tile it was issued for (a TMA load or a softmax store overwrote it early,
    or has not landed),
  * a softmax warp loads S lanes that do not hold its tile's scores,
  * an epilogue reads an O accumulator that is missing a PV of its item, holds
    one of another item, or is rescaled while a PV into it is in flight,
  * a role waits forever (deadlock: no role can move).

mbarrier semantics follow PTX: a barrier completes its current phase when the
pending arrival count and the transaction count both reach zero; a wait on
parity p succeeds once the phase with parity p has completed (a fresh barrier
satisfies a wait on parity 1). The model covers the default softmax hand-over
(P of a key tile released in one piece) and the split one (`split=True`, two
64-key halves), any number of items per CTA with 0-6 key tiles each, and
rescales of O in TMEM between PV steps (`rescale_every`).

Mutations (`mutation=`) that drop one ordering rule must be caught:
  "no_k_empty"     the producer refills a K stage without waiting for k_empty
  "s_before_pv"    the MMA thread issues S_t(j+1) before PV_t(j)
  "early_o_empty"  a softmax warp frees O before it has read it
  "p_count_3"      p_full expects three softmax warps instead of four
  "no_q_empty"     the producer loads the next item's Q without waiting for q_empty
  "t0_no_o_empty"  an item without visible key tiles commits o_full without
                   waiting for o_empty (the kernel before this model found it:
                   the MMA thread then runs a phase ahead of a slow epilogue,
                   whose parity wait aliases -- a deadlock, or the next item's
                   first PV overwriting O while it is still being read)
"""
from __future__ import annotations

import random
from dataclasses import dataclass
from typing import Dict, Generator, List, Optional, Tuple


class PipelineViolation(AssertionError):
    pass


@dataclass
class MBarrier:
    name: str
    count: int
    completed: int = 0     # phases completed so far
    pending: int = 0       # arrivals still missing in the current phase
    tx: int = 0            # transaction bytes still expected

    def __post_init__(self):
        self.pending = self.count

    def _maybe_complete(self):
        if self.pending == 0 and self.tx == 0:
            self.completed += 1
            self.pending = self.count

    def arrive(self, n: int = 1):
        if self.pending < n:
            raise PipelineViolation(f"{self.name}: {n} arrivals with {self.pending} pending")
        self.pending -= n
        self._maybe_complete()

    def arrive_expect_tx(self, nbytes: int):
        self.tx += nbytes
        self.arrive()

    def complete_tx(self, nbytes: int):
        self.tx -= nbytes
        self._maybe_complete()

    def ready(self, parity: int) -> bool:
        # current (incomplete) phase index = completed; its parity = completed & 1
        return (self.completed & 1) != parity


Tag = Tuple


class CtaModel:
    """One CTA processing `items` (a list of key-tile counts, one per work item)."""

    TILE_BYTES = 1

    def __init__(self, items: List[int], seed: int, split: bool = False,
                 rescale_every: int = 0, mutation: Optional[str] = None):
        self.items = list(items)
        self.rng = random.Random(seed)
        self.split = split
        self.rescale_every = rescale_every
        self.mut = mutation
        b = MBarrier
        self.bar: Dict[str, MBarrier] = {}
        for name, count in [("q_full", 1), ("q_empty", 1), ("drain", 1)]:
            self.bar[name] = b(name, count)
        for i in range(2):
            for name in ("k_full", "k_empty", "v_full", "v_empty", "s_full", "o_full",
                         "sched_full"):
                self.bar[f"{name}{i}"] = b(f"{name}{i}", 1)
            self.bar[f"o_empty{i}"] = b(f"o_empty{i}", 4)
            self.bar[f"sched_empty{i}"] = b(f"sched_empty{i}", 9)
            for h in range(2):
                self.bar[f"p_full{i}{h}"] = b(f"p_full{i}{h}", 3 if mutation == "p_count_3" else 4)
        # buffers: smem q[2], k[2], v[2]; TMEM S/P of tile t per lane group and
        # key half; O of tile t as (item, set of key tiles, in-flight PV count)
        self.q: List[Optional[Tag]] = [None, None]
        self.k: List[Optional[Tag]] = [None, None]
        self.v: List[Optional[Tag]] = [None, None]
        self.sp: Dict[Tuple[int, int, int], Optional[Tag]] = {
            (t, lg, h): None for t in range(2) for lg in range(4) for h in range(2)}
        self.o: List[Tuple[Optional[int], frozenset]] = [(None, frozenset()), (None, frozenset())]
        self.sched_item: List[Optional[int]] = [None, None]
        self.tma: List[Tuple[str, int, Tag, str]] = []   # pending loads (buf, idx, tag, barrier)
        self.pipe: List[tuple] = []                       # tensor-core FIFO
        self.done_items: List[int] = []
        self.waiting: Dict[str, Tuple[str, int]] = {}
        self._cur = ""

    # ---------------------------------------------------------------- engines
    def _tma_step(self):
        i = self.rng.randrange(len(self.tma))
        buf, idx, tag, barname = self.tma.pop(i)
        getattr(self, buf)[idx] = tag
        self.bar[barname].complete_tx(self.TILE_BYTES)

    def _pipe_step(self):
        op = self.pipe.pop(0)
        kind = op[0]
        if kind == "commit":
            self.bar[op[1]].arrive()
        elif kind == "S":
            _, t, item, g, st, h = op
            if self.q[t] != ("Q", item, t):
                raise PipelineViolation(f"S{t}({item},{g}) read Q buffer {self.q[t]}")
            if self.k[st] != ("K", item, g):
                raise PipelineViolation(f"S{t}({item},{g}) read K stage {st} = {self.k[st]}")
            for lg in range(4):
                for hh in range(2):
                    self.sp[(t, lg, hh)] = ("S", item, t, g)
        elif kind == "PV":
            _, t, item, g, st, h, first = op
            if self.v[st] != ("V", item, g):
                raise PipelineViolation(f"PV{t}({item},{g}) read V stage {st} = {self.v[st]}")
            for lg in range(4):
                if self.sp[(t, lg, h)] != ("P", item, t, g):
                    raise PipelineViolation(
                        f"PV{t}({item},{g}) half {h} read P lanes {lg} = {self.sp[(t, lg, h)]}")
            o_item, tiles = self.o[t]
            if first:
                self.o[t] = (item, frozenset({(g, h)}))
            else:
                if o_item != item:
                    raise PipelineViolation(f"PV{t}({item},{g}) accumulated into O of {o_item}")
                self.o[t] = (item, tiles | {(g, h)})
        else:
            raise AssertionError(kind)

    # ---------------------------------------------------------------- roles
    def _wait(self, name: str, parity: int):
        while not self.bar[name].ready(parity):
            self.waiting[self._cur] = (name, parity)
            yield False
        self.waiting.pop(self._cur, None)
        yield True

    def producer(self) -> Generator[bool, None, None]:
        it = 0
        n = 0
        queue = list(range(len(self.items)))
        while True:
            item = queue.pop(0) if queue else None
            slot = n & 1
            yield from self._wait(f"sched_empty{slot}", ((n >> 1) & 1) ^ 1)
            self.sched_item[slot] = item
            self.bar[f"sched_full{slot}"].arrive()
            yield True
            if item is None:
                break
            if self.mut != "no_q_empty":
                yield from self._wait("q_empty", (n & 1) ^ 1)
            self.bar["q_full"].arrive_expect_tx(2 * self.TILE_BYTES)
            for t in range(2):
                self.tma.append(("q", t, ("Q", item, t), "q_full"))
            yield True
            for g in range(self.items[item]):
                st, ph = it & 1, (it >> 1) & 1
                if self.mut != "no_k_empty":
                    yield from self._wait(f"k_empty{st}", ph ^ 1)
                self.bar[f"k_full{st}"].arrive_expect_tx(self.TILE_BYTES)
                self.tma.append(("k", st, ("K", item, g), f"k_full{st}"))
                yield True
                yield from self._wait(f"v_empty{st}", ph ^ 1)
                self.bar[f"v_full{st}"].arrive_expect_tx(self.TILE_BYTES)
                self.tma.append(("v", st, ("V", item, g), f"v_full{st}"))
                yield True
                it += 1
            n += 1

    def mma(self) -> Generator[bool, None, None]:
        it = 0
        n = 0
        P = self.pipe
        while True:
            slot = n & 1
            yield from self._wait(f"sched_full{slot}", (n >> 1) & 1)
            item = self.sched_item[slot]
            self.bar[f"sched_empty{slot}"].arrive()
            yield True
            if item is None:
                break
            T = self.items[item]
            yield from self._wait("q_full", n & 1)
            if T == 0:
                # an item with no visible key tile still takes one phase of each
                # O hand-over, so the epilogues' parity waits stay aligned
                P.append(("commit", "q_empty"))
                if self.mut != "t0_no_o_empty":
                    for t in range(2):
                        yield from self._wait(f"o_empty{t}", (n & 1) ^ 1)
                P += [("commit", "o_full0"), ("commit", "o_full1")]
                yield True
                n += 1
                continue
            st = it & 1
            yield from self._wait(f"k_full{st}", (it >> 1) & 1)
            P += [("S", 0, item, 0, st, 0), ("commit", "s_full0"),
                  ("S", 1, item, 0, st, 0), ("commit", "s_full1"), ("commit", f"k_empty{st}")]
            if T == 1:
                P.append(("commit", "q_empty"))
            yield True
            for j in range(T):
                g = it + j
                st, ph, pp = g & 1, (g >> 1) & 1, g & 1
                st1, ph1 = (g + 1) & 1, ((g + 1) >> 1) & 1
                more = j + 1 < T
                yield from self._wait(f"v_full{st}", ph)
                for t in range(2):
                    if j == 0:
                        yield from self._wait(f"o_empty{t}", (n & 1) ^ 1)
                    if self.mut == "s_before_pv" and more:
                        yield from self._wait(f"k_full{st1}", ph1)
                        P += [("S", t, item, j + 1, st1, 0), ("commit", f"s_full{t}")]
                    for h in range(2):
                        yield from self._wait(f"p_full{t}{h}", pp)
                        P.append(("PV", t, item, j, st, h, j == 0 and h == 0))
                        yield True
                    if t == 1:
                        P.append(("commit", f"v_empty{st}"))
                    if not more:
                        P.append(("commit", f"o_full{t}"))
                    elif self.mut != "s_before_pv":
                        if t == 0:
                            yield from self._wait(f"k_full{st1}", ph1)
                        P += [("S", t, item, j + 1, st1, 0), ("commit", f"s_full{t}")]
                    if more and t == 1:
                        P.append(("commit", f"k_empty{st1}"))
                        if j + 2 == T:
                            P.append(("commit", "q_empty"))
                    yield True
            it += T
            n += 1
        P.append(("commit", "drain"))
        yield from self._wait("drain", 0)

    def softmax(self, w: int) -> Generator[bool, None, None]:
        t, lg = w >> 2, w & 3
        g_all = 0
        n = 0
        while True:
            slot = n & 1
            yield from self._wait(f"sched_full{slot}", (n >> 1) & 1)
            item = self.sched_item[slot]
            self.bar[f"sched_empty{slot}"].arrive()
            yield True
            if item is None:
                break
            T = self.items[item]
            for j in range(T):
                yield from self._wait(f"s_full{t}", g_all & 1)
                for h in range(2):
                    if self.sp[(t, lg, h)] != ("S", item, t, j):
                        raise PipelineViolation(
                            f"softmax warp {w} loaded S lanes {self.sp[(t, lg, h)]} for "
                            f"({item},{j})")
                yield True
                rescale = self.rescale_every and j > 0 and j % self.rescale_every == 0
                for h in range(2):
                    if h == 0 and rescale:
                        # O is rescaled in TMEM before P goes out: every PV issued
                        # so far into O must have finished (they were issued before
                        # the S commit this warp waited for, except in a mutation)
                        for op in self.pipe:
                            if op[0] == "PV" and op[1] == t:
                                raise PipelineViolation(
                                    f"softmax warp {w} rescaled O{t} with PV {op[2:4]} in flight")
                    self.sp[(t, lg, h)] = ("P", item, t, j)
                    if self.split:
                        if self._arrives(w):
                            self.bar[f"p_full{t}{h}"].arrive()
                        yield True
                if not self.split:
                    if self._arrives(w):
                        self.bar[f"p_full{t}0"].arrive()
                        self.bar[f"p_full{t}1"].arrive()
                    yield True
                g_all += 1
            # epilogue
            if self.mut == "early_o_empty":
                self.bar[f"o_empty{t}"].arrive()
                yield True
            yield from self._wait(f"o_full{t}", n & 1)
            o_item, tiles = self.o[t]
            want = frozenset((j, h) for j in range(T) for h in range(2))
            if T > 0 and (o_item != item or tiles != want):
                raise PipelineViolation(
                    f"epilogue warp {w} of item {item} read O{t} = ({o_item}, {sorted(tiles)})")
            if self.mut != "early_o_empty":
                self.bar[f"o_empty{t}"].arrive()
            yield True
            if t == 0 and lg == 0:
                self.done_items.append(item)
            n += 1

    def _arrives(self, w: int) -> bool:
        # with the "p_count_3" mutation the barrier expects three arrivals, so the
        # fourth warp of a tile must not arrive (it would overflow the phase)
        return not (self.mut == "p_count_3" and (w & 3) == 3)

    # ---------------------------------------------------------------- run
    def run(self, max_steps: int = 400000) -> None:
        live = {"producer": self.producer(), "mma": self.mma()}
        for w in range(8):
            live[f"softmax{w}"] = self.softmax(w)
        for _ in range(max_steps):
            if not live and not self.tma and not self.pipe:
                break
            engines = (["TMA"] if self.tma else []) + (["tensor"] if self.pipe else [])
            pick = self.rng.choice(list(live) + engines)
            if pick == "TMA":
                self._tma_step()
            elif pick == "tensor":
                self._pipe_step()
            elif not self._step(live, pick) and not self.tma and not self.pipe:
                # nothing in flight: if no role can move now, none ever will
                if (not any(self._step(live, r) for r in self.rng.sample(list(live), len(live)))
                        and not self.tma and not self.pipe):
                    waits = {r: (w, self.bar[w[0]].completed) for r, w in self.waiting.items()}
                    raise PipelineViolation(f"deadlock: roles waiting on (barrier, parity), "
                                            f"completed phases: {waits}")
        else:
            raise PipelineViolation("step limit reached")
        want = list(range(len(self.items)))
        if sorted(self.done_items) != want:
            raise PipelineViolation(f"items finished {sorted(self.done_items)}, want {want}")

    def _step(self, live, role) -> bool:
        """Advance `role` by one action; True if it did something."""
        if role not in live:
            return False
        self._cur = role
        try:
            return next(live[role])
        except StopIteration:
            del live[role]
            return True


def check(items: List[int], seed: int, **kw) -> None:
    CtaModel(items, seed, **kw).run()
