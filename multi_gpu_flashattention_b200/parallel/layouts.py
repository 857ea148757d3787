"""Token-shard layouts for ring attention (backed by the C++ shard plans).

A layout says which global token positions each rank holds, in local order.
Queries and keys use the same layout. The kernels only need, per 128-token
local tile, the global position of its first token ("tile positions"), because
every layout here keeps the tokens of a tile consecutive:

  contiguous  rank r holds [r*n, (r+1)*n)       (reference layout,
              ring/attention/common/shard_utils.cuh:15-27)
  zigzag      2P chunks; rank r holds chunks r and 2P-1-r (causal balance)
  striped     token t on rank t % P; tiles are expressed in local-index
              coordinates with a diagonal offset of 0 (owner <= rank) or 1
  scheduler   block rows chosen by the workload schedulers (row LPT by
              default, or contiguous DP); shards may differ in length and are
              padded to the longest one

The scheduler layout defaults to the row-LPT partition
(workload/scheduler.c:254-281 in the reference): it interleaves block rows, so
every ring step carries about the same causal work on every rank. The
contiguous-DP partition (workload/scheduler.c:284-356) minimises each rank's
total work, the workload model's makespan, but a ring synchronises at every
step and the DP ranks' very different row ranges leave one rank with most of
the work at most steps (step-paced imbalance 4.667 at 128K on 8 ranks against
1.000 for row LPT); `policy="dp"` keeps it selectable as the model's answer for
unsynchronised work.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import torch

from .._ext import sched as _sched

TILE = 128
LAYOUTS = ("contiguous", "zigzag", "striped", "scheduler")


@dataclass
class RingLayout:
    kind: str
    seq: int
    world: int
    block: int = TILE
    mask: str = "causal"
    policy: str = "lpt"
    _plan: object = field(default=None, repr=False)

    def __post_init__(self):
        S = _sched()
        if self.kind == "contiguous":
            self._plan = S.make_contiguous(self.seq, self.world)
        elif self.kind == "zigzag":
            self._plan = S.make_zigzag(self.seq, self.world)
        elif self.kind == "striped":
            self._plan = S.make_striped(self.seq, self.world)
        elif self.kind == "scheduler":
            self._plan = S.make_scheduled(self.seq, self.world, self.block, self.mask, self.policy)
        else:
            raise ValueError(f"layout must be one of {LAYOUTS}, got {self.kind!r}")

    # ------------------------------------------------------------------ queries
    @property
    def plan(self):
        return self._plan

    def local_len(self, rank: int) -> int:
        return int(self._plan.local_len(rank))

    @property
    def max_local_len(self) -> int:
        return int(self._plan.max_local_len())

    def positions(self, rank: int) -> torch.Tensor:
        """Global positions of rank's tokens, in local order (int64)."""
        return torch.tensor(self._plan.positions(rank), dtype=torch.int64)

    def describe(self, rank: int) -> str:
        return self._plan.describe(rank)

    def compute_owner(self, rank: int, step: int) -> int:
        return int(self._plan.compute_owner(rank, step))

    def receive_owner(self, rank: int, step: int) -> int:
        return int(self._plan.receive_owner(rank, step))

    # ------------------------------------------------------------------ tensors
    def shard(self, x: torch.Tensor, rank: int, dim: int = 1) -> torch.Tensor:
        """Rank's local shard of a global tensor, padded with zeros to max_local_len."""
        idx = self.positions(rank).to(x.device)
        out = x.index_select(dim, idx)
        pad = self.max_local_len - out.shape[dim]
        if pad:
            shape = list(out.shape)
            shape[dim] = pad
            out = torch.cat([out, out.new_zeros(shape)], dim=dim)
        return out.contiguous()

    def unshard(self, shards: List[torch.Tensor], dim: int = 1) -> torch.Tensor:
        """Global tensor from every rank's (padded) local shard."""
        ref = shards[0]
        shape = list(ref.shape)
        shape[dim] = self.seq
        out = ref.new_empty(shape)
        for r, s in enumerate(shards):
            n = self.local_len(r)
            idx = self.positions(r).to(s.device)
            out.index_copy_(dim, idx.to(out.device), s.narrow(dim, 0, n).to(out.device))
        return out

    # ------------------------------------------------------------------ kernel metadata
    def _tile_starts(self, rank: int) -> List[int]:
        if self.kind == "striped":
            n = (self.max_local_len + TILE - 1) // TILE
            return [t * TILE for t in range(n)]
        starts = list(self._plan.tile_starts(rank, TILE))
        n_tiles = (self.max_local_len + TILE - 1) // TILE
        if any(s < 0 for s in starts):
            raise ValueError(f"{self.kind} layout: rank {rank} has a 128-token tile whose tokens "
                             "are not consecutive; use chunk sizes that are multiples of 128")
        # padding tiles (shorter shards) never see or are seen by anything real
        far = 1 << 30
        return starts + [far] * (n_tiles - len(starts))

    @staticmethod
    def _check_monotone(starts: List[int], what: str) -> List[int]:
        # the kernels find visible key tiles by prefix search over these tables
        if any(b < a for a, b in zip(starts, starts[1:])):
            raise ValueError(f"{what}: tile positions must be non-decreasing, got {starts[:8]}...")
        return starts

    def q_tile_pos(self, rank: int, device) -> torch.Tensor:
        return torch.tensor(self._check_monotone(self._tile_starts(rank), f"rank {rank}"),
                            dtype=torch.int32, device=device)

    def kv_tile_pos(self, rank: int, owner: int, device) -> torch.Tensor:
        """Tile positions of owner's shard as seen by rank's queries."""
        if self.kind == "striped":
            n = (self.max_local_len + TILE - 1) // TILE
            off = 1 if owner > rank else 0
            return torch.arange(n, dtype=torch.int32, device=device) * TILE + off
        return torch.tensor(self._check_monotone(self._tile_starts(owner), f"owner {owner}"),
                            dtype=torch.int32, device=device)

    def kv_tile_pos_by_owner(self, rank: int, device) -> torch.Tensor:
        return torch.stack([self.kv_tile_pos(rank, o, device) for o in range(self.world)])

    def kv_lens(self) -> List[int]:
        return [self.local_len(o) for o in range(self.world)]

    def q_positions_for_mask(self, rank: int) -> torch.Tensor:
        """Per-token positions in the coordinates the masks use (fp32 kernels, oracle)."""
        if self.kind == "striped":
            return torch.arange(self.max_local_len, dtype=torch.int64)
        pos = self.positions(rank)
        pad = self.max_local_len - pos.numel()
        return torch.cat([pos, torch.full((pad,), 1 << 40, dtype=torch.int64)]) if pad else pos

    def k_positions_for_mask(self, rank: int, owner: int) -> torch.Tensor:
        if self.kind == "striped":
            return torch.arange(self.max_local_len, dtype=torch.int64) + (1 if owner > rank else 0)
        pos = self.positions(owner)
        pad = self.max_local_len - pos.numel()
        return torch.cat([pos, torch.full((pad,), 1 << 41, dtype=torch.int64)]) if pad else pos

    def step_work(self, rank: int, owner: int, mask: Optional[str] = None) -> int:
        """Visible (query, key) pairs of one ring step."""
        return int(_sched().step_active(self._plan, rank, owner, mask or self.mask))


def make_layout(kind: str, seq: int, world: int, causal: bool = True, **kw) -> RingLayout:
    return RingLayout(kind=kind, seq=seq, world=world, mask="causal" if causal else "full", **kw)
