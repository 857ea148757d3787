"""Causal load balance of the ring layouts (host only, no GPU).

    python -m multi_gpu_flashattention_b200.benchmarks.layout_balance \
        [--seq 131072] [--world 8] [--mask causal|full] [--block 128] [--json]

For each layout -- contiguous (the reference's), zigzag, striped, and the
scheduler-driven ones (contiguous-DP and row-LPT partitions of the workload
model) -- prints every rank's visible (query, key) pairs over the whole ring,
the max/mean imbalance across ranks, and the slowest ring step's imbalance
(the ring advances at the pace of its slowest rank at every step)."""
from __future__ import annotations

import argparse
import json

from ..parallel.layouts import RingLayout

LAYOUTS = [("contiguous", {}), ("zigzag", {}), ("striped", {}),
           ("scheduler", {"policy": "dp"}), ("scheduler", {"policy": "lpt"})]


def balance(kind: str, seq: int, world: int, mask: str, block: int, **kw) -> dict:
    lay = RingLayout(kind, seq, world, block=block, mask=mask, **kw)
    # work[t][r]: pairs rank r computes at ring step t (on the shard of owner r - t)
    work = [[lay.step_work(r, lay.compute_owner(r, t)) for r in range(world)]
            for t in range(world)]
    totals = [sum(work[t][r] for t in range(world)) for r in range(world)]
    mean = sum(totals) / world
    # per step the slowest rank sets the pace: sum over steps of the max
    paced = sum(max(step) for step in work)
    return {"layout": kind + (f"-{kw['policy']}" if kw.get("policy") else ""),
            "per_rank_pairs": totals,
            "imbalance": max(totals) / mean if mean else 1.0,
            "ring_paced_imbalance": paced / mean if mean else 1.0}


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--seq", type=int, default=131072)
    ap.add_argument("--world", type=int, default=8)
    ap.add_argument("--mask", default="causal", choices=["causal", "full"])
    ap.add_argument("--block", type=int, default=128)
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args(argv)
    rows = []
    for kind, kw in LAYOUTS:
        try:
            rows.append(balance(kind, a.seq, a.world, a.mask, a.block, **kw))
        except ValueError as e:  # e.g. zigzag needs seq % (2 * world) == 0
            rows.append({"layout": kind, "error": str(e)})
    if a.json:
        print(json.dumps({"seq": a.seq, "world": a.world, "mask": a.mask, "layouts": rows}))
        return 0
    print(f"seq={a.seq} world={a.world} mask={a.mask}")
    print(f"{'layout':>16} {'max/mean':>9} {'ring-paced':>11}  per-rank pairs (millions)")
    for row in rows:
        if "error" in row:
            print(f"{row['layout']:>16}  {row['error']}")
            continue
        pairs = " ".join(f"{p / 1e6:.1f}" for p in row["per_rank_pairs"])
        print(f"{row['layout']:>16} {row['imbalance']:>9.3f} {row['ring_paced_imbalance']:>11.3f}"
              f"  {pairs}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
