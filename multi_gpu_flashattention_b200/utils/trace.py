"""Kernel timelines of the ring engines as Chrome trace events.

Per-step engine (backend "fused_stepwise"): enable with
`ENGINES.get(...).set_trace(True)`, run a forward, then `engine.last_trace()`
holds [steps, CTAs, 8] int64 words
per call: {sm << 32 | cta, start, kv_ready, epilogue, push_start, push_end,
end, visible key tiles} in %globaltimer nanoseconds. `to_chrome_events` turns
them into complete ("X") events -- one process per rank, one thread per SM --
for chrome://tracing or Perfetto.

One-launch engine (backend "fused"): `P_ENGINES.get(...).set_trace(True)`
gives [grid, 8] words per call; see summarize_one_launch and
one_launch_chrome_events."""
from __future__ import annotations

import json
from typing import Iterable, List, Optional

import torch


def to_chrome_events(trace: torch.Tensor, rank: int = 0, t0_ns: Optional[int] = None) -> List[dict]:
    t = trace.detach().cpu().to(torch.int64)
    valid = t[..., 6] != 0
    if t0_ns is None:
        t0_ns = int(t[..., 1][valid].min().item()) if valid.any() else 0
    ev = []
    steps, ctas, _ = t.shape
    for s in range(steps):
        for c in range(ctas):
            w = t[s, c].tolist()
            if w[6] == 0:
                continue
            sm = w[0] >> 32
            us = lambda x: (x - t0_ns) / 1e3
            args = {"step": s, "cta": w[0] & 0xFFFFFFFF, "key_tiles": w[7]}
            kv = w[2] or w[1]
            if kv > w[1]:
                ev.append({"name": "wait kv", "ph": "X", "pid": rank, "tid": sm, "ts": us(w[1]),
                           "dur": (kv - w[1]) / 1e3, "args": args})
            end_c = w[3] or w[6]
            ev.append({"name": f"attn step {s}", "ph": "X", "pid": rank, "tid": sm, "ts": us(kv),
                       "dur": max(0, end_c - kv) / 1e3, "args": args})
            ev.append({"name": "epilogue", "ph": "X", "pid": rank, "tid": sm, "ts": us(end_c),
                       "dur": max(0, w[6] - end_c) / 1e3, "args": args})
            if w[4] and w[5]:
                ev.append({"name": "push", "ph": "X", "pid": rank, "tid": 1000 + sm,
                           "ts": us(w[4]), "dur": (w[5] - w[4]) / 1e3, "args": args})
    return ev


def write_chrome_trace(events: Iterable[dict], path: str) -> None:
    with open(path, "w") as f:
        json.dump({"traceEvents": list(events), "displayTimeUnit": "ns"}, f)


def summarize(trace: torch.Tensor) -> dict:
    """Per step (ms): wall span, longest wait for the KV shard, push time (mean over
    all CTAs and over the pushing CTAs), CTA duration (all, pushing, other) and
    when the last chunk was pushed."""
    t = trace.detach().cpu().to(torch.int64)
    out = []
    for s in range(t.shape[0]):
        w = t[s]
        ok = w[:, 6] != 0
        if not ok.any():
            continue
        w = w[ok]
        span = (w[:, 6].max() - w[:, 1].min()).item() / 1e6
        kv_wait = ((w[:, 2] - w[:, 1]).clamp(min=0) * (w[:, 2] != 0)).max().item() / 1e6
        push = ((w[:, 5] - w[:, 4]) * (w[:, 4] != 0)).float().mean().item() / 1e6
        pushing = w[:, 4] != 0
        cta = (w[:, 6] - w[:, 1]).float()
        entry = {"step": s, "span_ms": span, "max_kv_wait_ms": kv_wait, "mean_push_ms": push,
                 "mean_cta_ms": cta.mean().item() / 1e6, "n_ctas": int(w.shape[0]),
                 "n_pushing": int(pushing.sum().item())}
        if pushing.any():
            pw = w[pushing]
            entry["mean_push_ms_pushing"] = (pw[:, 5] - pw[:, 4]).float().mean().item() / 1e6
            entry["mean_cta_ms_pushing"] = cta[pushing].mean().item() / 1e6
            entry["mean_cta_ms_other"] = (cta[~pushing].mean().item() / 1e6
                                          if (~pushing).any() else None)
            # when the last chunk of the shard was pushed, relative to the step start
            entry["push_done_ms"] = (pw[:, 5].max() - w[:, 1].min()).item() / 1e6
        out.append(entry)
    return {"steps": out}


def summarize_one_launch(trace: torch.Tensor) -> dict:
    """Summary of a one-launch ring call's per-CTA trace ([grid, 8] int64:
    {sm << 32 | cta, start, end, items, ns waiting for arrivals, -, push start,
    push end}), in ms: kernel span, CTA busy time (mean / min / max), how long
    CTAs waited for received shards (mean / max), and the push window (first
    start to last end, mean per push warp)."""
    t = trace.detach().cpu().to(torch.int64)
    ok = t[:, 1] != 0
    t = t[ok]
    if t.shape[0] == 0:
        return {}
    t0 = int(t[:, 1].min())
    busy = (t[:, 2] - t[:, 1]).double() / 1e6
    wait = t[:, 4].double() / 1e6
    out = {"span_ms": (int(t[:, 2].max()) - t0) / 1e6, "n_ctas": int(t.shape[0]),
           "items": int(t[:, 3].sum()), "cta_ms_mean": busy.mean().item(),
           "cta_ms_min": busy.min().item(), "cta_ms_max": busy.max().item(),
           "arrival_wait_ms_mean": wait.mean().item(), "arrival_wait_ms_max": wait.max().item()}
    pushed = t[:, 6] != 0
    if pushed.any():
        p = t[pushed]
        out["push_start_ms"] = (int(p[:, 6].min()) - t0) / 1e6
        out["push_end_ms"] = (int(p[:, 7].max()) - t0) / 1e6
        out["push_ms_mean"] = ((p[:, 7] - p[:, 6]).double() / 1e6).mean().item()
    return out


def one_launch_chrome_events(trace: torch.Tensor, rank: int = 0) -> List[dict]:
    """Chrome trace events of a one-launch ring call: per CTA its busy span and
    the push window of its push warps."""
    t = trace.detach().cpu().to(torch.int64)
    ok = t[:, 1] != 0
    if not ok.any():
        return []
    t0 = int(t[ok, 1].min())
    ev = []
    for w in t[ok].tolist():
        sm = w[0] >> 32
        args = {"cta": w[0] & 0xFFFFFFFF, "items": w[3], "arrival_wait_us": w[4] / 1e3}
        ev.append({"name": "attention", "ph": "X", "pid": rank, "tid": sm,
                   "ts": (w[1] - t0) / 1e3, "dur": (w[2] - w[1]) / 1e3, "args": args})
        if w[6] and w[7]:
            ev.append({"name": "push", "ph": "X", "pid": rank, "tid": 1000 + sm,
                       "ts": (w[6] - t0) / 1e3, "dur": (w[7] - w[6]) / 1e3, "args": args})
    return ev
