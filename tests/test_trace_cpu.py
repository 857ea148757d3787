"""Per-CTA kernel timelines: summary and Chrome-trace conversion on a synthetic
trace ([steps, CTAs, 8] words: {sm << 32 | cta, start, kv_ready, epilogue,
push_start, push_end, end, key tiles}, nanoseconds)."""
import json

import torch

from multi_gpu_flashattention_b200.utils.trace import (summarize, to_chrome_events,
                                                       write_chrome_trace)


def _trace():
    t = torch.zeros(2, 3, 8, dtype=torch.int64)
    base = 1_000_000
    for c in range(3):
        # step 0: every CTA starts at base, kv ready after 1 us, 1 ms of work;
        # CTAs 0 and 1 push for 200 us, CTA 2 pushes nothing
        t[0, c] = torch.tensor([(c << 32) | c, base, base + 1_000, base + 900_000,
                                base + 2_000 if c < 2 else 0, base + 202_000 if c < 2 else 0,
                                base + 1_000_000, 4])
        # step 1: starts after step 0, CTA 1 waits 50 us for the shard
        s1 = base + 1_100_000
        t[1, c] = torch.tensor([(c << 32) | c, s1, s1 + (50_000 if c == 1 else 1_000),
                                s1 + 800_000, 0, 0, s1 + 900_000, 2])
    return t


def test_summary_fields():
    out = summarize(_trace())["steps"]
    assert [s["step"] for s in out] == [0, 1]
    s0, s1 = out
    assert abs(s0["span_ms"] - 1.0) < 1e-6
    assert s0["n_ctas"] == 3 and s0["n_pushing"] == 2
    assert abs(s0["mean_push_ms_pushing"] - 0.2) < 1e-6
    assert abs(s0["mean_push_ms"] - 0.4 / 3) < 1e-6
    assert abs(s0["push_done_ms"] - 0.202) < 1e-6
    assert abs(s0["mean_cta_ms_other"] - 1.0) < 1e-6
    assert abs(s1["max_kv_wait_ms"] - 0.05) < 1e-6
    assert s1["n_pushing"] == 0 and "mean_push_ms_pushing" not in s1
    assert abs(s1["mean_cta_ms"] - 0.9) < 1e-6


def test_chrome_events(tmp_path):
    ev = to_chrome_events(_trace(), rank=3)
    names = {e["name"] for e in ev}
    assert {"attn step 0", "attn step 1", "epilogue", "push", "wait kv"} <= names
    assert all(e["pid"] == 3 for e in ev)
    assert sum(e["name"] == "push" for e in ev) == 2
    assert min(e["ts"] for e in ev) == 0.0
    path = tmp_path / "t.json"
    write_chrome_trace(ev, str(path))
    assert len(json.load(open(path))["traceEvents"]) == len(ev)
