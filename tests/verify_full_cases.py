"""Deterministic dump sets for the verify_full parity test (shared by the test
and by the script that records the golden reports)."""
import os

import numpy as np

CASES = {
    # name: (num_gpus, tokens per rank, edit)
    "pass2": (2, 1024, None),
    "pass3": (3, 512, None),
    "perturbed": (2, 1024, ("add", 1, 777, 2.0)),
    "nan_inf": (2, 1024, ("nan_inf", 0, 5, None)),
    "missing": (2, 1024, ("missing", 1, 0, None)),
    "short": (2, 1024, ("short", 1, 0, None)),
}


def _legacy(rank, n, dim=64):
    i = np.arange(n, dtype=np.int64)
    kv = np.float32(rank * 1000.0) + i.astype(np.float32)
    q = (np.float32(rank * 500.0) + (i % dim).astype(np.float32) * np.float32(0.01)) \
        * np.float32(0.001)
    return q.astype(np.float32), kv.astype(np.float32)


def write_case(name, out_dir):
    """Writes ring_output_rank<r>.bin files for case `name`; returns
    (num_gpus, kv_size_bytes)."""
    P, L, edit = CASES[name]
    dim = 64
    kv = np.concatenate([_legacy(r, L * dim)[1] for r in range(P)]).reshape(P * L, dim)
    kv64 = kv.astype(np.float64)
    os.makedirs(out_dir, exist_ok=True)
    for r in range(P):
        q = _legacy(r, L * dim)[0].reshape(L, dim).astype(np.float64)
        s = q @ kv64.T
        s -= s.max(axis=1, keepdims=True)
        p = np.exp(s)
        out = ((p @ kv64) / p.sum(axis=1, keepdims=True)).astype(np.float32).reshape(-1)
        path = os.path.join(out_dir, f"ring_output_rank{r}.bin")
        if edit and edit[1] == r:
            kind, _, idx, val = edit
            if kind == "missing":
                continue
            if kind == "add":
                out[idx] += np.float32(val)
            elif kind == "nan_inf":
                out[idx] = np.nan
                out[idx + 1] = np.inf
            elif kind == "short":
                out = out[: out.size // 2]
        out.astype("<f4").tofile(path)
    return P, L * dim * 4
