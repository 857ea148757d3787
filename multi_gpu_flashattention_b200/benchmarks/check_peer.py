"""Peer-access and interconnect report (the reference's ring/check_peer.cu).

    python -m multi_gpu_flashattention_b200.benchmarks.check_peer [--json]

Prints the cudaDeviceCanAccessPeer matrix like the reference and, when NVML
is available, the NVLink state of each GPU (active links and their peers)."""
from __future__ import annotations

import argparse
import json

import torch


def peer_matrix():
    n = torch.cuda.device_count()
    return [[(i == j) or bool(torch.cuda.can_device_access_peer(i, j)) for j in range(n)]
            for i in range(n)]


def nvlink_report():
    try:
        import pynvml
    except Exception:
        return None
    try:
        pynvml.nvmlInit()
    except Exception:
        return None
    out = []
    try:
        for i in range(pynvml.nvmlDeviceGetCount()):
            h = pynvml.nvmlDeviceGetHandleByIndex(i)
            links = 0
            for l in range(18):
                try:
                    if pynvml.nvmlDeviceGetNvLinkState(h, l) == pynvml.NVML_FEATURE_ENABLED:
                        links += 1
                except Exception:
                    break
            out.append({"gpu": i, "name": pynvml.nvmlDeviceGetName(h), "active_nvlinks": links})
    finally:
        pynvml.nvmlShutdown()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--json", action="store_true")
    a = ap.parse_args()
    m = peer_matrix()
    n = len(m)
    for i in range(n):
        for j in range(n):
            if i != j:  # the reference's line format
                print(f"GPU {i} -> GPU {j}: {'YES' if m[i][j] else 'NO'}")
    nv = nvlink_report()
    if nv:
        for g in nv:
            print(f"GPU {g['gpu']} ({g['name']}): {g['active_nvlinks']} active NVLink(s)")
    if a.json:
        print(json.dumps({"peer": m, "nvlink": nv}))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
