"""Single-GPU attention captured into CUDA graphs, for fixed shapes.

A call of `flash_attn_fwd` costs host work before its one kernel launch
(output allocations, default tile tables, tensor-map encoding, argument
checks); at a few thousand tokens that host path is longer than the kernel.
`GraphedAttention` runs the forward (and optionally the backward) once to warm
every cache, then captures it into a CUDA graph over static input and output
buffers; each call copies the new inputs in and replays the graph.

The ring engines are not captured: every ring call carries per-call flag
targets and owner tags computed on the host (use counters of the receive slots),
which a replayed graph would repeat unchanged.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .flash import flash_attn_bwd, flash_attn_fwd


class GraphedAttention:
    """Forward (and backward, with `backward=True`) of attention over fixed
    shapes, replayed from CUDA graphs.

    q [B,Sq,Hq,D], k/v [B,Sk,Hkv,D] give the shapes and dtype (their values are
    copied in as the first inputs). `forward(q, k, v)` returns (out, lse) in the
    graph's static buffers (overwritten by the next call; clone to keep them);
    `backward(dout)` returns fp32 (dq, dk, dv) of the last forward."""

    def __init__(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                 softmax_scale: Optional[float] = None, backward: bool = False,
                 warmup: int = 2):
        self.causal, self.scale = causal, softmax_scale
        self.q, self.k, self.v = (t.detach().clone().contiguous() for t in (q, k, v))
        self.status = torch.zeros(1, dtype=torch.int32, device=q.device)
        self.dout = torch.zeros_like(self.q) if backward else None
        side = torch.cuda.Stream(q.device)
        side.wait_stream(torch.cuda.current_stream(q.device))
        with torch.cuda.stream(side):  # warm-up outside capture fills every cache
            for _ in range(warmup):
                self._fwd()
                if backward:
                    self._bwd(*self._fwd())
        torch.cuda.current_stream(q.device).wait_stream(side)
        torch.cuda.synchronize(q.device)
        self.fwd_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.fwd_graph):
            self.out, self.lse = self._fwd()
        self.bwd_graph = None
        if backward:
            self.bwd_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.bwd_graph):
                self.dq, self.dk, self.dv = self._bwd(self.out, self.lse)

    def _fwd(self):
        return flash_attn_fwd(self.q, self.k, self.v, causal=self.causal,
                              softmax_scale=self.scale, status=self.status)

    def _bwd(self, out, lse):
        return flash_attn_bwd(self.dout, self.q, self.k, self.v, out, lse, causal=self.causal,
                              softmax_scale=self.scale, status=self.status)

    def forward(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor
                ) -> Tuple[torch.Tensor, torch.Tensor]:
        self.q.copy_(q)
        self.k.copy_(k)
        self.v.copy_(v)
        self.fwd_graph.replay()
        return self.out, self.lse

    __call__ = forward

    def backward(self, dout: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        if self.bwd_graph is None:
            raise RuntimeError("constructed without backward=True")
        self.dout.copy_(dout)
        self.bwd_graph.replay()
        return self.dq, self.dk, self.dv
