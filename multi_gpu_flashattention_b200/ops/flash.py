"""Single-GPU attention on the sm_100a kernels.

Tensors use the [batch, seq, heads, head_dim] layout. The tcgen05 kernels take
bf16 or fp16 q/k/v (one dtype) with head_dim 64 or 128, any number of query
heads that is a multiple of the kv heads (GQA/MQA), and write an output of the
input dtype plus an fp32 natural-log LSE [batch, heads, seq]; gradients are
fp32.

Causal masking is expressed with per-tile global token positions: key tile j
is visible to query tile i where kv_tile_pos[j] + c <= q_tile_pos[i] + r for
row r, column c. Contiguous self-attention uses tile t -> 128 * t for both
sides (top-left aligned); sharded layouts pass the positions of their tiles.
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch

from .._ext import C

TILE = 128
# bound of every in-kernel wait (ns); MGFA_WAIT_LIMIT_NS overrides it
DEFAULT_WAIT_LIMIT_NS = int(os.environ.get("MGFA_WAIT_LIMIT_NS", 2_000_000_000))


class KernelStatusError(RuntimeError):
    """A kernel reported a non-zero status word (timeout, tag mismatch...)."""


_CODES = {1: "mbarrier wait timed out", 2: "peer flag wait timed out",
          3: "received slot carried the wrong tag", 4: "bad argument",
          5: "out-of-bounds store skipped (debug build)"}


def _status_error(v: int, what: str) -> KernelStatusError:
    code, site, step = v & 0xFF, (v >> 8) & 0xFF, v >> 16
    return KernelStatusError(
        f"{what}: {_CODES.get(code, 'error')} (code {code}, site {site}, step {step})")


def check_status(status: torch.Tensor, what: str = "kernel") -> None:
    """Raise KernelStatusError when `status` (int32 CUDA tensor) is non-zero.
    Synchronises with the device."""
    v = int(status.view(-1)[0].item()) & 0xFFFFFFFF
    if v:
        raise _status_error(v, what)


class StatusMonitor:
    """The status word of public-API calls that pass none, for one device, and
    its asynchronous read-back.

    Every such call runs its kernels against this word (they record the first
    error with an atomic compare-and-swap from 0, so the word is sticky) and
    then enqueues a 4-byte copy of it into a pinned host slot, followed by an
    event. The next public call on the device (and check_errors()) looks at the
    read-backs whose events have completed, without waiting for the device, and
    raises KernelStatusError for a non-zero word; the word is re-armed (zeroed,
    stream-ordered) first. At most `depth` read-backs stay in flight; a call
    that would exceed that waits for the oldest one. So a kernel error surfaces
    at the latest a few calls later, without a device synchronisation per call
    (the reference aborts the job instead: ring/attention/bench/
    ring_attention_nccl_gpu_bench.cu:28-45).

    After a KernelStatusError from a ring call the ranks' flag states may
    disagree; re-arm them collectively with parallel.ring.reset_ring()."""

    def __init__(self, device, depth: int = 8):
        self.device = torch.device(device)
        self.word = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.depth = depth
        self.pending = []  # (event or None, pinned host slot, what)
        self._free = []

    def _slot(self):
        if self._free:
            return self._free.pop()
        return torch.zeros(1, dtype=torch.int32, pin_memory=self.device.type == "cuda")

    def after_launch(self, what: str) -> None:
        """Enqueue the read-back of the word behind the work just launched on
        the current stream (skipped under CUDA graph capture)."""
        cuda = self.device.type == "cuda"
        if cuda and torch.cuda.is_current_stream_capturing():
            return
        if len(self.pending) >= self.depth:
            self.poll(wait_oldest=True)
        host = self._slot()
        if cuda:
            with torch.cuda.device(self.device):
                host.copy_(self.word, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record()
        else:
            host.copy_(self.word)
            ev = None
        self.pending.append((ev, host, what))

    def poll(self, wait: bool = False, wait_oldest: bool = False) -> None:
        """Raise KernelStatusError for the first completed read-back that holds
        an error. wait=True waits for every read-back in flight;
        wait_oldest=True for the oldest one only."""
        done = []
        while self.pending:
            ev, host, what = self.pending[0]
            if ev is not None and not ev.query():
                if not (wait or (wait_oldest and not done)):
                    break
                ev.synchronize()
            self.pending.pop(0)
            done.append((host, what))
        bad = None
        for host, what in done:
            v = int(host[0]) & 0xFFFFFFFF
            if v and bad is None:
                bad = (v, what)
            self._free.append(host)
        if bad is not None:
            # later read-backs carry the same sticky word: drop them, re-arm
            for _, host, _ in self.pending:
                self._free.append(host)
            self.pending.clear()
            self.word.zero_()
            raise _status_error(*bad)


_MONITORS: dict = {}


def status_monitor(device) -> StatusMonitor:
    """The StatusMonitor of `device` (created on first use)."""
    key = str(torch.device(device))
    m = _MONITORS.get(key)
    if m is None:
        m = StatusMonitor(device)
        _MONITORS[key] = m
    return m


def check_errors(device=None, wait: bool = True) -> None:
    """Raise KernelStatusError if a kernel launched by a public call (one that
    was given no explicit status word) on `device` (default: every device used
    so far) reported an error. wait=True first waits for those calls to finish;
    wait=False only looks at the ones already finished."""
    mons = [status_monitor(device)] if device is not None else list(_MONITORS.values())
    for m in mons:
        m.poll(wait=wait)


def tile_positions(n_tokens: int, device, start: int = 0) -> torch.Tensor:
    """Global start positions of the 128-token tiles of a contiguous run."""
    n = (n_tokens + TILE - 1) // TILE
    return torch.arange(n, dtype=torch.int32, device=device) * TILE + start


_POS_CACHE: dict = {}


def _default_positions(n_tokens: int, device) -> torch.Tensor:
    """Cached read-only tile positions 0, 128, 256, ... (top-left aligned causal
    self-attention); built once per (tile count, device) with a synchronous copy,
    so later launches on any stream see finished data."""
    n = (n_tokens + TILE - 1) // TILE
    key = (n, str(device))
    t = _POS_CACHE.get(key)
    if t is None:
        t = torch.tensor([i * TILE for i in range(n)], dtype=torch.int32).to(device)
        _POS_CACHE[key] = t
    return t


# Forward kernel of flash_attn_fwd: "stepwise" (one CTA per query-tile pair,
# flash_fwd_sm100.cu, the kernel the per-step ring and the merge path use; the
# default, it measured faster at 128K) or "persistent" (one CTA per SM, dynamic
# tile scheduler, attn_fwd_persistent.cu).
FWD_KERNEL = os.environ.get("MGFA_FWD_KERNEL", "stepwise")
# softmax variant of the persistent forward (attn_fwd_persistent.cuh: bits 0-7
# exponential pairs of every 8 on the FMA pipe, bit 8 packed f32x2 arithmetic,
# bit 9 P handed over in two halves); -1: the kernel's default
FWD_TUNE = int(os.environ.get("MGFA_FWD_TUNE", "-1"), 0)

_SCHED: dict = {}


def sched_counters(device) -> torch.Tensor:
    """Work counters of the persistent forward for the current stream of
    `device`: two int32 zeros, which every launch leaves zeroed again. One pair
    per (device, stream), so launches that may overlap never share one."""
    dev = torch.device(device)
    if dev.type != "cuda":  # the kernel's argument checks reject host tensors
        return torch.zeros(2, dtype=torch.int32)
    key = (str(dev), torch.cuda.current_stream(dev).cuda_stream)
    t = _SCHED.get(key)
    if t is None:
        t = torch.zeros(2, dtype=torch.int32, device=dev)
        _SCHED[key] = t
    return t


def _scale(q: torch.Tensor, softmax_scale: Optional[float]) -> float:
    return softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])


def flash_attn_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                   softmax_scale: Optional[float] = None,
                   q_tile_pos: Optional[torch.Tensor] = None,
                   kv_tile_pos: Optional[torch.Tensor] = None,
                   out: Optional[torch.Tensor] = None,
                   status: Optional[torch.Tensor] = None,
                   wait_limit_ns: int = DEFAULT_WAIT_LIMIT_NS):
    """Forward attention; returns (out [B,Sq,Hq,D] in q's dtype, lse fp32 [B,Hq,Sq])."""
    B, Sq, Hq, _ = q.shape
    if causal:
        if q_tile_pos is None:
            q_tile_pos = _default_positions(Sq, q.device)
        if kv_tile_pos is None:
            kv_tile_pos = _default_positions(k.shape[1], q.device)
    o = out if out is not None else torch.empty_like(q)
    lse = torch.empty(B, Hq, Sq, dtype=torch.float32, device=q.device)
    mon = status_monitor(q.device) if status is None else None
    if mon is not None:
        mon.poll()  # an error of an earlier, finished call surfaces here
    st = status if status is not None else mon.word
    if FWD_KERNEL == "persistent":
        C().flash_fwd_persistent(q, k, v, o, lse, _scale(q, softmax_scale), causal, q_tile_pos,
                                 kv_tile_pos, st, int(wait_limit_ns), sched_counters(q.device),
                                 FWD_TUNE)
    else:
        C().flash_fwd(q, k, v, o, None, lse, _scale(q, softmax_scale), causal, q_tile_pos,
                      kv_tile_pos, False, True, st, int(wait_limit_ns))
    if mon is not None:
        mon.after_launch("flash_attn_fwd")
    return o, lse


def flash_attn_fwd_step(q, k, v, o_state, lse, *, causal, softmax_scale=None, q_tile_pos=None,
                        kv_tile_pos=None, merge: bool, final_out: bool, out=None, status=None,
                        wait_limit_ns: int = DEFAULT_WAIT_LIMIT_NS):
    """One partial pass of q over (k, v) merged into the running (o_state, lse).

    o_state: fp32 [B,Sq,Hq,D] normalised running output; lse: fp32 [B,Hq,Sq].
    With merge=False the pass starts a new state; with final_out=True the merged
    result is written to `out` (q's dtype) instead of o_state."""
    st = status if status is not None else torch.zeros(1, dtype=torch.int32, device=q.device)
    C().flash_fwd(q, k, v, out, o_state, lse, _scale(q, softmax_scale), causal, q_tile_pos,
                  kv_tile_pos, merge, final_out, st, int(wait_limit_ns))
    return st


# ---------------------------------------------------------------------- backward
def flash_attn_bwd(dout, q, k, v, out, lse, causal: bool = False,
                   softmax_scale: Optional[float] = None, q_tile_pos=None, kv_tile_pos=None,
                   dq=None, dk=None, dv=None, accumulate: bool = False, lse2=None, delta=None,
                   status=None, wait_limit_ns: int = DEFAULT_WAIT_LIMIT_NS):
    """Gradients of one attention pass into fp32 buffers (allocated when None).

    lse is the natural-log LSE of the complete attention the output came from
    (for ring attention: the merged LSE over all steps). Returns (dq, dk, dv) fp32."""
    if causal:
        if q_tile_pos is None:
            q_tile_pos = _default_positions(q.shape[1], q.device)
        if kv_tile_pos is None:
            kv_tile_pos = _default_positions(k.shape[1], q.device)
    f32 = dict(dtype=torch.float32, device=q.device)
    dq = dq if dq is not None else torch.empty(q.shape, **f32)
    dk = dk if dk is not None else torch.empty(k.shape, **f32)
    dv = dv if dv is not None else torch.empty(v.shape, **f32)
    mon = status_monitor(q.device) if status is None else None
    if mon is not None:
        mon.poll()
    st = status if status is not None else mon.word
    C().flash_bwd(dout.contiguous(), q, k, v, out, lse, dq, dk, dv, _scale(q, softmax_scale),
                  causal, q_tile_pos, kv_tile_pos, accumulate, lse2, delta, st, int(wait_limit_ns))
    if mon is not None:
        mon.after_launch("flash_attn_bwd")
    return dq, dk, dv


class _FlashAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, causal, softmax_scale):
        out, lse = flash_attn_fwd(q, k, v, causal=causal, softmax_scale=softmax_scale)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.cfg = (causal, softmax_scale)
        return out, lse

    @staticmethod
    def backward(ctx, d_out, d_lse):
        q, k, v, out, lse = ctx.saved_tensors
        causal, scale = ctx.cfg
        dq, dk, dv = flash_attn_bwd(d_out, q, k, v, out, lse, causal=causal, softmax_scale=scale)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None


def flash_attn(q, k, v, causal: bool = False, softmax_scale: Optional[float] = None,
               return_lse: bool = False):
    """Differentiable single-GPU attention on the sm_100a kernels.
    q [B,S,Hq,D], k/v [B,S,Hkv,D] bf16 or fp16 (D = 64 or 128) -> out [B,S,Hq,D]."""
    out, lse = _FlashAttnFn.apply(q, k, v, causal, softmax_scale)
    return (out, lse) if return_lse else out
