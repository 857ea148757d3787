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
from typing import Optional

import torch

from .._ext import C

TILE = 128
DEFAULT_WAIT_LIMIT_NS = 2_000_000_000


class KernelStatusError(RuntimeError):
    """A kernel reported a non-zero status word (timeout, tag mismatch...)."""


_CODES = {1: "mbarrier wait timed out", 2: "peer flag wait timed out",
          3: "received slot carried the wrong tag", 4: "bad argument",
          5: "out-of-bounds store skipped (debug build)"}


def check_status(status: torch.Tensor, what: str = "kernel") -> None:
    """Raise KernelStatusError when `status` (int32 CUDA tensor) is non-zero.
    Synchronises with the device."""
    v = int(status.view(-1)[0].item()) & 0xFFFFFFFF
    if v:
        code, site, step = v & 0xFF, (v >> 8) & 0xFF, v >> 16
        raise KernelStatusError(
            f"{what}: {_CODES.get(code, 'error')} (code {code}, site {site}, step {step})")


def tile_positions(n_tokens: int, device, start: int = 0) -> torch.Tensor:
    """Global start positions of the 128-token tiles of a contiguous run."""
    n = (n_tokens + TILE - 1) // TILE
    return torch.arange(n, dtype=torch.int32, device=device) * TILE + start


_POS_CACHE: dict = {}
_STATUS_CACHE: dict = {}


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


def _scratch_status(device) -> torch.Tensor:
    """Status word for calls that pass none: kernels only write it on an error
    nobody asked to see, so one zeroed word per device serves every such call."""
    key = str(device)
    t = _STATUS_CACHE.get(key)
    if t is None:
        t = torch.zeros(1, dtype=torch.int32, device=device)
        _STATUS_CACHE[key] = t
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
    st = status if status is not None else _scratch_status(q.device)
    C().flash_fwd(q, k, v, o, None, lse, _scale(q, softmax_scale), causal, q_tile_pos,
                  kv_tile_pos, False, True, st, int(wait_limit_ns))
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
    st = status if status is not None else _scratch_status(q.device)
    C().flash_bwd(dout.contiguous(), q, k, v, out, lse, dq, dk, dv, _scale(q, softmax_scale),
                  causal, q_tile_pos, kv_tile_pos, accumulate, lse2, delta, st, int(wait_limit_ns))
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
