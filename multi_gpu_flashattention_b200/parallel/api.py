"""User-facing ring attention: ring_attention(q, k, v, causal, group, layout)."""
from __future__ import annotations

from typing import Optional, Union

import torch
import torch.distributed as dist

from .layouts import RingLayout
from .ring import ring_attention_forward


def _world(group):
    if group is None and not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def resolve_layout(layout: Union[None, str, RingLayout], local_len: int, world: int,
                   causal: bool) -> RingLayout:
    """A RingLayout for equal local shards of `local_len` tokens. The default is
    zigzag for causal attention on more than one rank, contiguous otherwise."""
    if isinstance(layout, RingLayout):
        return layout
    kind = layout or ("zigzag" if causal and world > 1 else "contiguous")
    if kind == "scheduler":
        raise ValueError("pass a RingLayout for scheduler-driven shards (their lengths differ)")
    return RingLayout(kind, local_len * world, world, mask="causal" if causal else "full")


class _RingAttnFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, layout, causal, scale, group, backend, health):
        out, lse = ring_attention_forward(q, k, v, layout, causal=causal, softmax_scale=scale,
                                          group=group, backend=backend, health=health)
        ctx.save_for_backward(q, k, v, out, lse)
        ctx.cfg = (layout, causal, scale, group, backend, health)
        return out, lse

    @staticmethod
    def backward(ctx, d_out, d_lse):
        from .ring_bwd import ring_attention_backward
        q, k, v, out, lse = ctx.saved_tensors
        layout, causal, scale, group, backend, health = ctx.cfg
        dq, dk, dv = ring_attention_backward(d_out, q, k, v, out, lse, layout, causal=causal,
                                             softmax_scale=scale, group=group, backend=backend,
                                             health=health)
        return dq, dk, dv, None, None, None, None, None, None


def ring_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                   group=None, layout: Union[None, str, RingLayout] = None,
                   softmax_scale: Optional[float] = None, backend: Optional[str] = None,
                   return_lse: bool = False, health=None):
    """Context-parallel attention over `group` (default: the world group).

    q [B, L, Hq, D], k/v [B, L, Hkv, D]: this rank's shard under `layout`
    (RingLayout.shard() produces it from a global tensor). Returns this rank's
    shard of the output (and the fp32 LSE [B, Hq, L] with return_lse=True).
    Differentiable: the backward pass runs its own ring (dK/dV travel with K/V).
    With `health` (a parallel.health.RingHealth), forward and backward first
    pass the liveness gate, so a departed or silent peer raises PeerLostError
    before anything is launched.
    """
    _, world = _world(group)
    lay = resolve_layout(layout, q.shape[1], world, causal)
    out, lse = _RingAttnFn.apply(q, k, v, lay, causal, softmax_scale, group, backend, health)
    return (out, lse) if return_lse else out
