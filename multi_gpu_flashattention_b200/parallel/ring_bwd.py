"""Ring attention backward.

Each rank keeps its queries, output, dO and the merged LSE of the forward; the
KV shards travel around the ring again, this time together with fp32
accumulators for their dK and dV. At step t rank r adds its contribution to
owner (r - t) mod P's accumulators and passes shard + accumulators on; after
P steps each accumulator holds every rank's contribution and takes one last
hop to its owner. dQ accumulates locally.

Backends: "fused" (default on CUDA) runs the native RingBwdEngine: the dK/dV
kernel pushes K/V to the right neighbour and stores the updated accumulators
straight into its receive slot over NVLink (see csrc/comm/ring_bwd_engine.cpp);
"nccl" is the baseline that moves K/V and the accumulators with NCCL send/recv
on a side stream; "torch" is the fp32 PyTorch oracle on any device.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist

from .._ext import C
from ..ops.flash import DEFAULT_WAIT_LIMIT_NS, flash_attn_bwd, status_monitor
from .layouts import RingLayout


def _world(group):
    if group is None and not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def _global(group, r):
    return dist.get_global_rank(group, r) if group is not None else r


def _p2p(group, sends, recvs, right, left):
    ops = [dist.P2POp(dist.isend, t, right, group) for t in sends]
    ops += [dist.P2POp(dist.irecv, t, left, group) for t in recvs]
    return dist.batch_isend_irecv(ops) if ops else []


def ring_attention_backward(dout, q, k, v, out, lse, layout: RingLayout, causal: bool = False,
                            softmax_scale: Optional[float] = None, group=None,
                            backend: Optional[str] = None, health=None):
    """Gradients (dq, dk, dv) of the ring forward for this rank's shard. With a
    `health` (RingHealth) every rank first passes its gate, as in the forward."""
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    rank, world = _world(group)
    if health is not None and world > 1:
        health.gate()
    if backend == "torch" or not q.is_cuda:
        return _bwd_torch(dout, q, k, v, layout, causal, scale, group)
    from .ring import _meta
    qtp, kvtp, kv_lens = _meta(layout, rank, q.device)
    dout = dout.contiguous()
    if world == 1:
        dq, dk, dv = flash_attn_bwd(dout, q, k[:, :kv_lens[0]], v[:, :kv_lens[0]], out, lse,
                                    causal=causal, softmax_scale=scale, q_tile_pos=qtp,
                                    kv_tile_pos=kvtp[0])
        dk_full = torch.zeros(k.shape, dtype=torch.float32, device=q.device)
        dv_full = torch.zeros(v.shape, dtype=torch.float32, device=q.device)
        dk_full[:, :kv_lens[0]] = dk
        dv_full[:, :kv_lens[0]] = dv
        return dq.to(q.dtype), dk_full.to(k.dtype), dv_full.to(v.dtype)

    if backend in (None, "fused", "fused_stepwise", "fused_one_launch"):
        return _bwd_fused(dout, q, k, v, out, lse, causal, scale, group, qtp, kvtp, kv_lens)
    right, left = _global(group, (rank + 1) % world), _global(group, (rank - 1) % world)
    lse2, delta = C().flash_bwd_preprocess(dout, out, lse)
    compute = torch.cuda.current_stream(q.device)
    comm = torch.cuda.Stream(q.device)
    f32 = dict(dtype=torch.float32, device=q.device)
    dq = torch.empty(q.shape, **f32)
    # K/V arrive in two alternating receive pairs (the caller's k and v, which
    # autograd saved, are never written); the fp32 accumulators alternate too
    kv_recv = [[torch.empty_like(k), torch.empty_like(v)] for _ in range(min(2, world - 1))]
    acc = [[torch.empty(k.shape, **f32), torch.empty(v.shape, **f32)] for _ in range(2)]
    cur = [k.contiguous(), v.contiguous()] + acc[0]
    for t in range(world):
        owner = (rank - t) % world
        kl = kv_lens[owner]
        nxt = (kv_recv[t % 2] if t < world - 1 else [None, None]) + acc[(t + 1) % 2]
        # K/V of the next step can move while this step computes
        reqs = []
        if t < world - 1:
            comm.wait_stream(compute)
            with torch.cuda.stream(comm):
                reqs = _p2p(group, cur[:2], nxt[:2], right, left)
        flash_attn_bwd(dout, q, cur[0][:, :kl], cur[1][:, :kl], out, lse, causal=causal,
                       softmax_scale=scale, q_tile_pos=qtp, kv_tile_pos=kvtp[owner],
                       dq=dq, dk=cur[2][:, :kl], dv=cur[3][:, :kl], accumulate=t > 0,
                       lse2=lse2, delta=delta)
        if kl < k.shape[1] and t == 0:
            cur[2][:, kl:].zero_()
            cur[3][:, kl:].zero_()
        # the accumulators follow once this step's contribution is in
        comm.wait_stream(compute)
        with torch.cuda.stream(comm):
            for rq in reqs:
                rq.wait()
            if t < world - 1:
                acc_reqs = _p2p(group, cur[2:], nxt[2:], right, left)
            else:  # last hop: each accumulator goes home
                home = [torch.empty_like(cur[2]), torch.empty_like(cur[3])]
                acc_reqs = _p2p(group, cur[2:], home, right, left)
            for rq in acc_reqs:
                rq.wait()
        compute.wait_stream(comm)
        if t < world - 1:
            cur = nxt
    return dq.to(q.dtype), home[0].to(k.dtype), home[1].to(v.dtype)


def _bwd_torch(dout, q, k, v, layout, causal, scale, group):
    """fp32 oracle: gradients of the ring forward computed with autograd on
    all-gathered keys/values (exact, for tests)."""
    rank, world = _world(group)
    from ..ops.reference import attention_ref
    ks = [torch.empty_like(k) for _ in range(world)]
    vs = [torch.empty_like(v) for _ in range(world)]
    if world > 1:
        dist.all_gather(ks, k.contiguous(), group=group)
        dist.all_gather(vs, v.contiguous(), group=group)
    else:
        ks, vs = [k], [v]
    kv_lens = layout.kv_lens()
    q_pos = layout.q_positions_for_mask(rank).to(q.device)
    k_pos = torch.cat([layout.k_positions_for_mask(rank, o)[:kv_lens[o]] for o in range(world)])
    with torch.enable_grad():  # also when called from an autograd.Function backward
        kfull = torch.cat([ks[o][:, :kv_lens[o]] for o in range(world)], 1).detach().float()
        vfull = torch.cat([vs[o][:, :kv_lens[o]] for o in range(world)], 1).detach().float()
        kfull.requires_grad_()
        vfull.requires_grad_()
        qf = q.detach().float().requires_grad_()
        o_ref, _ = attention_ref(qf, kfull, vfull, causal=causal, softmax_scale=scale,
                                 q_pos=q_pos, k_pos=k_pos.to(q.device))
        dq, dkf, dvf = torch.autograd.grad(o_ref, (qf, kfull, vfull), dout.float())
    # gradients of every owner's keys: sum over ranks, then keep ours
    offs = [0]
    for o in range(world):
        offs.append(offs[-1] + kv_lens[o])
    dk_parts = [torch.zeros(k.shape, dtype=torch.float32, device=q.device) for _ in range(world)]
    dv_parts = [torch.zeros(v.shape, dtype=torch.float32, device=q.device) for _ in range(world)]
    for o in range(world):
        dk_parts[o][:, :kv_lens[o]] = dkf[:, offs[o]:offs[o + 1]]
        dv_parts[o][:, :kv_lens[o]] = dvf[:, offs[o]:offs[o + 1]]
    dk_all = torch.stack(dk_parts)
    dv_all = torch.stack(dv_parts)
    if world > 1:
        dist.all_reduce(dk_all, group=group)
        dist.all_reduce(dv_all, group=group)
    return dq.to(q.dtype), dk_all[rank].to(k.dtype), dv_all[rank].to(v.dtype)


class _BwdEngines:
    """One native RingBwdEngine per (process group, device); creation is collective."""

    def __init__(self):
        self._by_key = {}

    def get(self, group, device, kv_bytes):
        rank, world = _world(group)
        key = (id(group), device.index)
        eng = self._by_key.get(key)
        if eng is not None and eng.kv_bytes() >= kv_bytes:
            return eng
        if eng is not None:
            torch.cuda.synchronize(device)
            dist.barrier(group)
            self._by_key.pop(key)
            del eng
        size = max(kv_bytes, 1 << 20)
        size = (size + (2 << 20) - 1) // (2 << 20) * (2 << 20)
        eng = C().RingBwdEngine(rank, world, device.index, size, 0)
        handles = [None] * world
        dist.all_gather_object(handles, eng.ipc_handle(), group=group)
        eng.connect(handles)
        torch.cuda.synchronize(device)
        dist.barrier(group)
        self._by_key[key] = eng
        return eng

    def clear(self):
        self._by_key.clear()


BWD_ENGINES = _BwdEngines()


def _bwd_fused(dout, q, k, v, out, lse, causal, scale, group, qtp, kvtp, kv_lens,
               status=None, wait_limit_ns=DEFAULT_WAIT_LIMIT_NS):
    rank, world = _world(group)
    eng = BWD_ENGINES.get(group, q.device, k.numel() * k.element_size())
    mon = None
    if status is None:  # report into the device's StatusMonitor (see ops.flash)
        mon = status_monitor(q.device)
        mon.poll()
        st = mon.word
    else:
        st = status
    dq, dk, dv = eng.backward(dout, q.contiguous(), k.contiguous(), v.contiguous(), out.contiguous(),
                              lse, scale, causal, qtp if causal else None,
                              kvtp if causal else None, kv_lens, st, int(wait_limit_ns))
    if mon is not None:
        mon.after_launch("ring attention backward (fused)")
    kl = kv_lens[rank]
    if kl < k.shape[1]:  # padding rows of a shorter shard carry no gradient
        dk[:, kl:].zero_()
        dv[:, kl:].zero_()
    return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype)
