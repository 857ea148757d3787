"""Ring attention over a torch.distributed process group.

Every rank holds the local shard (given by a RingLayout) of q, k and v in the
[batch, local_seq, heads, head_dim] layout. Over P ring steps the KV shards
travel to the right neighbour while each rank attends its queries to the shard
it currently holds; the partial results are merged with their log-sum-exp.
The schedule is the reference's: at step t rank r computes on the shard of
owner (r - t) mod P and receives the shard of owner (r - t - 1) mod P
(ring/attention/common/shard_utils.cuh:29-35,
ring/attention/bench/ring_attention_nccl_gpu_bench.cu:349-397).

Backends
--------
fused   (default on CUDA) the fused ring engine that MGFA_RING_ENGINE selects:
        "stepwise" (default) or "one_launch".
fused_stepwise
        one sm_100a kernel launch per ring step that computes, merges in-kernel
        and pushes the current shard into the right neighbour's receive slot
        (native RingEngine).
fused_one_launch
        the whole ring in ONE launch of the persistent sm_100a kernel (native
        RingEngineP): every rank keeps a receive slot per ring step, computes
        each query tile against its own shard and then every received shard as
        its kv-head chunk arrives, with the softmax state on chip across steps
        (no per-step merge), while the kernel's push warps forward each received
        chunk to the right neighbour with peer stores.
p2p_unfused, ce_unfused
        ablations of `fused_stepwise`: the same engine, slots and flags, with the
        shard moved on a second stream by the standalone push kernel or by the
        copy engine (forward only; their backward uses the nccl path).
nccl    baseline: NCCL send/recv on a side stream, overlapped with the same
        attention kernel (merge in-kernel).
staged  baseline: device -> pinned host -> gloo send/recv -> device, the
        reference's staged-MPI path re-expressed without MPI.
torch   pure PyTorch fp32 on any device (the protocol oracle; CPU + gloo).
"""
from __future__ import annotations

import math
import os
from typing import Optional, Tuple

import torch
import torch.distributed as dist

from .._ext import C
from ..ops.flash import (DEFAULT_WAIT_LIMIT_NS, check_status, flash_attn_fwd,
                         flash_attn_fwd_step, status_monitor)
from ..ops.reference import attention_ref
from .layouts import RingLayout

BACKENDS = ("fused", "fused_stepwise", "fused_one_launch", "p2p_unfused", "ce_unfused", "nccl",
            "staged", "torch")
# The engine behind backend "fused": "stepwise" (one kernel launch per ring step,
# the default) or "one_launch" (the whole ring in one persistent-kernel launch).
RING_ENGINE = os.environ.get("MGFA_RING_ENGINE", "stepwise")


def resolve_backend(backend: Optional[str], is_cuda: bool = True) -> str:
    """The concrete backend a name selects: None means "fused" on CUDA and
    "torch" elsewhere, and "fused" means the engine MGFA_RING_ENGINE names."""
    if backend is None:
        backend = "fused" if is_cuda else "torch"
    if backend == "fused":
        backend = "fused_one_launch" if RING_ENGINE == "one_launch" else "fused_stepwise"
    return backend


# transport modes of the per-step engine (RingEngine.set_transport_mode)
_ENGINE_MODES = {"fused_stepwise": 0, "p2p_unfused": 1, "ce_unfused": 2}


def _world(group) -> Tuple[int, int]:
    if group is None and not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def _global_rank(group, r: int) -> int:
    return dist.get_global_rank(group, r) if group is not None else r


_HOST_GROUPS: dict = {}


def _host_group(group):
    """Process group for the staged transport's pinned host buffers: `group`
    itself when it is gloo, else a gloo group over the whole world, created
    once (collectively) for the default group. A non-gloo sub-group needs an
    explicit `cpu_group`, because creating a group is collective over every
    rank of the job."""
    if dist.get_backend(group) == "gloo":
        return group
    if group is not None:
        raise ValueError("backend='staged' on a sub-group needs cpu_group=<gloo group over the "
                         "same ranks>")
    g = _HOST_GROUPS.get(None)
    if g is None:
        g = dist.new_group(list(range(dist.get_world_size())), backend="gloo")
        _HOST_GROUPS[None] = g
    return g


# ---------------------------------------------------------------------- engine cache
class _Engines:
    """One native RingEngine per (process group, device); grown on demand.
    Creating or growing an engine is collective over the group."""

    def __init__(self):
        self._by_key = {}

    def get(self, group, device: torch.device, slot_bytes: int):
        rank, world = _world(group)
        key = (id(group), device.index)
        eng = self._by_key.get(key)
        if eng is not None and eng.slot_bytes() >= slot_bytes:
            return eng
        slot = max(slot_bytes, 1 << 20)
        slot = (slot + (2 << 20) - 1) // (2 << 20) * (2 << 20)
        if eng is not None:
            torch.cuda.synchronize(device)
            dist.barrier(group)  # every rank is past its last use of the old slots
            self._by_key.pop(key)
            del eng
        eng = C().RingEngine(rank, world, device.index, slot, int(os.environ.get("MGFA_RING_CHUNKS", 0)))
        # MGFA_TAG_CHECK=0 skips the consumers' owner-tag check (an experiment
        # knob: one system-scope load less per CTA and step)
        eng.set_tag_check(os.environ.get("MGFA_TAG_CHECK", "1") != "0")
        # Arrival counts keep growing (cumulative targets, wrap-safe waits), so
        # dependent launch stays on for every grid size; MGFA_CUMULATIVE_ARRIVALS=0
        # re-arms them per use instead (small grids then run without dependent
        # launch at P >= 5)
        eng.set_cumulative_arrivals(os.environ.get("MGFA_CUMULATIVE_ARRIVALS", "1") != "0")
        handles = [None] * world
        dist.all_gather_object(handles, eng.ipc_handle(), group=group)
        eng.connect(handles)
        torch.cuda.synchronize(device)
        dist.barrier(group)
        self._by_key[key] = eng
        return eng

    def clear(self):
        self._by_key.clear()


ENGINES = _Engines()


class _PEngines:
    """One native RingEngineP (the one-launch ring) per (process group,
    device); grown on demand. Creating or growing an engine is collective."""

    def __init__(self):
        self._by_key = {}

    def get(self, group, device: torch.device, shard_bytes: int):
        rank, world = _world(group)
        key = (id(group), device.index)
        eng = self._by_key.get(key)
        if eng is not None and eng.shard_bytes() >= shard_bytes:
            return eng
        cap = max(shard_bytes, 1 << 20)
        cap = (cap + (2 << 20) - 1) // (2 << 20) * (2 << 20)
        if eng is not None:
            torch.cuda.synchronize(device)
            dist.barrier(group)  # every rank is past its last use of the old slots
            self._by_key.pop(key)
            del eng
        eng = C().RingEngineP(rank, world, device.index, cap)
        # MGFA_P_PUSH_CTAS=k: the last k CTAs of the one-launch grid only push and
        # the others only compute (an experiment on the ring's open defect)
        eng.set_push_ctas(int(os.environ.get("MGFA_P_PUSH_CTAS", "0")))
        handles = [None] * world
        dist.all_gather_object(handles, eng.ipc_handle(), group=group)
        eng.connect(handles)
        torch.cuda.synchronize(device)
        dist.barrier(group)
        self._by_key[key] = eng
        return eng

    def clear(self):
        self._by_key.clear()


P_ENGINES = _PEngines()


# ---------------------------------------------------------------------- metadata cache
_META = {}


def _meta(layout: RingLayout, rank: int, device):
    key = (layout.kind, layout.seq, layout.world, layout.policy, layout.block, rank, str(device))
    m = _META.get(key)
    if m is None:
        m = (layout.q_tile_pos(rank, device), layout.kv_tile_pos_by_owner(rank, device).contiguous(),
             layout.kv_lens())
        _META[key] = m
    return m


# ---------------------------------------------------------------------- forward backends
def _fwd_fused(q, k, v, layout, causal, scale, group, status, wait_ns, mode="fused_stepwise"):
    """The per-step engine's ring. mode "fused_stepwise": the transport runs
    inside each step's attention kernel; "p2p_unfused": the same NVLink push as
    a separate all-SM kernel on a second stream; "ce_unfused": the copy engine
    moves the shard on a second stream (both ablations keep the flags and
    slots)."""
    rank, world = _world(group)
    qtp, kvtp, kv_lens = _meta(layout, rank, q.device)
    shard_bytes = k.numel() * k.element_size()
    eng = ENGINES.get(group, q.device, shard_bytes)
    eng.set_transport_mode(_ENGINE_MODES[mode])
    try:
        o, lse = eng.forward(q, k, v, scale, causal, qtp if causal else None,
                             kvtp if causal else None, kv_lens, status, int(wait_ns))
    finally:
        eng.set_transport_mode(0)
    return o, lse


def _fwd_persistent(q, k, v, layout, causal, scale, group, status, wait_ns):
    """The one-launch ring of the persistent kernel (RingEngineP)."""
    rank, world = _world(group)
    qtp, kvtp, kv_lens = _meta(layout, rank, q.device)
    eng = P_ENGINES.get(group, q.device, k.numel() * k.element_size())
    return eng.forward(q, k, v, scale, causal, qtp if causal else None,
                       kvtp if causal else None, kv_lens, status, int(wait_ns))


def _fwd_nccl(q, k, v, layout, causal, scale, group, status, wait_ns, overlap=True):
    rank, world = _world(group)
    qtp, kvtp, kv_lens = _meta(layout, rank, q.device)
    right = _global_rank(group, (rank + 1) % world)
    left = _global_rank(group, (rank - 1) % world)
    compute = torch.cuda.current_stream(q.device)
    comm = torch.cuda.Stream(q.device) if overlap else compute
    o_state = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    lse = torch.empty(q.shape[0], q.shape[2], q.shape[1], dtype=torch.float32, device=q.device)
    out = torch.empty_like(q)
    # step t computes on cur while receive pair t % 2 fills; the caller's k and v
    # (saved for the backward pass) are never written
    cur = (k, v)
    recv = [(torch.empty_like(k), torch.empty_like(v)) for _ in range(min(2, world - 1))]
    for t in range(world):
        owner = (rank - t) % world
        reqs = []
        if t < world - 1:
            nxt = recv[t % 2]
            comm.wait_stream(compute)
            with torch.cuda.stream(comm):
                ops = [dist.P2POp(dist.isend, cur[0], right, group),
                       dist.P2POp(dist.isend, cur[1], right, group),
                       dist.P2POp(dist.irecv, nxt[0], left, group),
                       dist.P2POp(dist.irecv, nxt[1], left, group)]
                reqs = dist.batch_isend_irecv(ops)
            if not overlap:
                for rq in reqs:
                    rq.wait()
        kl = kv_lens[owner]
        flash_attn_fwd_step(q, cur[0][:, :kl], cur[1][:, :kl], o_state, lse, causal=causal,
                            softmax_scale=scale, q_tile_pos=qtp, kv_tile_pos=kvtp[owner],
                            merge=t > 0, final_out=t == world - 1, out=out, status=status,
                            wait_limit_ns=wait_ns)
        if t < world - 1:
            if overlap:
                with torch.cuda.stream(comm):
                    for rq in reqs:
                        rq.wait()
                compute.wait_stream(comm)
            cur = nxt
    return out, lse


def _fwd_staged(q, k, v, layout, causal, scale, group, status, wait_ns, cpu_group=None):
    """Device -> pinned host -> gloo -> pinned host -> device per step."""
    rank, world = _world(cpu_group)
    qtp, kvtp, kv_lens = _meta(layout, rank, q.device)
    right, left = (rank + 1) % world, (rank - 1) % world
    o_state = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    lse = torch.empty(q.shape[0], q.shape[2], q.shape[1], dtype=torch.float32, device=q.device)
    out = torch.empty_like(q)
    cur = (k, v)
    h_send = [torch.empty(k.shape, dtype=k.dtype, pin_memory=True) for _ in range(2)]
    h_recv = [torch.empty(k.shape, dtype=k.dtype, pin_memory=True) for _ in range(2)]
    for t in range(world):
        owner = (rank - t) % world
        kl = kv_lens[owner]
        flash_attn_fwd_step(q, cur[0][:, :kl], cur[1][:, :kl], o_state, lse, causal=causal,
                            softmax_scale=scale, q_tile_pos=qtp, kv_tile_pos=kvtp[owner],
                            merge=t > 0, final_out=t == world - 1, out=out, status=status,
                            wait_limit_ns=wait_ns)
        if t < world - 1:
            for i in range(2):
                h_send[i].copy_(cur[i], non_blocking=False)
            reqs = []
            for i in range(2):
                reqs.append(dist.isend(h_send[i].view(torch.int16), _global_rank(cpu_group, right),
                                       group=cpu_group))
                reqs.append(dist.irecv(h_recv[i].view(torch.int16), _global_rank(cpu_group, left),
                                       group=cpu_group))
            for rq in reqs:
                rq.wait()
            cur = (h_recv[0].to(q.device, non_blocking=False), h_recv[1].to(q.device, non_blocking=False))
    return out, lse


def _fwd_torch(q, k, v, layout, causal, scale, group):
    """Pure PyTorch fp32 ring (any device; gloo on CPU). Returns fp32 out, lse."""
    rank, world = _world(group)
    right = _global_rank(group, (rank + 1) % world)
    left = _global_rank(group, (rank - 1) % world)
    q_pos = layout.q_positions_for_mask(rank).to(q.device)
    kv_lens = layout.kv_lens()
    cur = (k.contiguous(), v.contiguous())
    o = lse = None
    for t in range(world):
        owner = (rank - t) % world
        reqs, nxt = [], None
        if t < world - 1:
            nxt = (torch.empty_like(cur[0]), torch.empty_like(cur[1]))
            for i in range(2):
                reqs.append(dist.isend(cur[i], right, group=group))
                reqs.append(dist.irecv(nxt[i], left, group=group))
        kl = kv_lens[owner]
        k_pos = layout.k_positions_for_mask(rank, owner)[:kl].to(q.device)
        o_t, lse_t = attention_ref(q, cur[0][:, :kl], cur[1][:, :kl], causal=causal,
                                   softmax_scale=scale, q_pos=q_pos, k_pos=k_pos)
        if o is None:
            o, lse = o_t, lse_t
        else:
            new = torch.logaddexp(lse, lse_t)
            w_old = torch.exp(lse - new).nan_to_num(0.0).transpose(1, 2).unsqueeze(-1)
            w_new = torch.exp(lse_t - new).nan_to_num(0.0).transpose(1, 2).unsqueeze(-1)
            o = o * w_old + o_t * w_new
            lse = new
        for rq in reqs:
            rq.wait()
        if nxt is not None:
            cur = nxt
    return o, lse


def ring_attention_forward(q, k, v, layout: RingLayout, causal: bool = False,
                           softmax_scale: Optional[float] = None, group=None,
                           backend: Optional[str] = None, status: Optional[torch.Tensor] = None,
                           wait_limit_ns: int = DEFAULT_WAIT_LIMIT_NS, check: bool = False,
                           cpu_group=None, health=None):
    """Forward ring attention on local shards; returns (out, lse).

    out has q's dtype ([B, L, Hq, D]); lse is fp32 [B, Hq, L] (natural log).
    Without a `status` the kernels report into the device's StatusMonitor
    word: an error (a bounded wait that expired, a wrong slot tag) raises
    KernelStatusError at the entry of a later public call on this device, or
    in ops.flash.check_errors(), without a device sync per call. With
    check=True the status is read back right away (a device sync) and the
    error raised here. After such an error re-arm the ring on every rank with
    reset_ring(group). With a `health` (RingHealth) every rank first passes
    its gate, so a peer that left or went silent raises PeerLostError here
    instead of leaving launched kernels waiting."""
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(q.shape[-1])
    if backend is not None and backend not in BACKENDS:
        raise ValueError(f"backend must be one of {BACKENDS}")
    backend = resolve_backend(backend, q.is_cuda)
    rank, world = _world(group)
    if health is not None and world > 1:
        health.gate()
    if backend == "torch":
        return _fwd_torch(q, k, v, layout, causal, scale, group)
    mon = None
    if status is None:
        mon = status_monitor(q.device)
        mon.poll()  # an error of an earlier, finished call surfaces before any launch
        st = mon.word
    else:
        st = status
    if world == 1:
        qtp, kvtp, kv_lens = _meta(layout, rank, q.device)
        out, lse = flash_attn_fwd(q, k[:, :kv_lens[0]], v[:, :kv_lens[0]], causal=causal,
                                  softmax_scale=scale, q_tile_pos=qtp, kv_tile_pos=kvtp[0],
                                  status=st, wait_limit_ns=wait_limit_ns)
    elif backend == "fused_one_launch":
        out, lse = _fwd_persistent(q, k, v, layout, causal, scale, group, st, wait_limit_ns)
    elif backend in _ENGINE_MODES:
        out, lse = _fwd_fused(q, k, v, layout, causal, scale, group, st, wait_limit_ns,
                              mode=backend)
    elif backend == "nccl":
        out, lse = _fwd_nccl(q, k, v, layout, causal, scale, group, st, wait_limit_ns)
    else:
        if cpu_group is None:
            cpu_group = _host_group(group)
        out, lse = _fwd_staged(q, k, v, layout, causal, scale, group, st, wait_limit_ns,
                               cpu_group=cpu_group)
    what = f"ring attention ({backend})"
    if mon is not None:
        mon.after_launch(what)
        if check:
            mon.poll(wait=True)
    elif check:
        check_status(st, what)
    return out, lse


def reset_ring(group=None) -> None:
    """Re-arm the ring after a KernelStatusError (collective: every rank of
    `group` calls it). Waits for this device's work, then past a barrier zeroes
    the flag words and use counters of the group's forward and backward
    engines and this device's status word, and meets the other ranks again, so
    the next ring call starts from the same state everywhere."""
    from .ring_bwd import BWD_ENGINES
    rank, world = _world(group)
    dev = torch.device("cuda", torch.cuda.current_device())
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier(group)
    for engines in (ENGINES, P_ENGINES, BWD_ENGINES):
        eng = engines._by_key.get((id(group), dev.index))
        if eng is not None:
            eng.reset()
    mon = status_monitor(dev)
    mon.pending.clear()
    mon.word.zero_()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier(group)
