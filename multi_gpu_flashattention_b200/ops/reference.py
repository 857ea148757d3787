"""Plain PyTorch fp32 attention used as the numerics oracle in tests and checks."""
from __future__ import annotations

import math
from typing import Optional

import torch


def attention_ref(q, k, v, causal: bool = False, softmax_scale: Optional[float] = None,
                  q_pos: Optional[torch.Tensor] = None, k_pos: Optional[torch.Tensor] = None):
    """Exact attention in fp32. q [B,Sq,Hq,D], k/v [B,Sk,Hkv,D] (any float dtype).

    Causal visibility is k_pos[j] <= q_pos[i] (defaults: 0..S-1 on both sides).
    Returns (out fp32 [B,Sq,Hq,D], lse fp32 [B,Hq,Sq]); rows that see no key get
    out = 0 and lse = -inf."""
    q, k, v = q.float(), k.float(), v.float()
    B, Sq, Hq, D = q.shape
    Sk, Hkv = k.shape[1], k.shape[2]
    scale = softmax_scale if softmax_scale is not None else 1.0 / math.sqrt(D)
    if Hq != Hkv:
        k = k.repeat_interleave(Hq // Hkv, dim=2)
        v = v.repeat_interleave(Hq // Hkv, dim=2)
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) * scale
    if causal:
        if q_pos is None:
            q_pos = torch.arange(Sq, device=q.device)
        if k_pos is None:
            k_pos = torch.arange(Sk, device=q.device)
        vis = k_pos.view(1, -1).to(q.device) <= q_pos.view(-1, 1).to(q.device)
        s = s.masked_fill(~vis, float("-inf"))
    lse = torch.logsumexp(s, dim=-1)
    p = torch.exp(s - lse.unsqueeze(-1))
    p = torch.nan_to_num(p, nan=0.0)
    o = torch.einsum("bhqk,bkhd->bqhd", p, v)
    return o, lse
