"""A context-parallel transformer block whose attention is ring attention.

Each rank holds its token shard of the hidden states ([B, L, d_model], in the
RingLayout's local order). Projections, norms, the MLP and rotary position
embeddings are ordinary per-token PyTorch ops; rotary angles use the tokens'
GLOBAL positions from the layout, so a zigzag or striped shard computes
exactly what the unsharded model computes. Attention (causal, GQA) runs over
the process group with `ring_attention`.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F

from ..parallel.api import ring_attention
from ..parallel.layouts import RingLayout


class RMSNorm(nn.Module):
    def __init__(self, dim: int, eps: float = 1e-6):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype) * self.weight


def rotary(x: torch.Tensor, positions: torch.Tensor, base: float = 10000.0) -> torch.Tensor:
    """Rotate pairs (x[..., i], x[..., i + D/2]) by position * base^(-2i/D).
    x [B, L, H, D], positions [L] (global token positions)."""
    D = x.shape[-1]
    inv = base ** (-torch.arange(0, D // 2, device=x.device, dtype=torch.float32) * 2 / D)
    ang = positions.to(x.device, torch.float32)[:, None] * inv[None, :]
    cos, sin = ang.cos()[None, :, None, :], ang.sin()[None, :, None, :]
    x1, x2 = x[..., : D // 2].float(), x[..., D // 2:].float()
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1).to(x.dtype)


class RingAttentionBlock(nn.Module):
    """Pre-norm block: x + Attn(RMSNorm(x)); then + SwiGLU(RMSNorm(.))."""

    def __init__(self, d_model: int, n_heads: int, n_kv_heads: Optional[int] = None,
                 head_dim: int = 128, mlp_mult: int = 4, causal: bool = True):
        super().__init__()
        self.h, self.hkv = n_heads, n_kv_heads or n_heads
        self.d = head_dim
        self.causal = causal
        self.norm1, self.norm2 = RMSNorm(d_model), RMSNorm(d_model)
        self.wq = nn.Linear(d_model, self.h * head_dim, bias=False)
        self.wk = nn.Linear(d_model, self.hkv * head_dim, bias=False)
        self.wv = nn.Linear(d_model, self.hkv * head_dim, bias=False)
        self.wo = nn.Linear(self.h * head_dim, d_model, bias=False)
        hidden = mlp_mult * d_model
        self.w1 = nn.Linear(d_model, hidden, bias=False)
        self.w3 = nn.Linear(d_model, hidden, bias=False)
        self.w2 = nn.Linear(hidden, d_model, bias=False)

    def forward(self, x: torch.Tensor, layout: RingLayout, rank: int = 0, group=None,
                backend: Optional[str] = None) -> torch.Tensor:
        B, L, _ = x.shape
        pos = layout.positions(rank)
        pos = torch.cat([pos, pos.new_zeros(L - pos.numel())]) if pos.numel() < L else pos
        h = self.norm1(x)
        q = rotary(self.wq(h).view(B, L, self.h, self.d), pos)
        k = rotary(self.wk(h).view(B, L, self.hkv, self.d), pos)
        v = self.wv(h).view(B, L, self.hkv, self.d)
        a = ring_attention(q.contiguous(), k.contiguous(), v.contiguous(), causal=self.causal,
                           group=group, layout=layout, backend=backend)
        x = x + self.wo(a.reshape(B, L, self.h * self.d).to(x.dtype))
        h = self.norm2(x)
        return x + self.w2(F.silu(self.w1(h)) * self.w3(h))


IGNORE_INDEX = -100


def shard_targets(ids: torch.Tensor, layout: RingLayout, rank: int) -> torch.Tensor:
    """Next-token targets of rank's shard, in the layout's local order.

    ids: the full sequence [B, S] (int64). The target of the token at global
    position p is ids[:, p + 1]; the last position and padding rows get
    IGNORE_INDEX. With zigzag or striped layouts the next token usually lives on
    another rank, so targets are cut from the full sequence on the host."""
    B, S = ids.shape
    nxt = torch.full_like(ids, IGNORE_INDEX)
    nxt[:, :-1] = ids[:, 1:]
    out = layout.shard(nxt, rank)
    n = layout.local_len(rank)
    out[:, n:] = IGNORE_INDEX
    return out


class RingTransformerLM(nn.Module):
    """Decoder-only language model with context-parallel ring attention.

    Each rank runs every layer on its own token shard (ids [B, L] in the
    layout's local order, padded to the layout's max_local_len); attention is
    the ring over `group`, everything else is per token. Parameters are
    replicated, so after `loss(...).backward()` the gradients are summed over
    the group (all-reduce, as in data parallelism) to give the unsharded
    model's gradients."""

    def __init__(self, vocab: int, d_model: int, n_layers: int, n_heads: int,
                 n_kv_heads: Optional[int] = None, head_dim: int = 128, mlp_mult: int = 4,
                 tie_embeddings: bool = True):
        super().__init__()
        self.embed = nn.Embedding(vocab, d_model)
        self.blocks = nn.ModuleList(
            RingAttentionBlock(d_model, n_heads, n_kv_heads, head_dim, mlp_mult, causal=True)
            for _ in range(n_layers))
        self.norm = RMSNorm(d_model)
        self.head = nn.Linear(d_model, vocab, bias=False)
        # small embeddings (std 0.02): with the default N(0, 1) and tied weights the
        # initial logits would have std ~sqrt(d_model) and the first losses would be
        # far above ln(vocab)
        nn.init.normal_(self.embed.weight, std=0.02)
        if tie_embeddings:
            self.head.weight = self.embed.weight

    def forward(self, ids: torch.Tensor, layout: RingLayout, rank: int = 0, group=None,
                backend: Optional[str] = None) -> torch.Tensor:
        """Logits [B, L, vocab] of the local shard."""
        x = self.embed(ids)
        for blk in self.blocks:
            x = blk(x, layout, rank, group=group, backend=backend)
        return self.head(self.norm(x))

    def loss(self, ids: torch.Tensor, targets: torch.Tensor, layout: RingLayout, rank: int = 0,
             group=None, backend: Optional[str] = None) -> torch.Tensor:
        """Mean next-token cross entropy over every real token of the sequence:
        this shard's summed loss divided by the token count of all shards."""
        import torch.distributed as dist
        logits = self(ids, layout, rank, group=group, backend=backend)
        local = F.cross_entropy(logits.float().flatten(0, 1), targets.flatten(),
                                ignore_index=IGNORE_INDEX, reduction="sum")
        count = (targets != IGNORE_INDEX).sum().to(torch.float32)
        if dist.is_initialized() and dist.get_world_size(group) > 1:
            count = count.clone()
            dist.all_reduce(count, group=group)
        return local / count.clamp(min=1.0)
