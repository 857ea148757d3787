"""B200-native ring attention.

Public API
----------
ring_attention(q, k, v, causal=False, group=None, layout=None, ...)
    Context-parallel attention over a torch.distributed group; each rank holds
    its token shard of q, k, v ([batch, local_seq, heads, head_dim]).
RingLayout(kind, seq, world)
    contiguous / zigzag / striped / scheduler-driven token ownership.
flash_attn(q, k, v, causal=False, softmax_scale=None)
    Single-GPU attention on the sm_100a kernels (differentiable);
    flash_attn_fwd / flash_attn_bwd are the explicit passes.
GraphedAttention(q, k, v, causal=False, backward=False)
    The single-GPU passes captured into CUDA graphs for fixed shapes.
RingHealth, PeerLostError
    Liveness gate for ring calls (`ring_attention(..., health=RingHealth())`).
RingAttentionBlock, RingTransformerLM, shard_targets
    Model layer whose attention is the ring (models/).
"""
from .version import __version__  # noqa: F401
from .parallel.layouts import RingLayout, make_layout  # noqa: F401
from .parallel.api import ring_attention  # noqa: F401
from .parallel.health import PeerLostError, RingHealth  # noqa: F401
from .ops.flash import KernelStatusError, flash_attn, flash_attn_bwd, flash_attn_fwd  # noqa: F401
from .ops.graphs import GraphedAttention  # noqa: F401
from .models import RingAttentionBlock, RingTransformerLM, shard_targets  # noqa: F401
