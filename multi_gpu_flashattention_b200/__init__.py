"""B200-native ring attention.

Public API
----------
ring_attention(q, k, v, causal=False, group=None, layout=None, ...)
    Context-parallel attention over a torch.distributed group; each rank holds
    its token shard of q, k, v ([batch, local_seq, heads, head_dim]).
RingLayout(kind, seq, world)
    contiguous / zigzag / striped / scheduler-driven token ownership.
flash_attn(q, k, v, causal=False, softmax_scale=None)
    Single-GPU attention on the sm_100a kernels.
"""
from .version import __version__  # noqa: F401
from .parallel.layouts import RingLayout, make_layout  # noqa: F401
from .parallel.api import ring_attention  # noqa: F401
from .ops.flash import flash_attn_fwd, KernelStatusError  # noqa: F401
