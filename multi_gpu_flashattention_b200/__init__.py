"""B200-native ring attention.

Public API
----------
ring_attention(q, k, v, causal=False, group=None, layout="zigzag", ...)
    Context-parallel attention over a torch.distributed group; each rank holds
    its token shard of q, k, v ([batch, local_seq, heads, head_dim]).
flash_attn(q, k, v, causal=False, softmax_scale=None)
    Single-GPU attention on the sm_100a kernels (forward + backward).
sched
    Workload model, static schedulers and shard plans (C++).
"""
from .version import __version__  # noqa: F401
