"""Model building blocks that use ring attention."""
from .transformer import RingAttentionBlock, RMSNorm, rotary  # noqa: F401
