"""Model building blocks that use ring attention."""
from .transformer import (IGNORE_INDEX, RingAttentionBlock, RingTransformerLM, RMSNorm,  # noqa: F401
                          rotary, shard_targets)
