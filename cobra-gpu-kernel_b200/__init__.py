"""cobra-gpu-kernel_b200: the reference's single transformer-layer forward on B200.

Public API (mirrors dalberrt/COBRA-GPU-Kernel's drop-in module):
    TransformerConfig, B200TransformerLayer, SelfAttentionWeights
    ShardedLayer / sharded_forward: the layer split by batch over one process per GPU
    HeadShardedLayer / head_sharded_forward: split by head, for batches smaller than the GPU count
    B200Transformer (= UserOptimizedTransformer): the full stack, blocks with the GELU FFN
Native boundary: ``include/cobra_b200.h`` (ctypes binding in ``_lib``).
"""

from .layer import B200TransformerLayer, SelfAttentionWeights, TransformerConfig  # noqa: F401
from . import _lib  # noqa: F401
from .sharding import ShardedLayer, batch_shards, sharded_forward  # noqa: F401
from .headshard import HeadShardedLayer, head_sharded_forward, head_shards  # noqa: F401
from .model import B200Transformer, B200TransformerBlock, UserOptimizedTransformer  # noqa: F401

__all__ = ["B200TransformerLayer", "SelfAttentionWeights", "TransformerConfig",
           "ShardedLayer", "batch_shards", "sharded_forward",
           "HeadShardedLayer", "head_sharded_forward", "head_shards",
           "B200Transformer", "B200TransformerBlock", "UserOptimizedTransformer"]
