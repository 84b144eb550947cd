"""SigLIP-2 NaFlex vision tower forward on B200 (sm_100a).

The public modules mirror tohskai/SigLIP-2 (``model.py`` /
``optimized_siglip2``); their forward calls ``libsiglip2_b200.so`` through
its C ABI (``include/siglip2_b200.h``).
"""
from .model import (  # noqa: F401
    Siglip2Attention,
    Siglip2Encoder,
    Siglip2EncoderLayer,
    Siglip2MLP,
    Siglip2MultiheadAttentionPoolingHead,
    Siglip2Output,
    Siglip2SequenceEmbeddings,
    Siglip2SequenceVisionTransformer,
    Siglip2SequenceVisionTransformerOptimized,
    Siglip2VisionConfig,
    Siglip2VisionTransformer,
)

__all__ = [
    "Siglip2VisionConfig",
    "Siglip2SequenceVisionTransformer",
    "Siglip2SequenceVisionTransformerOptimized",
    "Siglip2VisionTransformer",
    "Siglip2Output",
]
