"""SigLIP-2 NaFlex vision tower forward on B200 (sm_100a).

The public modules mirror tohskai/SigLIP-2 (``model.py`` /
``optimized_siglip2``); their forwards call ``libsiglip2_b200.so`` through
its C ABI (``include/siglip2_b200.h``).  The kernels are also registered as
``torch.ops.siglip2_b200.*`` (``torch_ops``).
"""
from .model import (  # noqa: F401
    LayerNorm,
    LayerNormImproved,
    MLPImproved,
    Sequences,
    Siglip2Attention,
    Siglip2AttentionImproved,
    Siglip2Encoder,
    Siglip2EncoderImproved,
    Siglip2EncoderLayer,
    Siglip2EncoderLayerImproved,
    Siglip2MLP,
    Siglip2MultiheadAttentionPoolingHead,
    Siglip2Output,
    Siglip2SequenceEmbeddings,
    Siglip2SequenceEmbeddingsImproved,
    Siglip2SequenceVisionTransformer,
    Siglip2SequenceVisionTransformerOptimized,
    Siglip2VisionConfig,
    Siglip2VisionTransformer,
    create_document_ids,
)

__all__ = [
    "Siglip2VisionConfig",
    "Siglip2SequenceVisionTransformer",
    "Siglip2SequenceVisionTransformerOptimized",
    "Siglip2VisionTransformer",
    "Siglip2Output",
    "Siglip2SequenceEmbeddings",
    "Siglip2SequenceEmbeddingsImproved",
    "Siglip2Attention",
    "Siglip2AttentionImproved",
    "Siglip2MLP",
    "MLPImproved",
    "LayerNorm",
    "LayerNormImproved",
    "Siglip2EncoderLayer",
    "Siglip2EncoderLayerImproved",
    "Siglip2Encoder",
    "Siglip2EncoderImproved",
    "Siglip2MultiheadAttentionPoolingHead",
    "Sequences",
    "create_document_ids",
]
