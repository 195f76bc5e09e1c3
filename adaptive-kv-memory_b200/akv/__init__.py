"""akv — B200-native warm tier of Adaptive KV Memory.

Block-affine quantise + bit-pack, packed warm block records, mixed-tier
(FP16 hot + packed warm) split-K decode attention and tensor-core prefill
attention, importance update and
demote/promote, behind the reference package's Python API.  Every op runs in
the sm_100a library ``akv/_lib/libakv_sm100.so``; there is no CPU fallback.
"""
from . import _C
from .affine_quantizer import AffineQuantConfig, AffineQuantizer
from .bitpack import pack, unpack, packed_bytes
from .fused_attention import (fused_int4_decode_attention, int4_group_dequant, mixed_precision_decode_attention,
                              mixed_tier_decode_attention, prefill_attention)
from .packed_layout import WarmArena, measure_packed_bytes
from .drop_in import AKVCache, AKVLayer, recommend_preset
from .graphs import DecodeGraph
from .tiering import fused_importance_update
from .triton_ops import HAS_TRITON, fused_mixed_precision_attention, fused_quantized_attention
from .triton_kernels import fused_decode_attention, fused_quantize_evict

__version__ = "0.1.0"

__all__ = [
    "AKVCache", "AKVLayer", "recommend_preset", "DecodeGraph",
    "AffineQuantConfig", "AffineQuantizer", "WarmArena", "measure_packed_bytes",
    "mixed_tier_decode_attention", "mixed_precision_decode_attention", "fused_int4_decode_attention",
    "int4_group_dequant", "prefill_attention",
    "HAS_TRITON", "fused_quantized_attention", "fused_mixed_precision_attention", "fused_importance_update",
    "fused_decode_attention", "fused_quantize_evict",
    "pack", "unpack", "packed_bytes",
]
