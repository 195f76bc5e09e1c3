"""The reference's ``akv.triton_ops`` entry points, served by this package's CUDA kernels.

The reference implements these with Triton kernels and torch fallbacks
(akv/triton_ops.py:330-650).  Here the group-format tiers are dequantised by
``akv_group_dequant`` and attended by the split-K decode kernel with the LSE
combine (``akv.group_format``); no Triton code is involved.  ``HAS_TRITON``
keeps the reference's flag name so callers that branch on it take the fused
path: it is True whenever the CUDA library is present.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from . import _C
from .group_format import group_attention, group_dequantize
from .tiering import fused_importance_update

HAS_TRITON = os.path.exists(_C.LIB_PATH)

__all__ = ["HAS_TRITON", "fused_quantized_attention", "fused_mixed_precision_attention", "fused_importance_update"]


def fused_quantized_attention(query: torch.Tensor, key_packed: torch.Tensor, key_scales: torch.Tensor,
                              key_zeros: torch.Tensor, value_packed: torch.Tensor, value_scales: torch.Tensor,
                              value_zeros: torch.Tensor, bits: int = 4, group_size: int = 128,
                              sm_scale: Optional[float] = None) -> torch.Tensor:
    """(B, H, M, D) attention of every query over one group-format tier of
    N = key_scales.shape[0] tokens shared by the batch and heads (reference
    akv/triton_ops.py:330-376)."""
    D = query.shape[-1]
    N = key_scales.shape[0]
    k = group_dequantize(key_packed, key_scales, key_zeros, bits, group_size, N, D)
    v = group_dequantize(value_packed, value_scales, value_zeros, bits, group_size, N, D)
    return group_attention(query, None, None, k, v, sm_scale)


def fused_mixed_precision_attention(query: torch.Tensor, key_hot: torch.Tensor, value_hot: torch.Tensor,
                                    key_warm_packed: torch.Tensor, key_warm_scales: torch.Tensor,
                                    key_warm_zeros: torch.Tensor, value_warm_packed: torch.Tensor,
                                    value_warm_scales: torch.Tensor, value_warm_zeros: torch.Tensor,
                                    bits: int = 4, group_size: int = 128, sm_scale: Optional[float] = None):
    """Attention over the FP16 hot tier (B, H, N_hot, D) plus a group-format
    warm tier shared by the batch and heads (reference
    akv/triton_ops.py:466-515).  Returns (output (B, H, M, D), attention
    weights (B, H, M, N_hot + N_warm) fp32, hot columns first) — the weights
    feed importance scoring and promotion."""
    D = query.shape[-1]
    N_warm = key_warm_scales.shape[0]
    wk = wv = None
    if N_warm:
        wk = group_dequantize(key_warm_packed, key_warm_scales, key_warm_zeros, bits, group_size, N_warm, D)
        wv = group_dequantize(value_warm_packed, value_warm_scales, value_warm_zeros, bits, group_size, N_warm, D)
    return group_attention(query, key_hot, value_hot, wk, wv, sm_scale, return_weights=True)
