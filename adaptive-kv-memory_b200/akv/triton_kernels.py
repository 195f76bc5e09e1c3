"""The reference's ``akv.triton_kernels`` entry points, served by this package's CUDA kernels.

``fused_decode_attention`` (reference akv/triton_kernels.py:281-423) attends
a decode query over the FP16 hot tier plus a group-format warm tier;
``fused_quantize_evict`` (:426-500) gathers the tokens an eviction mask
selects and quantises them to the group format in one kernel
(``akv_group_quantize``).  No Triton code is involved.
"""
from __future__ import annotations

from typing import Optional

import torch

from .group_format import group_attention, group_dequantize, group_quantize

__all__ = ["fused_decode_attention", "fused_quantize_evict"]


def fused_decode_attention(query: torch.Tensor, key_hot: torch.Tensor, value_hot: torch.Tensor,
                           key_warm_packed: Optional[torch.Tensor] = None,
                           key_warm_scales: Optional[torch.Tensor] = None,
                           key_warm_zeros: Optional[torch.Tensor] = None,
                           value_warm_packed: Optional[torch.Tensor] = None,
                           value_warm_scales: Optional[torch.Tensor] = None,
                           value_warm_zeros: Optional[torch.Tensor] = None,
                           bits: int = 4, group_size: int = 128, sm_scale: Optional[float] = None) -> torch.Tensor:
    """(B, H, 1, D) decode attention over [hot; warm]; warm None = hot only."""
    D = query.shape[-1]
    wk = wv = None
    if key_warm_packed is not None and key_warm_scales is not None and key_warm_scales.shape[0] > 0:
        n = key_warm_scales.shape[0]
        wk = group_dequantize(key_warm_packed, key_warm_scales, key_warm_zeros, bits, group_size, n, D)
        wv = group_dequantize(value_warm_packed, value_warm_scales, value_warm_zeros, bits, group_size, n, D)
    return group_attention(query, key_hot, value_hot, wk, wv, sm_scale)


def fused_quantize_evict(keys: torch.Tensor, values: torch.Tensor, evict_mask: torch.Tensor, bits: int = 4,
                         group_size: int = 128):
    """Quantise the rows of keys / values (N, D) where ``evict_mask`` (N,) is
    True.  Returns (k_packed, k_scales, k_zeros, v_packed, v_scales, v_zeros);
    empty tensors when nothing is evicted."""
    idx = evict_mask.nonzero(as_tuple=True)[0]
    if idx.numel() == 0:
        empty = torch.empty(0, device=keys.device, dtype=torch.uint8)
        empty_f = torch.empty(0, device=keys.device, dtype=keys.dtype)
        return empty, empty_f, empty_f, empty, empty_f, empty_f
    kp, ks, kz = group_quantize(keys, bits, group_size, row_idx=idx)
    vp, vs, vz = group_quantize(values, bits, group_size, row_idx=idx)
    return kp, ks, kz, vp, vs, vz
