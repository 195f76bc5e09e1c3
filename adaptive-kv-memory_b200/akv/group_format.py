"""Per-token, per-D-group ("group format") tiers of the reference's older kernel API.

The reference's ``triton_ops`` / ``triton_kernels`` modules (and its
``KVQuantizer.QuantizedTensor``) store a quantised tier as packed byte rows
of N tokens x D channels (padded with zeros to whole groups), with one fp16
scale and zero per (token, group) (akv/triton_ops.py:657-715,
akv/triton_kernels.py:426-500).  This module runs that format on CUDA:

* ``group_dequantize``  codes -> fp16 (``akv_group_dequant``)
* ``group_quantize``    fp16 rows, optionally gathered by index -> codes
                        (``akv_group_quantize``)
* ``group_attention``   attention of (B, H, M, D) queries over an optional
                        per-row FP16 tier plus a group-format tier shared by
                        the batch and heads, on the split-K decode kernel
                        (query rows as the query heads of one KV head) and the
                        LSE combine, with the optional softmax weights of
                        every key (``akv_attention_probs``)
"""
from __future__ import annotations

import math
from typing import Optional

import torch

from . import _C
from .fused_attention import _pad_dim, kernel_head_dim, mixed_tier_decode_attention


def padded_dim(D: int, group_size: int) -> int:
    return -(-D // group_size) * group_size


def _fp16(t: torch.Tensor, what: str) -> torch.Tensor:
    if t.dtype != torch.float16:
        raise TypeError(f"{what} must be fp16 (got {t.dtype})")
    return t


def group_dequantize(packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, bits: int, group_size: int,
                     N: int, D: int, symmetric: Optional[bool] = None) -> torch.Tensor:
    """(N, D) fp16 from a group-format tier (the reference's ``_dequantize_packed``).

    ``packed`` holds N rows of padded_dim(D)*bits/8 bytes (any shape, read
    flat, as the reference does); scales / zeros (N, n_groups) fp16.
    ``symmetric`` None decides on the device, like the reference: the
    symmetric formula applies when every zero is 0."""
    _C.require_cuda(packed, scales, zeros)
    if bits not in (2, 4, 8):
        raise ValueError(f"Unsupported bits: {bits}")
    Dp = padded_dim(D, group_size)
    row = Dp * bits // 8
    flat = packed.reshape(-1)
    if flat.numel() < N * row:
        raise ValueError(f"packed tier holds {flat.numel()} bytes, {N * row} needed")
    ng = Dp // group_size
    s = _fp16(scales, "scales").reshape(N, ng)
    z = _fp16(zeros, "zeros").reshape(N, ng)
    if s.stride() != z.stride() or s.stride(-1) != 1:
        s, z = s.contiguous(), z.contiguous()
    if symmetric is None:
        sym = (z == 0).all().to(torch.int32)
    else:
        sym = torch.full((1,), int(bool(symmetric)), dtype=torch.int32, device=packed.device)
    Dk = -(-D // 8) * 8
    out = torch.empty(N, Dk, dtype=torch.float16, device=packed.device)
    rc = _C.load().akv_group_dequant(flat.data_ptr(), 0, row, s.data_ptr(), z.data_ptr(), 0, s.stride(0), 1, N, Dk,
                                     group_size, bits, sym.data_ptr(), out.data_ptr(), 0, out.stride(0),
                                     _C.stream_of(packed))
    _C.check(rc, "akv_group_dequant")
    return out[:, :D] if Dk != D else out


def group_quantize(x: torch.Tensor, bits: int = 4, group_size: int = 128, row_idx: Optional[torch.Tensor] = None,
                   status: Optional[torch.Tensor] = None):
    """Quantise fp16 rows x (n_src, D) (rows ``row_idx`` of it, if given) to the group format.

    Returns (packed (n, padded_D*bits/8) uint8, scales (n, n_groups) fp16,
    zeros (n, n_groups) fp16), the arithmetic of the reference's
    ``fused_quantize_evict`` (akv/triton_kernels.py:470-500)."""
    _C.require_cuda(x, row_idx)
    if bits not in (2, 4, 8):
        raise ValueError(f"Unsupported bits: {bits}")
    x = _fp16(x, "rows")
    if x.dim() != 2 or x.stride(-1) != 1:
        x = x.reshape(-1, x.shape[-1]).contiguous()
    n_src, D = x.shape
    idx = None
    if row_idx is not None:
        idx = row_idx.to(device=x.device, dtype=torch.int64).contiguous()
    n = n_src if idx is None else idx.numel()
    ng = -(-D // group_size)
    row = ng * group_size * bits // 8
    packed = torch.empty(n, row, dtype=torch.uint8, device=x.device)
    scales = torch.empty(n, ng, dtype=torch.float16, device=x.device)
    zeros = torch.empty_like(scales)
    rc = _C.load().akv_group_quantize(x.data_ptr(), x.stride(0), _C.ptr(idx), n_src, n, D, group_size, bits,
                                      packed.data_ptr(), row, scales.data_ptr(), zeros.data_ptr(), _C.ptr(status),
                                      _C.stream_of(x))
    _C.check(rc, "akv_group_quantize")
    return packed, scales, zeros


def _partial(q3, k, v, sm_scale, Hkv):
    """(B*Hq, Dp+2) split-K partial of q3 (B, Hq, Dp) over k / v (B, Hkv, N, Dp) (strides may be 0)."""
    p = torch.empty(q3.shape[0] * q3.shape[1], q3.shape[2] + 2, dtype=torch.float32, device=q3.device)
    mixed_tier_decode_attention(q3, k, v, sm_scale=sm_scale, partial_out=p)
    return p


def group_attention(query: torch.Tensor, hot_k: Optional[torch.Tensor], hot_v: Optional[torch.Tensor],
                    warm_k: Optional[torch.Tensor], warm_v: Optional[torch.Tensor],
                    sm_scale: Optional[float] = None, return_weights: bool = False):
    """softmax(q [K_hot; K_warm]^T * sm_scale) [V_hot; V_warm] for (B, H, M, D) queries.

    hot_k / hot_v: (B, H, N_hot, D) fp16 per batch row and head, or None;
    warm_k / warm_v: (N_warm, D) fp16 shared by every row and head, or None.
    No causal mask: every query sees every key, as in the reference.
    Returns (B, H, M, D) in the query's dtype, and with ``return_weights``
    the (B, H, M, N_hot + N_warm) fp32 softmax weights in [hot; warm] order."""
    _C.require_cuda(query, hot_k, hot_v, warm_k, warm_v)
    B, H, M, D = query.shape
    if not kernel_head_dim(D) or D % 8:
        raise ValueError(f"head_dim {D} unsupported (multiple of 8, at most 256)")
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    dev = query.device
    q = query.to(torch.float16)
    # query row (h, m) is query head h*M + m of KV head h: M query heads per KV head
    q3 = _pad_dim(q.reshape(B, H * M, D))
    parts = []
    n_hot = 0 if hot_k is None else hot_k.shape[2]
    n_warm = 0 if warm_k is None else warm_k.shape[0]
    if n_hot:
        hk, hv = _pad_dim(hot_k.to(torch.float16)), _pad_dim(hot_v.to(torch.float16))
        if hk.stride() != hv.stride():
            hk, hv = hk.contiguous(), hv.contiguous()
        parts.append(_partial(q3, hk, hv, sm_scale, H))
    if n_warm:
        wk, wv = _pad_dim(warm_k.to(torch.float16)), _pad_dim(warm_v.to(torch.float16))
        if wk.stride() != wv.stride():
            wk, wv = wk.contiguous(), wv.contiguous()
        # one tier shared by every batch row and head: strides 0
        parts.append(_partial(q3, wk.expand(B, H, n_warm, wk.shape[-1]), wv.expand(B, H, n_warm, wv.shape[-1]),
                              sm_scale, H))
    Dp = q3.shape[-1]
    rows = B * H * M
    out = torch.empty(rows, Dp, dtype=torch.float16, device=dev)
    lse = torch.empty(rows, dtype=torch.float32, device=dev)
    if not parts:
        out.zero_()
        lse.fill_(float("-inf"))
    else:
        part = torch.stack(parts, 1)  # (rows, splits, Dp+2)
        _C.check(_C.load().akv_lse_combine(part.data_ptr(), part.stride(1), part.stride(0), rows, part.shape[1], Dp,
                                           out.data_ptr(), out.stride(0), lse.data_ptr(), None, _C.stream_of(part)),
                 "akv_lse_combine")
    res = out[:, :D].reshape(B, H, M, D).to(query.dtype)
    if not return_weights:
        return res
    w = torch.empty(B, H, M, n_hot + n_warm, dtype=torch.float32, device=dev)
    lib = _C.load()
    if q.stride(-1) != 1:
        q = q.contiguous()
    qs = q.stride()
    if n_hot:
        k = hot_k.to(torch.float16)
        k = k if k.stride(-1) == 1 else k.contiguous()
        ks = k.stride()
        _C.check(lib.akv_attention_probs(q.data_ptr(), qs[0], qs[1], qs[2], k.data_ptr(), ks[0], ks[1], ks[2],
                                         lse.data_ptr(), B, H, M, n_hot, D, float(sm_scale), w.data_ptr(),
                                         w.stride(0), w.stride(1), w.stride(2), 0, _C.stream_of(q)),
                 "akv_attention_probs")
    if n_warm:
        k = warm_k.to(torch.float16)
        k = k if k.stride(-1) == 1 else k.contiguous()
        _C.check(lib.akv_attention_probs(q.data_ptr(), qs[0], qs[1], qs[2], k.data_ptr(), 0, 0, k.stride(0),
                                         lse.data_ptr(), B, H, M, n_warm, D, float(sm_scale), w.data_ptr(),
                                         w.stride(0), w.stride(1), w.stride(2), n_hot, _C.stream_of(q)),
                 "akv_attention_probs")
    return res, w
