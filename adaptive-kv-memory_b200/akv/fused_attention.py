"""Fused mixed-tier decode attention (CUDA).

``mixed_tier_decode_attention`` is the warm-tier hot path: one decode query
per sequence attends over the FP16 hot window and the packed warm tier
(``WarmArena`` block records) in one split-K kernel with an LSE combine
(``akv_mixed_decode`` in ``libakv_sm100.so``).  The warm tier is never
dequantised into memory.

``mixed_precision_decode_attention`` keeps the reference signature
(akv/fused_attention.py:324-366) for callers of the reference API.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _C

_workspaces: dict = {}


def _workspace(device: torch.device, nbytes: int) -> torch.Tensor:
    key = (device.type, device.index)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def mixed_tier_decode_attention(query: torch.Tensor,
                                hot_keys: Optional[torch.Tensor] = None,
                                hot_values: Optional[torch.Tensor] = None,
                                warm=None,
                                n_hot: Optional[int] = None,
                                sm_scale: Optional[float] = None,
                                hot_len: Optional[torch.Tensor] = None,
                                warm_len: Optional[torch.Tensor] = None,
                                return_lse: bool = False,
                                out: Optional[torch.Tensor] = None,
                                status: Optional[torch.Tensor] = None,
                                partial_out: Optional[torch.Tensor] = None):
    """softmax(q [K_warm; K_hot]^T * sm_scale) [V_warm; V_hot] for one query token.

    query:      (B, Hq, 1, D) or (B, Hq, D) fp16
    hot_keys:   (B, Hkv, >= n_hot, D) fp16 (last dim contiguous), or None
    warm:       a ``WarmArena`` (packed block records), or None
    n_hot:      hot tokens to read (default: hot_keys.shape[2])
    hot_len / warm_len: optional int32 (B,) per-row hot tokens / warm blocks
    Returns (B, Hq, 1, D) fp16 (same rank as ``query``), plus the natural-log
    LSE (B, Hq) fp32 when ``return_lse``.  ``partial_out`` (fp32 (B*Hq, D+2))
    additionally receives the (acc, m, l) partial record of these tokens for a
    cross-GPU sequence split (see ``akv.parallel``).
    """
    _C.require_cuda(query, hot_keys, hot_values)
    q3 = query.reshape(query.shape[0], query.shape[1], query.shape[-1]) if query.dim() == 4 else query
    if q3.stride(-1) != 1:
        q3 = q3.contiguous()
    B, Hq, D = q3.shape
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if hot_keys is not None:
        Hkv = hot_keys.shape[1]
        nh = hot_keys.shape[2] if n_hot is None else int(n_hot)
        if hot_keys.stride() != hot_values.stride():
            raise ValueError("hot keys and values must share strides")
        if hot_keys.stride(-1) != 1:
            raise ValueError("hot keys/values need a contiguous last dim")
    else:
        Hkv = warm.H if warm is not None else Hq
        nh = 0
    nwb = warm.n_blocks if warm is not None else 0
    if warm is not None and (warm.B != B or warm.H != Hkv or warm.D != D):
        raise ValueError("warm arena shape does not match the query / hot tier")
    lib = _C.load()
    need = lib.akv_decode_workspace_bytes(B, Hq, Hkv, D, nh, nwb)
    if need == 0:
        raise ValueError(f"unsupported decode shape B={B} Hq={Hq} Hkv={Hkv} D={D}")
    ws = _workspace(q3.device, need)
    o = out if out is not None else torch.empty(B, Hq, D, dtype=torch.float16, device=q3.device)
    lse = torch.empty(B, Hq, dtype=torch.float32, device=q3.device) if return_lse else None
    hk_ptr = hot_keys.data_ptr() if nh > 0 else None
    hv_ptr = hot_values.data_ptr() if nh > 0 else None
    hs = hot_keys.stride() if nh > 0 else (0, 0, 0, 1)
    layout = ctypes.byref(warm.layout) if warm is not None else None
    wptr = warm.buf.data_ptr() if warm is not None else None
    wsb = warm.buf.stride(0) if warm is not None else 0
    wsh = warm.buf.stride(1) if warm is not None else 0
    rc = lib.akv_mixed_decode(
        q3.data_ptr(), q3.stride(0), q3.stride(1),
        hk_ptr, hv_ptr, hs[0], hs[1], hs[2], nh, _C.ptr(hot_len),
        wptr, wsb, wsh, layout, nwb, _C.ptr(warm_len),
        B, Hq, Hkv, D, float(sm_scale),
        o.data_ptr(), o.stride(0), o.stride(1), _C.ptr(lse), _C.ptr(partial_out),
        ws.data_ptr(), ws.numel(), _C.ptr(status), _C.stream_of(q3))
    _C.check(rc, "akv_mixed_decode")
    res = o.unsqueeze(2) if query.dim() == 4 else o
    return (res, lse) if return_lse else res


def mixed_precision_decode_attention(query, hot_keys, hot_values,
                                     warm_k_packed=None, warm_k_scales=None, warm_k_zeros=None,
                                     warm_v_packed=None, warm_v_scales=None, warm_v_zeros=None,
                                     group_size: int = 128):
    """Reference-signature entry (akv/fused_attention.py:324-366).

    The hot-only form (no warm tier) runs through ``akv_mixed_decode``.  The
    reference's INT4 per-token-group warm layout is a different quantiser
    from the affine warm tier and is not supported by this build.
    """
    if warm_k_packed is not None and warm_k_packed.shape[1] > 0:
        raise NotImplementedError("INT4 per-token-group warm layout: use WarmArena + mixed_tier_decode_attention")
    return mixed_tier_decode_attention(query, hot_keys, hot_values)
