"""Fused mixed-tier decode attention (CUDA).

``mixed_tier_decode_attention`` is the warm-tier hot path: one decode query
per sequence attends over the FP16 hot window and the packed warm tier
(``WarmArena`` block records) in one split-K kernel with an LSE combine
(``akv_mixed_decode`` in ``libakv_sm100.so``).  The warm tier is never
dequantised into memory.

``mixed_precision_decode_attention`` and ``fused_int4_decode_attention``
keep the reference signatures (akv/fused_attention.py:213-366) on the
reference's INT4 per-token-group warm layout: the layout is dequantised by a
CUDA kernel and attended by the same decode kernel, hot and warm partials
merged by the LSE combine.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _C

_workspaces: dict = {}
KERNEL_HEAD_DIMS = (64, 128, 256)  # head dims the decode kernel is built for
KERNEL_HEAD_DIM = 128  # the prefill kernel's head dim


def kernel_head_dim(D: int) -> int:
    """The smallest decode-kernel head dim >= D (0 when D is larger than all)."""
    for d in KERNEL_HEAD_DIMS:
        if D <= d:
            return d
    return 0


def _pad_dim(x: torch.Tensor, d: Optional[int] = None) -> torch.Tensor:
    """Zero-pad the last dim to d (default: the next decode-kernel head dim):
    padded channels add 0 to every q.k and give all-zero output columns."""
    if d is None:
        d = kernel_head_dim(x.shape[-1]) or x.shape[-1]
    if x.shape[-1] == d:
        return x
    out = torch.zeros(*x.shape[:-1], d, dtype=x.dtype, device=x.device)
    out[..., : x.shape[-1]] = x
    return out


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
    if (D not in KERNEL_HEAD_DIMS and kernel_head_dim(D) and D % 8 == 0 and warm is None and partial_out is None
            and out is None):
        nh = hot_keys.shape[2] if n_hot is None else int(n_hot)
        res = mixed_tier_decode_attention(_pad_dim(q3), _pad_dim(hot_keys[:, :, :nh]), _pad_dim(hot_values[:, :, :nh]),
                                          None, nh, sm_scale, hot_len, None, return_lse, None, status, None)
        o, lse = res if return_lse else (res, None)
        o = o[..., :D]
        o = o.unsqueeze(2) if query.dim() == 4 else o
        return (o, lse) if return_lse else o
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
    need = _C.workspace_bytes("akv_decode_workspace_bytes", B, Hq, Hkv, D, nh, nwb)
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


def int4_group_dequant(packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor, head_dim: int,
                       group_size: int, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """The reference's ``_dequant_int4_tile`` (akv/fused_attention.py:293-317) on CUDA: (H, N, D) fp16."""
    _C.require_cuda(packed, scales, zeros)
    H, N, _ = packed.shape
    if scales.dtype != torch.float16 or zeros.dtype != torch.float16:
        raise TypeError("INT4 scales / zeros are fp16")
    if scales.stride() != zeros.stride() or scales.stride(-1) != 1 or packed.stride(-1) != 1:
        raise ValueError("scales and zeros need equal strides and a contiguous last dim; packed rows contiguous")
    if out is None:
        out = torch.empty(H, N, head_dim, dtype=torch.float16, device=packed.device)
    rc = _C.load().akv_int4_group_dequant(packed.data_ptr(), packed.stride(0), packed.stride(1),
                                          scales.data_ptr(), zeros.data_ptr(), scales.stride(0), scales.stride(1),
                                          H, N, head_dim, group_size, out.data_ptr(), out.stride(0), out.stride(1),
                                          _C.stream_of(packed))
    _C.check(rc, "akv_int4_group_dequant")
    return out


def _int4_partials(query, packed_k, ks, kz, packed_v, vs, vz, group_size, sm_scale, tile_tokens, parts):
    """Partial records of the shared INT4 warm tier, dequantised one bounded tile at a time."""
    B, H, Dp = query.shape  # query already padded to the kernel head dim
    D = 2 * packed_k.shape[2]
    N = packed_k.shape[1]
    tile = max(32, min(N, tile_tokens))
    kbuf = torch.zeros(H, tile, Dp, dtype=torch.float16, device=query.device)
    vbuf = torch.zeros_like(kbuf)
    for t0 in range(0, N, tile):
        n = min(tile, N - t0)
        int4_group_dequant(packed_k[:, t0:t0 + n], ks[:, t0:t0 + n], kz[:, t0:t0 + n], D, group_size,
                           out=kbuf[:, :n, :D])
        int4_group_dequant(packed_v[:, t0:t0 + n], vs[:, t0:t0 + n], vz[:, t0:t0 + n], D, group_size,
                           out=vbuf[:, :n, :D])
        k, v = kbuf[:, :n], vbuf[:, :n]
        p = torch.empty(B * H, Dp + 2, dtype=torch.float32, device=query.device)
        # the tier is shared by every batch row: batch stride 0
        mixed_tier_decode_attention(query, k.unsqueeze(0).expand(B, -1, -1, -1),
                                    v.unsqueeze(0).expand(B, -1, -1, -1), n_hot=n, sm_scale=sm_scale,
                                    partial_out=p)
        parts.append(p)


def _combine(parts, B, H, D, device) -> torch.Tensor:
    part = torch.stack(parts, 1).contiguous()  # (B*H, splits, D+2)
    out = torch.empty(B, H, D, dtype=torch.float16, device=device)
    rc = _C.load().akv_lse_combine(part.data_ptr(), D + 2, part.stride(0), B * H, part.shape[1], D,
                                   out.data_ptr(), D, None, None, _C.stream_of(part))
    _C.check(rc, "akv_lse_combine")
    return out


def fused_int4_decode_attention(query: torch.Tensor, k_packed: torch.Tensor, k_scales: torch.Tensor,
                                k_zeros: torch.Tensor, v_packed: torch.Tensor, v_scales: torch.Tensor,
                                v_zeros: torch.Tensor, group_size: int = 128,
                                memory_limit_mb: float = 512.0) -> torch.Tensor:
    """Reference signature (akv/fused_attention.py:213-290): attention of (B, H, 1, D) queries over one
    INT4 tier (H, N, D/2) shared by the batch.  The tier is dequantised by the CUDA kernel in tiles of at
    most ``memory_limit_mb`` (K + V fp16), each tile runs through the split-K decode kernel, and the
    tiles' partials are merged by the LSE combine.  Returns (B, H, 1, D) fp16."""
    _C.require_cuda(query, k_packed, v_packed)
    B, H, _, D = query.shape
    q = _pad_dim(query.reshape(B, H, D))
    tile = int(memory_limit_mb * 1e6 // (2 * H * D * 2))
    parts: list = []
    _int4_partials(q, k_packed, k_scales, k_zeros, v_packed, v_scales, v_zeros, group_size,
                   1.0 / math.sqrt(D), tile, parts)
    return _combine(parts, B, H, q.shape[-1], q.device)[..., :D].unsqueeze(2)


def mixed_precision_decode_attention(query, hot_keys, hot_values,
                                     warm_k_packed=None, warm_k_scales=None, warm_k_zeros=None,
                                     warm_v_packed=None, warm_v_scales=None, warm_v_zeros=None,
                                     group_size: int = 128):
    """Reference signature (akv/fused_attention.py:324-366): (B, H, 1, D) queries over the per-row FP16
    hot tier (B, H, N_hot, D) plus an optional INT4 warm tier (H, N_warm, D/2) shared by the batch.
    Hot and warm each give a split-K partial record; the LSE combine merges them.  Returns (B, H, 1, D)."""
    if warm_k_packed is None or warm_k_packed.shape[1] == 0:
        return mixed_tier_decode_attention(query, hot_keys, hot_values)
    _C.require_cuda(query, hot_keys, hot_values, warm_k_packed)
    B, H, _, D = query.shape
    q = _pad_dim(query.reshape(B, H, D))
    Dp = q.shape[-1]
    sm_scale = 1.0 / math.sqrt(D)
    parts: list = []
    if hot_keys is not None and hot_keys.shape[2] > 0:
        p = torch.empty(B * H, Dp + 2, dtype=torch.float32, device=q.device)
        mixed_tier_decode_attention(q, _pad_dim(hot_keys), _pad_dim(hot_values), sm_scale=sm_scale, partial_out=p)
        parts.append(p)
    _int4_partials(q, warm_k_packed, warm_k_scales, warm_k_zeros, warm_v_packed, warm_v_scales, warm_v_zeros,
                   group_size, sm_scale, warm_k_packed.shape[1], parts)
    return _combine(parts, B, H, Dp, q.device)[..., :D].unsqueeze(2)


def prefill_attention(query: torch.Tensor, q_pos: torch.Tensor,
                      hot_keys: Optional[torch.Tensor] = None, hot_values: Optional[torch.Tensor] = None,
                      hot_pos: Optional[torch.Tensor] = None, warm=None, warm_pos: Optional[torch.Tensor] = None,
                      sm_scale: Optional[float] = None, out: Optional[torch.Tensor] = None,
                      return_lse: bool = False, status: Optional[torch.Tensor] = None):
    """Causal attention of many query tokens over the FP16 hot tier and the packed warm tier.

    The prefill attention the reference runs with SDPA over ``AKVLayer``'s
    chronological FP16 view (akv/drop_in.py:753-787), on the tcgen05 tensor
    cores (``akv_prefill_attention``): query token m sees key token j iff
    ``pos(j) <= q_pos[m]``; warm records are dequantised exactly like the
    reference inside the kernel, never written back to memory.

    query:      (B, Hq, M, D) fp16, D = 128
    q_pos:      (B, M) or (M,) int32 query positions
    hot_keys:   (B, Hkv, N_hot, D) fp16 and hot_pos (B, N_hot) or (N_hot,) int32
    warm:       a ``WarmArena``; warm_pos (B, n_blocks*32) or (n_blocks*32,) int32
                positions of the record slots (slots with a clear mask bit are skipped)
    Returns (B, Hq, M, D) fp16 (and the natural-log LSE (B, Hq, M) fp32).
    """
    _C.require_cuda(query, hot_keys, hot_values)
    B, Hq, M, D = query.shape
    if query.stride(-1) != 1:
        query = query.contiguous()
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    dev = query.device

    def pos2(p, n):
        p = p.to(device=dev, dtype=torch.int32)
        p = p.unsqueeze(0).expand(B, n) if p.dim() == 1 else p
        if p.stride(-1) != 1:
            p = p.contiguous()
        return p

    qp = pos2(q_pos, M)
    nh = 0 if hot_keys is None else hot_keys.shape[2]
    if nh:
        Hkv = hot_keys.shape[1]
        if hot_keys.stride() != hot_values.stride() or hot_keys.stride(-1) != 1:
            raise ValueError("hot keys / values need equal strides and a contiguous last dim")
        hp = pos2(hot_pos, nh)
    else:
        Hkv = warm.H if warm is not None else Hq
        hp = None
    nwb = warm.n_blocks if warm is not None else 0
    wp = pos2(warm_pos, nwb * _C.BLOCK_TOKENS) if nwb else None
    if warm is not None and (warm.B != B or warm.H != Hkv or warm.D != D):
        raise ValueError("warm arena shape does not match the query / hot tier")
    o = out if out is not None else torch.empty(B, Hq, M, D, dtype=torch.float16, device=dev)
    lse = torch.empty(B, Hq, M, dtype=torch.float32, device=dev) if return_lse else None
    hs = hot_keys.stride() if nh else (0, 0, 0, 1)
    rc = _C.load().akv_prefill_attention(
        query.data_ptr(), query.stride(0), query.stride(1), query.stride(2), qp.data_ptr(), qp.stride(0), M,
        hot_keys.data_ptr() if nh else None, hot_values.data_ptr() if nh else None, hs[0], hs[1], hs[2], nh,
        hp.data_ptr() if nh else None, hp.stride(0) if nh else 0,
        warm.buf.data_ptr() if nwb else None, warm.buf.stride(0) if nwb else 0, warm.buf.stride(1) if nwb else 0,
        ctypes.byref(warm.layout) if nwb else None, nwb, wp.data_ptr() if nwb else None, wp.stride(0) if nwb else 0,
        B, Hq, Hkv, D, float(sm_scale), o.data_ptr(), o.stride(0), o.stride(1), o.stride(2), _C.ptr(lse),
        _C.ptr(status), _C.stream_of(query))
    _C.check(rc, "akv_prefill_attention")
    return (o, lse) if return_lse else o


# ---------------------------------------------------------------------------- compatibility entry points
def _dequantize_any(qt, quantizer) -> torch.Tensor:
    """A group-format quantised tensor (the reference's ``QuantizedTensor``
    fields: data, scales, zeros, shape, bits, group_size) dequantised by the
    CUDA kernel; anything else through ``quantizer.dequantize``."""
    fields = ("data", "scales", "zeros", "shape", "bits", "group_size")
    if all(hasattr(qt, f) for f in fields) and qt.data.is_cuda:
        from .group_format import group_dequantize
        shape = tuple(qt.shape)
        rows = int(math.prod(shape[:-1]))
        return group_dequantize(qt.data, qt.scales, qt.zeros, qt.bits, qt.group_size, rows, shape[-1]).reshape(shape)
    return quantizer.dequantize(qt)


def fused_decode_attention(query: torch.Tensor, keys_quantized, values_quantized, quantizer) -> torch.Tensor:
    """Reference compatibility wrapper (akv/fused_attention.py:373-390):
    decode attention of (B, H, 1, D) queries over quantised K / V of shape
    (B, H, N, D).  The tiers are dequantised (on CUDA for the group format)
    and attended by the decode kernel as one FP16 tier."""
    k = _dequantize_any(keys_quantized, quantizer).to(torch.float16)
    v = _dequantize_any(values_quantized, quantizer).to(torch.float16)
    B, H, _, D = query.shape
    if k.stride(-1) != 1 or k.stride() != v.stride():
        k, v = k.contiguous(), v.contiguous()
    out = mixed_tier_decode_attention(query.to(torch.float16), k, v, sm_scale=1.0 / math.sqrt(D))
    return out.to(query.dtype)


def fused_quantize_evict(keys: torch.Tensor, values: torch.Tensor, scores, evict_mask: torch.Tensor, quantizer):
    """Reference compatibility wrapper (akv/fused_attention.py:393-401): the
    tokens (dim 2 of (B, H, N, D) keys / values) where ``evict_mask`` is True,
    gathered by the row-gather kernel and passed to ``quantizer.quantize``.
    Returns (quantised keys, quantised values), or (None, None)."""
    from .tiering import gather_rows
    idx = evict_mask.nonzero(as_tuple=True)[0]
    if idx.numel() == 0:
        return None, None
    k_evict = gather_rows(keys, idx)
    v_evict = gather_rows(values, idx)
    return quantizer.quantize(k_evict), quantizer.quantize(v_evict)
