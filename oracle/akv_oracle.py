"""CPU oracle for the AKV warm-tier hot path.  TEST INFRASTRUCTURE ONLY.

This module is a numpy restatement of the reference package ``akv`` (v1.4.0)
arithmetic for the warm tier.  It exists so that the CUDA path can be checked
against the reference's algorithm on the same seeded inputs.  Only the test
suite, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline / reference
arm may import it; the product path (``akv`` package) never does.

Parity is pinned: every function here is checked against golden vectors that
``tests/golden/make_golden.py`` produced by calling the reference package
itself (``tests/test_oracle_golden.py``).

FP16 semantics.  The reference runs its quantiser on FP16 tensors with torch
CPU elementwise ops.  Each op widens both operands to fp32, computes, and
rounds the result back to fp16 (round-to-nearest-even).  For + - * / the
double rounding fp32 -> fp16 is innocuous (24 >= 2*11 + 2), so each op equals
the correctly rounded fp16 op.  ``_h`` below applies that rounding.
"""
from __future__ import annotations

import math

import numpy as np

F16 = np.float16
F32 = np.float32


def _h(x) -> np.ndarray:
    """Round an fp32 array to fp16 (RNE), like torch's per-op Half result.

    Overflow to +-inf is the expected IEEE result (e.g. 65504 - (-65504))."""
    with np.errstate(over="ignore", invalid="ignore"):
        return np.asarray(x, dtype=F32).astype(F16)


def _f(x) -> np.ndarray:
    return np.asarray(x).astype(F32)


# ---------------------------------------------------------------------------
# Bit packing — reference akv/bitpack.py
# ---------------------------------------------------------------------------

def pack_uint4(codes: np.ndarray) -> np.ndarray:
    """akv/bitpack.py:13-19 — even index -> high nibble, odd -> low nibble."""
    c = np.asarray(codes).astype(np.uint8)
    if c.shape[-1] % 2:
        c = np.concatenate([c, np.zeros(c.shape[:-1] + (1,), np.uint8)], -1)
    return (((c[..., 0::2] & 0x0F) << 4) | (c[..., 1::2] & 0x0F)).astype(np.uint8)


def unpack_uint4(packed: np.ndarray, orig_dim: int) -> np.ndarray:
    """akv/bitpack.py:22-30."""
    p = np.asarray(packed).astype(np.uint8)
    out = np.empty(p.shape[:-1] + (orig_dim,), np.uint8)
    out[..., 0::2] = ((p >> 4) & 0x0F)[..., : orig_dim // 2 + orig_dim % 2]
    out[..., 1::2] = (p & 0x0F)[..., : orig_dim // 2]
    return out


def pack_uint3(codes: np.ndarray) -> np.ndarray:
    """akv/bitpack.py:35-51 — 8 codes -> 24-bit word c0<<21|..|c7 -> 3 bytes big-endian."""
    c = np.asarray(codes).astype(np.int64) & 0x07
    if c.shape[-1] % 8:
        pad = 8 - c.shape[-1] % 8
        c = np.concatenate([c, np.zeros(c.shape[:-1] + (pad,), np.int64)], -1)
    g = c.reshape(c.shape[:-1] + (-1, 8))
    word = np.zeros(g.shape[:-1], np.int64)
    for j in range(8):
        word |= g[..., j] << (21 - 3 * j)
    out = np.stack([(word >> 16) & 0xFF, (word >> 8) & 0xFF, word & 0xFF], -1)
    return out.reshape(c.shape[:-1] + (-1,)).astype(np.uint8)


def unpack_uint3(packed: np.ndarray, orig_dim: int) -> np.ndarray:
    """akv/bitpack.py:54-68."""
    p = np.asarray(packed).astype(np.int64)
    k = p.shape[-1] // 3
    p = p.reshape(p.shape[:-1] + (k, 3))
    word = (p[..., 0] << 16) | (p[..., 1] << 8) | p[..., 2]
    out = np.stack([(word >> (21 - 3 * j)) & 0x7 for j in range(8)], -1)
    return out.reshape(out.shape[:-2] + (k * 8,))[..., :orig_dim].astype(np.uint8)


def pack_uint2(codes: np.ndarray) -> np.ndarray:
    """akv/bitpack.py:73-79 — 4 codes per byte, first code in the top bits."""
    c = np.asarray(codes).astype(np.uint8)
    if c.shape[-1] % 4:
        pad = 4 - c.shape[-1] % 4
        c = np.concatenate([c, np.zeros(c.shape[:-1] + (pad,), np.uint8)], -1)
    c = c & 0x03
    return ((c[..., 0::4] << 6) | (c[..., 1::4] << 4) | (c[..., 2::4] << 2) | c[..., 3::4]).astype(np.uint8)


def unpack_uint2(packed: np.ndarray, orig_dim: int) -> np.ndarray:
    """akv/bitpack.py:82-90 (orig_dim must be the padded width's multiple of 4)."""
    p = np.asarray(packed).astype(np.uint8)
    out = np.empty(p.shape[:-1] + (orig_dim,), np.uint8)
    out[..., 0::4] = (p >> 6) & 0x03
    out[..., 1::4] = (p >> 4) & 0x03
    out[..., 2::4] = (p >> 2) & 0x03
    out[..., 3::4] = p & 0x03
    return out


def pack(codes: np.ndarray, bits: int) -> np.ndarray:
    """akv/bitpack.py:95-103."""
    if bits == 4:
        return pack_uint4(codes)
    if bits == 3:
        return pack_uint3(codes)
    if bits == 2:
        return pack_uint2(codes)
    return np.asarray(codes)


def unpack(packed: np.ndarray, bits: int, orig_dim: int) -> np.ndarray:
    """akv/bitpack.py:106-114."""
    if bits == 4:
        return unpack_uint4(packed, orig_dim)
    if bits == 3:
        return unpack_uint3(packed, orig_dim)
    if bits == 2:
        return unpack_uint2(packed, orig_dim)
    return np.asarray(packed)


def packed_width(dim: int, bits: int) -> int:
    """Bytes per row after packing (right-padded to the pack group)."""
    if bits == 4:
        return (dim + 1) // 2
    if bits == 3:
        return (dim + 7) // 8 * 3
    if bits == 2:
        return (dim + 3) // 4
    return dim


# ---------------------------------------------------------------------------
# Block-affine quantiser — reference akv/affine_quantizer.py
# ---------------------------------------------------------------------------

def outlier_norm_sum(x16: np.ndarray) -> np.ndarray:
    """Sum over heads of the per-(head, channel) fp32 L2 norms over tokens: (D,).

    The reference's channel score is this sum divided by the head count
    (affine_quantizer.py:79 / :146); with heads sharded over GPUs each GPU
    contributes its heads' sum and the sums are all-reduced."""
    xf = _f(x16)
    norms = np.sqrt(np.sum(xf * xf, axis=1, dtype=F32)).astype(F32)  # (H, D)
    return np.sum(norms, axis=0, dtype=F32).astype(F32)


def _outlier_select(x16: np.ndarray, fraction: float, score_sum=None, score_heads: int = 0):
    """affine_quantizer.py:75-85 (keys) / :143-151 (values).

    Channel score = L2 norm over tokens (fp32) per (head, channel), then the
    mean over heads; top-n channels, largest first.  torch's CPU ``topk`` does
    not promise an order for equal scores; this restatement takes the lower
    channel index first.
    """
    D = x16.shape[-1]
    n = max(1, int(D * fraction))
    if score_sum is None:
        score = (outlier_norm_sum(x16) / F32(x16.shape[0])).astype(F32)
    else:  # scores over heads held elsewhere too (sharded heads)
        score = (np.asarray(score_sum, F32) / F32(score_heads)).astype(F32)
    idx = np.argsort(-score, kind="stable")[:n]
    data = x16[..., idx].astype(F16)
    x16 = x16.copy()
    x16[..., idx] = F16(0.0)
    return x16, idx.astype(np.int64), data


def _affine_codes(x16: np.ndarray, lo: np.ndarray, hi: np.ndarray, bits: int):
    """affine_quantizer.py:91-95 / :157-161, op by op in fp16.

    ``clamp(min=1e-8)`` is a no-op on fp16: 1e-8 is below fp16's smallest
    subnormal, so a zero range keeps scale == 0.  0/0 then gives NaN, which
    ``.to(uint8)`` turns into 0 on x86; x/0 for x > 0 gives inf -> clamp -> maxval.
    """
    maxval = (1 << bits) - 1
    with np.errstate(over="ignore", invalid="ignore"):
        scale = _h(_f(hi) - _f(lo))
    scale = _h(_f(scale) / F32(maxval))
    zero = lo.astype(F16)
    diff = _h(_f(x16) - _f(zero))
    with np.errstate(divide="ignore", invalid="ignore"):
        ratio = _h(_f(diff) / _f(scale))
    r = np.rint(_f(ratio))
    r = np.where(np.isnan(r), F32(0.0), np.clip(r, 0, maxval))
    return r.astype(np.uint8), scale, zero


def quantize_keys(k: np.ndarray, bits: int, outlier_fraction: float = 0.0, packed: bool = True,
                  score_sum=None, score_heads: int = 0) -> dict:
    """affine_quantizer.py:63-110 — per-(head, channel) min/max over the tokens of the call.

    k: (H, N, D) fp16.  Returns the reference's dict layout.
    """
    k16 = np.asarray(k).astype(F16)
    out = {}
    if outlier_fraction > 0:
        k16, idx, data = _outlier_select(k16, outlier_fraction, score_sum, score_heads)
        out["outlier_idx"] = idx
        out["outlier_data"] = data
    lo = k16.min(axis=1, keepdims=True)
    hi = k16.max(axis=1, keepdims=True)
    codes, scale, zero = _affine_codes(k16, lo, hi, bits)
    out.update(scale=scale, zero=zero, orig_dim=codes.shape[-1], bits=bits)
    out["codes"] = pack(codes, bits) if packed else codes
    return out


def quantize_values(v: np.ndarray, bits: int, outlier_fraction: float = 0.0, packed: bool = True,
                    score_sum=None, score_heads: int = 0) -> dict:
    """affine_quantizer.py:131-176 — per-(head, token) min/max over channels."""
    v16 = np.asarray(v).astype(F16)
    out = {}
    if outlier_fraction > 0:
        v16, idx, data = _outlier_select(v16, outlier_fraction, score_sum, score_heads)
        out["outlier_idx"] = idx
        out["outlier_data"] = data
    lo = v16.min(axis=2, keepdims=True)
    hi = v16.max(axis=2, keepdims=True)
    codes, scale, zero = _affine_codes(v16, lo, hi, bits)
    out.update(scale=scale, zero=zero, orig_dim=codes.shape[-1], bits=bits)
    out["codes"] = pack(codes, bits) if packed else codes
    return out


def _dequant(q: dict) -> np.ndarray:
    """affine_quantizer.py:112-124 / :178-189 — fp16 multiply, then fp16 add (no FMA)."""
    codes = np.asarray(q["codes"])
    if q["bits"] in (2, 3, 4) and codes.shape[-1] != q["orig_dim"]:  # packed=True layout
        codes = unpack(codes, q["bits"], q["orig_dim"])
    c = _f(codes.astype(F16))
    with np.errstate(invalid="ignore", over="ignore"):  # 0 * inf -> NaN, as in torch
        out = _h(_h(c * _f(q["scale"])).astype(F32) + _f(q["zero"]))
    if "outlier_idx" in q:
        out[..., q["outlier_idx"]] = q["outlier_data"]
    return out


dequantize_keys = _dequant
dequantize_values = _dequant


def measure_packed_bytes(q: dict, bits: int) -> int:
    """akv/packed_layout.py:501-543 — packed codes + scale + zero bytes.

    Outlier side-store bytes are NOT counted by the reference.
    """
    total = int(np.asarray(q["codes"]).nbytes)
    for key in ("scale", "zero"):
        if key in q:
            total += int(np.asarray(q[key]).nbytes)
    return total


def quantize_groups(x: np.ndarray, bits: int, group: int, is_key: bool,
                    outlier_fraction: float = 0.0) -> list:
    """Per batch row, per ``group``-token slice: one reference quantiser call each.

    The reference's ``AKVLayer`` quantises one demote event per call and
    breaks for batch > 1 (``drop_in.py:334``: ``squeeze(0)`` is a no-op), so
    the oracle for a (B, H, N, D) warm tier is one call per batch row and per
    token group.  Returns ``out[b][j]`` = the dict of group j of row b.
    """
    x = np.asarray(x).astype(F16)
    B, H, N, D = x.shape
    fn = quantize_keys if is_key else quantize_values
    res = []
    for b in range(B):
        row = []
        for j in range(0, N, group):
            row.append(fn(x[b, :, j:j + group], bits, outlier_fraction))
        res.append(row)
    return res


def dequantize_groups(groups: list) -> np.ndarray:
    """Inverse of ``quantize_groups``: (B, H, N, D) fp16."""
    rows = []
    for row in groups:
        rows.append(np.concatenate([_dequant(g) for g in row], axis=1))
    return np.stack(rows, 0)


# ---------------------------------------------------------------------------
# Attention — reference akv/fused_attention.py:324-366
# ---------------------------------------------------------------------------

def decode_attention(q: np.ndarray, keys: np.ndarray, values: np.ndarray,
                     sm_scale: float | None = None, return_lse: bool = False):
    """softmax(q.K^T * sm_scale).V in fp32 (fused_attention.py:362-366).

    q: (B, Hq, D); keys/values: (B, Hkv, N, D) fp16 (already dequantised warm
    tokens concatenated with the FP16 hot window — order does not matter for a
    single decode query).  Query head h reads KV head h // (Hq // Hkv), the
    HF ``repeat_kv`` mapping.  Returns fp32 (B, Hq, D) (and the natural-log LSE
    of the scaled logits when asked).
    """
    q = _f(q)
    B, Hq, D = q.shape
    Hkv = keys.shape[1]
    g = Hq // Hkv
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    kf = _f(keys)
    vf = _f(values)
    out = np.zeros((B, Hq, D), F32)
    lse = np.zeros((B, Hq), F32)
    for b in range(B):
        for h in range(Hq):
            kv = h // g
            s = (kf[b, kv] @ q[b, h]).astype(F32) * F32(sm_scale)
            if s.size == 0:
                continue
            m = s.max()
            p = np.exp(s - m)
            l = p.sum(dtype=F32)
            out[b, h] = (p / l) @ vf[b, kv]
            lse[b, h] = m + np.log(l)
    return (out, lse) if return_lse else out



def prefill_attention(q: np.ndarray, q_pos: np.ndarray, keys: np.ndarray, values: np.ndarray,
                      key_pos: np.ndarray, sm_scale: float | None = None) -> np.ndarray:
    """Causal attention by position in fp32: the SDPA the reference runs over
    AKVLayer's chronological FP16 view during prefill (akv/drop_in.py:753-787;
    the view holds every token once, in position order, so the causal mask of
    query i is "key position <= position of i").

    q: (B, Hq, M, D); q_pos: (B, M); keys/values: (B, Hkv, N, D) fp16 (the
    dequantised warm tokens and the hot tokens in any order); key_pos: (B, N)
    (a key with position > every query position is never seen).  GQA as in
    decode_attention.  A row that sees no key is zero.  Returns fp32 (B, Hq, M, D).
    """
    q = _f(q)
    B, Hq, M, D = q.shape
    Hkv = keys.shape[1]
    g = Hq // Hkv
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    kf = _f(keys)
    vf = _f(values)
    out = np.zeros((B, Hq, M, D), F32)
    for b in range(B):
        vis = key_pos[b][None, :] <= q_pos[b][:, None]  # (M, N)
        for h in range(Hq):
            kv = h // g
            s = (q[b, h] @ kf[b, kv].T).astype(F32) * F32(sm_scale)
            s = np.where(vis, s, -np.inf)
            m = s.max(axis=1, keepdims=True)
            m = np.where(np.isfinite(m), m, 0.0).astype(F32)
            p = np.exp(s - m)
            l = p.sum(axis=1, keepdims=True, dtype=F32)
            out[b, h] = np.where(l > 0, (p @ vf[b, kv]) / np.where(l > 0, l, 1.0), 0.0)
    return out


LOG2E = 1.4426950408889634


def decode_partial(q: np.ndarray, keys: np.ndarray, values: np.ndarray, sm_scale: float | None = None) -> np.ndarray:
    """Split-K partial record of one token range: (B*Hq, D+2) fp32 rows
    (acc[D] = sum_t 2^(x_t - m) v_t, m = max_t x_t, l = sum_t 2^(x_t - m)),
    x = q.k * sm_scale * log2(e); an empty range gives (0, -inf, 0).  This is
    the record ``akv_mixed_decode`` writes to ``partial_out``."""
    q = _f(q)
    B, Hq, D = q.shape
    Hkv = keys.shape[1]
    g = Hq // Hkv
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    kf, vf = _f(keys), _f(values)
    out = np.zeros((B * Hq, D + 2), F32)
    for b in range(B):
        for h in range(Hq):
            r = b * Hq + h
            if kf.shape[2] == 0:
                out[r, D] = -np.inf
                continue
            x = (kf[b, h // g] @ q[b, h]).astype(F32) * F32(sm_scale * LOG2E)
            m = x.max()
            p = np.exp2(x - m).astype(F32)
            out[r, :D] = p @ vf[b, h // g]
            out[r, D], out[r, D + 1] = m, p.sum(dtype=F32)
    return out


def lse_combine(part: np.ndarray) -> np.ndarray:
    """Merge split partial records (rows, splits, D+2) -> (rows, D) fp32 outputs."""
    part = np.asarray(part, F32)
    D = part.shape[-1] - 2
    m = part[..., D]
    M = m.max(axis=1, keepdims=True)
    Mb = np.where(np.isneginf(M), 0.0, M)
    w = np.exp2(m - Mb)  # (rows, splits)
    L = (part[..., D + 1] * w).sum(axis=1)
    acc = (part[..., :D] * w[..., None]).sum(axis=1)
    return np.where(L[:, None] > 0, acc / np.where(L[:, None] > 0, L[:, None], 1.0), 0.0).astype(F32)

def int4_group_dequant(packed: np.ndarray, scales: np.ndarray, zeros: np.ndarray,
                       head_dim: int, group_size: int) -> np.ndarray:
    """fused_attention.py:293-317 — INT4 (H, N, D/2) per-token per-D-group affine.

    fp32 ``c * s + z`` (two roundings), then one rounding to fp16.
    """
    p = np.asarray(packed).astype(np.uint8)
    H, N, _ = p.shape
    c = np.empty((H, N, head_dim), F32)
    c[..., 0::2] = ((p >> 4) & 0x0F).astype(F32)
    c[..., 1::2] = (p & 0x0F).astype(F32)
    gi = np.arange(head_dim) // group_size
    s = _f(scales)[:, :, gi]
    z = _f(zeros)[:, :, gi]
    return _h((c * s).astype(F32) + z)


# ---------------------------------------------------------------------------
# Group format: per token, per D-group, packed bytes (the kernel API of
# triton_ops / triton_kernels and KVQuantizer's QuantizedTensor)
# ---------------------------------------------------------------------------

def group_unpack(packed: np.ndarray, bits: int, count: int) -> np.ndarray:
    """triton_ops.py:672-686 / quantizer.py:221-243 — codes of a flat byte stream (MSB first)."""
    p = np.asarray(packed).astype(np.uint8).reshape(-1)
    if bits == 8:
        c = p
    elif bits == 4:
        c = np.stack([(p >> 4) & 15, p & 15], -1).reshape(-1)
    elif bits == 2:
        c = np.stack([(p >> 6) & 3, (p >> 4) & 3, (p >> 2) & 3, p & 3], -1).reshape(-1)
    else:
        raise ValueError(f"Unsupported bits: {bits}")
    return c[:count]


def group_pack(codes: np.ndarray, bits: int) -> np.ndarray:
    """quantizer.py:193-219 — flat codes -> bytes (MSB first, zero padded)."""
    c = np.asarray(codes).astype(np.uint8).reshape(-1)
    per = 8 // bits
    c = np.concatenate([c, np.zeros((-c.size) % per, np.uint8)]).reshape(-1, per)
    out = np.zeros(c.shape[0], np.uint8)
    for t in range(per):
        out |= (c[:, t] << (8 - bits * (t + 1))).astype(np.uint8)
    return out


def group_dequantize(packed: np.ndarray, scales: np.ndarray, zeros: np.ndarray, bits: int, group_size: int,
                     N: int, D: int) -> np.ndarray:
    """triton_ops.py:657-715 (``_dequantize_packed``) — (N, D) fp16.

    Rows are padded to whole groups; fp32 arithmetic: ``codes*s + z`` (two
    roundings) or, when every zero is 0, ``(codes - max//2) * s``; one
    rounding to fp16 at the end."""
    Dp = -(-D // group_size) * group_size
    c = group_unpack(packed, bits, N * Dp).astype(F32).reshape(N, -1, group_size)
    s = _f(scales).reshape(N, -1)[..., None]
    z = _f(zeros).reshape(N, -1)[..., None]
    if np.all(z == 0):
        out = ((c - F32(((1 << bits) - 1) // 2)) * s).astype(F32)
    else:
        out = ((c * s).astype(F32) + z).astype(F32)
    return _h(out.reshape(N, -1)[:, :D])


def group_quantize_fp16(x: np.ndarray, bits: int, group_size: int):
    """triton_kernels.py:470-500 (``fused_quantize_evict``'s quantiser) on
    fp16 rows (n, D): every half op is a float op rounded to fp16.  The
    ``clamp(min=1e-8)`` on the fp16 scale changes nothing (every positive
    fp16 exceeds 1e-8 and fp16(1e-8) is 0); a zero scale makes 0/0 = NaN,
    whose uint8 cast the reference leaves to the platform: 0 here.
    Returns (packed (n, Dp*bits/8), scales (n, ng) fp16, zeros (n, ng) fp16)."""
    x = np.asarray(x, F16)
    n, d = x.shape
    Dp = -(-d // group_size) * group_size
    xp = np.zeros((n, Dp), F16)
    xp[:, :d] = x
    g = xp.reshape(n, -1, group_size)
    mn, mx = g.min(-1), g.max(-1)
    maxint = (1 << bits) - 1
    scale = _h(_f(_h(_f(mx) - _f(mn))) / F32(maxint))
    with np.errstate(invalid="ignore", divide="ignore"):
        q = _f(_h(_f(_h(_f(g) - _f(mn)[..., None])) / _f(scale)[..., None]))
    q = np.rint(q)
    q = np.where(np.isnan(q), 0, np.clip(q, 0, maxint)).astype(np.uint8)
    packed = np.stack([group_pack(q[r], bits) for r in range(n)]) if n else np.zeros((0, Dp * bits // 8), np.uint8)
    return packed, scale, mn.astype(F16)


# ---------------------------------------------------------------------------
# Importance update and demote selection
# ---------------------------------------------------------------------------

def _cascade(rows: np.ndarray) -> np.ndarray:
    """Sum over axis 0 in torch's CPU cascade order (PyTorch
    aten/src/ATen/native/cpu/SumKernel.cpp, multi_row_sum): with
    lp = max(4, ceil(log2(R)) // 4) rows go one by one into level 0; after
    every 2^lp rows level 0 moves into level 1, at multiples of 2^(2lp) level
    1 into 2, at 2^(3lp) level 2 into 3; then levels 0 + 1 + 2 + 3."""
    R = rows.shape[0]
    lp = max(4, (int(math.ceil(math.log2(R))) if R > 1 else 0) // 4)
    step, mask = 1 << lp, (1 << lp) - 1
    acc = np.zeros((4,) + rows.shape[1:], F32)
    i = 0
    while i + step <= R:
        for _ in range(step):
            acc[0] = acc[0] + rows[i]
            i += 1
        for j in range(1, 4):
            acc[j] = acc[j] + acc[j - 1]
            acc[j - 1] = 0
            if i & (mask << (j * lp)):
                break
    while i < R:
        acc[0] = acc[0] + rows[i]
        i += 1
    out = acc[0]
    for j in range(1, 4):
        out = (out + acc[j]).astype(F32)
    return out.astype(F32)


def _cascade_ilp4(rows: np.ndarray) -> np.ndarray:
    """torch's row_sum: four interleaved cascades (rows 4i + k), the last
    R % 4 rows added to cascade 0, then cascades 1, 2, 3 added in order."""
    R = rows.shape[0]
    s = R // 4
    if s:
        p = np.stack([_cascade(rows[k:4 * s:4]) for k in range(4)])
    else:
        p = np.zeros((4,) + rows.shape[1:], F32)
    out = p[0]
    for i in range(4 * s, R):
        out = (out + rows[i]).astype(F32)
    for k in range(1, 4):
        out = (out + p[k]).astype(F32)
    return out


def torch_outer_sum(x: np.ndarray, vec_width: int = 16) -> np.ndarray:
    """torch.sum(x, dim=0) on the CPU for a contiguous fp32 (R, C) array,
    bit for bit: columns below the last multiple of 2*vec_width (torch sums
    them in blocks of four and two vector registers) in cascade order, the
    rest (one register's worth and the scalar tail) in the interleaved form.
    vec_width = floats per SIMD register (16 with AVX-512, 8 with AVX2)."""
    x = np.asarray(x, F32)
    R, C = x.shape
    jv = C // (2 * vec_width) * (2 * vec_width)
    out = np.empty(C, F32)
    if jv:
        out[:jv] = _cascade(x[:, :jv])
    if jv < C:
        out[jv:] = _cascade_ilp4(x[:, jv:])
    return out


def importance_update(attn: np.ndarray, scores: np.ndarray, decay: float, vec_width: int = 16) -> np.ndarray:
    """triton_ops.py:604-650 (CPU branch): scores*decay + sum_M mean_{B,H} attn.

    ``attention_weights.float().mean(dim=(0, 1)).sum(dim=0)`` in torch's CPU
    reduction order (``torch_outer_sum``; the mean is the sum divided by
    B*H), then two roundings (``mul_`` then ``add_``); the importance vector
    is truncated or zero-padded to len(scores) (:627-633).
    """
    a = _f(attn)
    B, H, M, N = a.shape
    tot = torch_outer_sum(a.reshape(B * H, M * N), vec_width).reshape(M, N)
    avg = (tot / F32(B * H)).astype(F32)
    imp = torch_outer_sum(avg, vec_width) if M > 1 else avg[0]
    n = scores.shape[0]
    if imp.shape[0] > n:
        imp = imp[:n]
    elif imp.shape[0] < n:
        imp = np.concatenate([imp, np.zeros(n - imp.shape[0], F32)])
    return ((_f(scores) * F32(decay)).astype(F32) + imp).astype(F32)


def select_demote(scores: np.ndarray, n_demote: int, hot_budget: int,
                  protect_initial: int = 4) -> np.ndarray:
    """drop_in.py:392-413 — bottom-k of scores with protected ends, sorted ascending.

    The first ``protect_initial`` and the last ``min(16, hot_budget // 4)``
    positions get +inf.  For equal scores this restatement takes the lower
    index first (torch's CPU topk leaves that order unspecified).
    """
    s = _f(scores).copy()
    n = s.shape[0]
    protect_recent = min(16, hot_budget // 4)
    s[:protect_initial] = np.inf
    s[max(0, n - protect_recent):] = np.inf
    order = np.argsort(s, kind="stable")[:n_demote]
    return np.sort(order).astype(np.int64)


def recency_decay(scores: np.ndarray, n_new: int, decay: float = 0.3) -> np.ndarray:
    """drop_in.py:376-390 — old scores * decay, new tokens at 1.0."""
    s = (_f(scores) * F32(decay)).astype(F32)
    return np.concatenate([s, np.ones(n_new, F32)])
