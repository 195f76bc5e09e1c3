"""Paged warm pool: block records of many sequences in one buffer.

A page is the records of one 32-token block for every KV head of one
sequence: ``buf`` is ``(n_pages, Hkv, rec)`` uint8, so the record of KV head
h on page p starts at ``buf + (p * Hkv + h) * rec``.  Each sequence owns an
ordered list of pages (its block table row); pages come from a free list and
go back to it when the sequence ends, so sequences of any length share one
pool without per-sequence capacity.  ``paged_decode_attention`` runs the
mixed-tier decode over a batch of sequences through their block tables
(``akv_mixed_decode_paged``): one launch for the whole batch, whatever the
pages' order in the pool.

Quantisation writes straight into the pages when they form one ascending
run; otherwise into a staging buffer whose rows are then copied to the pages
(one ``index_copy_`` on the device).
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional, Sequence

import torch

from . import _C
from .affine_quantizer import n_outliers
from .packed_layout import BLOCK, record_dest

_workspaces: dict = {}


class PagedWarmPool:
    """``n_pages`` pages of block records for ``kv_heads`` heads."""

    def __init__(self, n_pages: int, kv_heads: int, head_dim: int, key_bits: int, value_bits: int,
                 outlier_fraction: float = 0.0, device="cuda"):
        self.H, self.D = kv_heads, head_dim
        self.key_bits, self.value_bits = key_bits, value_bits
        self.n_out = n_outliers(head_dim, outlier_fraction)
        self.layout = _C.warm_layout(head_dim, key_bits, value_bits, self.n_out)
        self.rec = self.layout.bytes
        self.n_pages = n_pages
        self.buf = torch.zeros(n_pages, kv_heads, self.rec, dtype=torch.uint8, device=device)
        self._free = list(range(n_pages - 1, -1, -1))  # pop() hands out ascending pages

    @property
    def device(self):
        return self.buf.device

    @property
    def free_pages(self) -> int:
        return len(self._free)

    def alloc(self, n: int) -> list:
        if n > len(self._free):
            raise RuntimeError(f"paged warm pool exhausted ({n} pages wanted, {len(self._free)} free)")
        return [self._free.pop() for _ in range(n)]

    def release(self, pages: Sequence[int]) -> None:
        self._free.extend(sorted(pages, reverse=True))

    def write(self, k: torch.Tensor, v: torch.Tensor, pages: Sequence[int], group: int = BLOCK,
              status: Optional[torch.Tensor] = None, tok_idx: Optional[torch.Tensor] = None) -> None:
        """Quantise (1, H, N, D) fp16 K/V (any strides, last dim contiguous)
        into ``pages`` (ceil(N / 32) of them, block j -> pages[j]); ``group``
        tokens share one K scale (32: one per block).  ``tok_idx`` (int64
        device, n entries): the rows of k / v to take, in that order (the
        quantiser gathers them; N is then n and k / v's third dim is the
        source's row count)."""
        _C.require_cuda(k, v)
        _, H, N, D = k.shape
        n_src = N
        if tok_idx is not None:
            N = tok_idx.numel()
        nblk = (N + BLOCK - 1) // BLOCK
        if (H, D) != (self.H, self.D) or len(pages) != nblk or k.shape[0] != 1:
            raise ValueError("K/V shape or page count does not match the pool")
        run = all(pages[i] == pages[0] + i for i in range(nblk))
        if run:
            target, base = None, self.buf[pages[0]].data_ptr()
        else:
            # zeroed: the unused slots of a partial block must decode to finite
            # values (their weight is 0, and 0 * NaN would poison the output)
            target = torch.zeros(nblk, H, self.rec, dtype=torch.uint8, device=self.device)
            base = target.data_ptr()
        sp = None if status is None else status.data_ptr()
        for x, is_key, bits in ((k, True, self.key_bits), (v, False, self.value_bits)):
            if x.stride(-1) != 1:
                x = x.contiguous()
            dest = record_dest(self.layout, base, 0, self.rec, H * self.rec, is_key)
            _C.quantize(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2),
                        None if tok_idx is None else tok_idx.data_ptr(), 0,
                        1, H, N, D, bits, is_key, min(group, N), self.n_out, dest, sp, x.device,
                        n_src=n_src if tok_idx is not None else 0)
        if target is not None:
            idx = torch.tensor(pages, dtype=torch.int64).pin_memory().to(self.device, non_blocking=True)
            self.buf.index_copy_(0, idx, target)

    def dequantize(self, pages: Sequence[int], n_tokens: Optional[int] = None) -> tuple:
        """FP16 (1, H, N, D) K and V of the blocks on ``pages`` in order (the
        first ``n_tokens`` slots; masked-out slots are returned as decoded)."""
        N = len(pages) * BLOCK if n_tokens is None else n_tokens
        lib = _C.load()
        # akv_dequantize addresses (b, h, blk, slot): one call per run of
        # consecutive pages, token t of the run in block t // 32 of the run
        outs = [torch.empty(1, self.H, N, self.D, dtype=torch.float16, device=self.device) for _ in range(2)]
        t0 = 0
        while t0 < N:
            j = t0 // BLOCK
            j1 = j + 1
            while j1 < len(pages) and pages[j1] == pages[j1 - 1] + 1:
                j1 += 1
            t1 = min(N, j1 * BLOCK)
            base = self.buf[pages[j]].data_ptr()
            for o, (is_key, bits) in zip(outs, ((True, self.key_bits), (False, self.value_bits))):
                src = record_dest(self.layout, base, 0, self.rec, self.H * self.rec, is_key)
                view = o[:, :, t0:t1]
                rc = lib.akv_dequantize(ctypes.byref(src), None, 0, 0, 1, self.H, t1 - t0, self.D, bits,
                                        int(is_key), self.n_out, view.data_ptr(), view.stride(0), view.stride(1),
                                        view.stride(2), None, _C.stream_of(self.buf))
                _C.check(rc, "akv_dequantize")
            t0 = t1
        return tuple(outs)

    def resident_bytes(self) -> int:
        return self.buf.numel()


def paged_decode_attention(query: torch.Tensor, hot_keys: Optional[torch.Tensor], hot_values: Optional[torch.Tensor],
                           hot_len: Optional[torch.Tensor], pool: PagedWarmPool, block_table: torch.Tensor,
                           warm_len: torch.Tensor, sm_scale: Optional[float] = None,
                           out: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode attention of one query per row over its hot tier and its paged warm blocks.

    query (B, Hq, D) fp16; hot_keys / hot_values (B, Hkv, >= max hot, D) fp16
    with per-row ``hot_len`` int32 (B,); block_table int32 (B, max_blocks):
    row b's warm block j is page block_table[b, j] for j < warm_len[b].
    Returns (B, Hq, D) fp16."""
    _C.require_cuda(query, block_table, warm_len)
    q3 = query if query.stride(-1) == 1 else query.contiguous()
    B, Hq, D = q3.shape
    Hkv = pool.H
    if sm_scale is None:
        sm_scale = 1.0 / math.sqrt(D)
    if block_table.dtype != torch.int32 or warm_len.dtype != torch.int32 or block_table.stride(-1) != 1:
        raise ValueError("block_table and warm_len must be int32 (block_table rows contiguous)")
    max_blocks = block_table.shape[1]
    nh = 0 if hot_keys is None else hot_keys.shape[2]
    lib = _C.load()
    need = _C.workspace_bytes("akv_decode_workspace_bytes", B, Hq, Hkv, D, nh, max_blocks)
    if need == 0:
        raise ValueError(f"unsupported decode shape B={B} Hq={Hq} Hkv={Hkv} D={D}")
    key = (q3.device.type, q3.device.index)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < need:
        ws = _workspaces[key] = torch.empty(max(need, 1 << 20), dtype=torch.uint8, device=q3.device)
    o = out if out is not None else torch.empty(B, Hq, D, dtype=torch.float16, device=q3.device)
    hs = hot_keys.stride() if nh else (0, 0, 0, 1)
    rc = lib.akv_mixed_decode_paged(
        q3.data_ptr(), q3.stride(0), q3.stride(1),
        hot_keys.data_ptr() if nh else None, hot_values.data_ptr() if nh else None, hs[0], hs[1], hs[2], nh,
        _C.ptr(hot_len) if nh else None,
        pool.buf.data_ptr(), pool.n_pages, Hkv * pool.rec, pool.rec, block_table.data_ptr(), block_table.stride(0),
        ctypes.byref(pool.layout) if max_blocks else None, max_blocks, warm_len.data_ptr(),
        B, Hq, Hkv, D, float(sm_scale), o.data_ptr(), o.stride(0), o.stride(1), None, None,
        ws.data_ptr(), ws.numel(), _C.ptr(status), _C.stream_of(q3))
    _C.check(rc, "akv_mixed_decode_paged")
    return o
