"""Packed warm-tier storage and byte accounting.

``measure_packed_bytes`` keeps the reference's accounting
(akv/packed_layout.py:501-543): packed codes + scale + zero bytes, outlier
side-store not counted.

``WarmArena`` is the packed warm tier of one layer.  Tokens live in 32-token
block records (layout in include/akv_b200.h, ``akv_warm_layout``), one run of
records per (batch row, KV head), preallocated for ``max_blocks`` blocks.  A
record carries exactly what one reference quantiser call returns for those
tokens, so the arena is the source of truth for attention (read in place by
``akv_mixed_decode``), promotion (``akv_dequantize``) and the cold tier
(byte-for-byte copies of records).
"""
from __future__ import annotations

import ctypes

import torch

from . import _C
from .affine_quantizer import n_outliers
from .bitpack import packed_width

BLOCK = _C.BLOCK_TOKENS


def key_scale_channels(bits: int, head_dim: int) -> list:
    """Channel stored in each slot of a warm record's K scale / zero field.

    Records keep the per-channel K scale and zero of every 32-channel chunk in
    the decode kernel's pair order (include/akv_b200.h, ``akv_warm_layout``):
    slot 2i / 2i+1 of a chunk hold channels a / b of pair i.
    """
    out = []
    for base in range(0, head_dim, 32):
        for i in range(16):
            j = i % 8
            if bits == 4:
                a = 8 * (i // 4) + ((i % 4) ^ 1)
                b = a + 4
            else:
                a = 16 * (i // 8) + ((3 - j if j < 4 else 11 - j) if bits == 2 else 7 - j)
                b = a + 8
            out += [base + a, base + b]
    return out


def measure_packed_bytes(qdata: dict, bits: int) -> int:
    """Bytes a quantiser call's output occupies (reference packed_layout.py:501-543)."""
    if "codes" not in qdata:
        return 0
    codes = qdata["codes"]
    if "bits" in qdata:
        total = codes.element_size() * codes.numel()
    else:
        D = codes.shape[-1]
        rows = codes.numel() // D if D else 0
        total = rows * packed_width(D, bits) if bits in (2, 3, 4) else codes.element_size() * codes.numel()
    for key in ("group_mean", "group_std", "scale", "zero"):
        t = qdata.get(key)
        if isinstance(t, torch.Tensor):
            total += t.element_size() * t.numel()
    return int(total)


def record_dest(L: _C.WarmLayout, base: int, sb: int, sh: int, sblk: int, is_key: bool) -> _C.QDest:
    """QDest addressing the K (or V) fields of block records: the record of
    (b, h, blk) starts at base + b*sb + h*sh + blk*sblk (bytes)."""
    n = L.n_outlier
    d = _C.QDest()
    if is_key:
        d.pair_order = 1  # records keep K scale / zero in the decode pair order
        d.codes = _C.View(base + L.kc, sb, sh, sblk, packed_width(L.head_dim, L.key_bits))
        d.scale = _C.View(base + L.ks, sb, sh, sblk, 0)
        d.zero = _C.View(base + L.kz, sb, sh, sblk, 0)
        if n:
            d.out_data = _C.View(base + L.ko, sb, sh, sblk, 2 * n)
            d.out_idx = _C.View(base + L.ki, sb, sh, sblk, 0)
    else:
        d.codes = _C.View(base + L.vc, sb, sh, sblk, packed_width(L.head_dim, L.value_bits))
        d.scale = _C.View(base + L.vs, sb, sh, sblk, 2)
        d.zero = _C.View(base + L.vz, sb, sh, sblk, 2)
        if n:
            d.out_data = _C.View(base + L.vo, sb, sh, sblk, 2 * n)
            d.out_idx = _C.View(base + L.vi, sb, sh, sblk, 0)
            d.out_vdq = _C.View(base + L.vd, sb, sh, sblk, 2 * n)
    d.mask = _C.View(base + L.mask, sb, sh, sblk, 0)
    d.flags = _C.View(base + L.flags + (0 if is_key else 1), sb, sh, sblk, 0)
    return d


class WarmArena:
    """Packed warm tier: (B, H, max_blocks) block records in one uint8 buffer."""

    def __init__(self, batch: int, heads: int, head_dim: int, key_bits: int, value_bits: int,
                 outlier_fraction: float = 0.0, max_blocks: int = 64, device="cuda"):
        self.B, self.H, self.D = batch, heads, head_dim
        self.key_bits, self.value_bits = key_bits, value_bits
        self.n_out = n_outliers(head_dim, outlier_fraction)
        self.layout = _C.warm_layout(head_dim, key_bits, value_bits, self.n_out)
        self.rec = self.layout.bytes
        self.max_blocks = max_blocks
        self.buf = torch.zeros(batch, heads, max_blocks, self.rec, dtype=torch.uint8, device=device)
        self.n_blocks = 0

    # -------------------------------------------------------------- views
    @property
    def device(self):
        return self.buf.device

    def _base(self, blk0: int) -> int:
        return self.buf.data_ptr() + blk0 * self.rec

    def dest(self, is_key: bool, blk0: int = 0) -> _C.QDest:
        """QDest addressing K (or V) fields of the records starting at block blk0."""
        rec = self.rec
        return record_dest(self.layout, self._base(blk0), self.H * self.max_blocks * rec, self.max_blocks * rec, rec,
                           is_key)

    def grow(self, min_blocks: int) -> None:
        """Make room for at least ``min_blocks`` blocks (capacity doubles; records are copied)."""
        if min_blocks <= self.max_blocks:
            return
        new_max = max(min_blocks, 2 * self.max_blocks)
        buf = torch.zeros(self.B, self.H, new_max, self.rec, dtype=torch.uint8, device=self.buf.device)
        buf[:, :, : self.n_blocks] = self.buf[:, :, : self.n_blocks]
        self.buf, self.max_blocks = buf, new_max

    def select_batch(self, index: torch.Tensor) -> None:
        """Keep / repeat batch rows (beam search reorder, batch_select_indices)."""
        self.buf = self.buf.index_select(0, index.to(self.buf.device))
        self.B = self.buf.shape[0]

    # -------------------------------------------------------------- writes
    def append(self, k: torch.Tensor, v: torch.Tensor, group: int = BLOCK, tok_idx: torch.Tensor | None = None,
               status: torch.Tensor | None = None, score_sums: tuple | None = None, score_heads: int = 0) -> int:
        """Quantise (B, H, N, D) fp16 K/V (optionally gathered by ``tok_idx``) into new blocks.

        ``group`` tokens share one K scale (32 = one block; N = one reference
        call over the whole event).  ``score_sums`` = (K, V) all-reduced
        outlier norm sums (B, n_groups, D) when the heads are sharded over
        GPUs (``akv.parallel``), over ``score_heads`` heads in total.
        Returns the first block index written.
        """
        _C.require_cuda(k, v)
        B, H, N, D = (k.shape if tok_idx is None else (k.shape[0], k.shape[1], tok_idx.shape[-1], k.shape[3]))
        if (B, H, D) != (self.B, self.H, self.D):
            raise ValueError("K/V shape does not match the arena")
        nblk = (N + BLOCK - 1) // BLOCK
        if self.n_blocks + nblk > self.max_blocks:
            raise RuntimeError(f"warm arena full ({self.n_blocks}+{nblk} > {self.max_blocks} blocks)")
        blk0 = self.n_blocks
        ti = None if tok_idx is None else tok_idx.contiguous()
        tsb = 0 if ti is None or ti.dim() == 1 else ti.stride(0)
        sp = None if status is None else status.data_ptr()
        if score_sums is None and k.shape == v.shape:  # both fields in one call (akv_warm_append)
            kx = k if k.stride(-1) == 1 else k.contiguous()
            vx = v if v.stride(-1) == 1 else v.contiguous()
            g = min(group, N)
            lib = _C.load()
            needs = self.__dict__.setdefault("_append_ws", {})
            need = needs.get((N, g))
            if need is None:
                need = needs[(N, g)] = lib.akv_warm_append_workspace_bytes(B, H, N, D, g, self.n_out)
            ws = torch.empty(need + 256, dtype=torch.uint8, device=kx.device) if need else None
            wp = None if ws is None else (ws.data_ptr() + 255) // 256 * 256
            _C.check(lib.akv_warm_append(self.buf.data_ptr(), self.buf.stride(0), self.buf.stride(1),
                                         ctypes.byref(self.layout), blk0, kx.data_ptr(), kx.stride(0), kx.stride(1),
                                         kx.stride(2), vx.data_ptr(), vx.stride(0), vx.stride(1), vx.stride(2),
                                         None if ti is None else ti.data_ptr(), tsb, kx.shape[2], B, H, N, g, wp,
                                         need, sp, _C.stream_of(kx)), "akv_warm_append")
            self.n_blocks += nblk
            return blk0
        for i, (x, is_key, bits) in enumerate(((k, True, self.key_bits), (v, False, self.value_bits))):
            if x.stride(-1) != 1:
                x = x.contiguous()
            dest = self.dest(is_key, blk0)
            ss = None if score_sums is None else score_sums[i].contiguous()
            _C.quantize(x.data_ptr(), x.stride(0), x.stride(1), x.stride(2),
                        None if ti is None else ti.data_ptr(), tsb,
                        B, H, N, D, bits, is_key, min(group, N), self.n_out, dest, sp, x.device,
                        score_sum=ss, score_heads=score_heads, n_src=x.shape[2])
        self.n_blocks += nblk
        return blk0

    def dequantize(self, tok_idx: torch.Tensor | None = None, n_tokens: int | None = None,
                   status: torch.Tensor | None = None) -> tuple:
        """FP16 (B, H, N, D) K and V of warm token slots (``tok_idx`` = slot = blk*32 + s).

        A slot outside the arena's written blocks records AKV_ERR_SHAPE in
        ``status`` (an int32 device word, when given) and reads slot 0."""
        lib = _C.load()
        N = tok_idx.shape[-1] if tok_idx is not None else (n_tokens if n_tokens is not None
                                                            else self.n_blocks * BLOCK)
        outs = []
        for is_key, bits in ((True, self.key_bits), (False, self.value_bits)):
            out = torch.empty(self.B, self.H, N, self.D, dtype=torch.float16, device=self.device)
            src = self.dest(is_key, 0)
            rc = lib.akv_dequantize(ctypes.byref(src), None if tok_idx is None else tok_idx.data_ptr(),
                                    0 if tok_idx is None or tok_idx.dim() == 1 else tok_idx.stride(0),
                                    max(self.n_blocks, 1) * BLOCK,
                                    self.B, self.H, N, self.D, bits, int(is_key), self.n_out,
                                    out.data_ptr(), out.stride(0), out.stride(1), out.stride(2),
                                    _C.ptr(status), _C.stream_of(self.buf))
            _C.check(rc, "akv_dequantize")
            outs.append(out)
        return tuple(outs)

    def masks(self) -> torch.Tensor:
        """(B, H, n_blocks) int64 valid-slot masks (host-side bookkeeping / tests)."""
        L = self.layout
        m = self.buf[:, :, : self.n_blocks, L.mask:L.mask + 4].contiguous().view(torch.int32)
        return m[..., 0].to(torch.int64) & 0xFFFFFFFF

    def write_head(self, k: torch.Tensor, v: torch.Tensor, src_head: int, dst_head: int, blk0: int, group: int,
                   tok_idx: torch.Tensor | None = None) -> None:
        """Quantise model head ``src_head`` of (B, H, N, D) K/V (gathered by
        ``tok_idx``) on its own (outlier channels from that head alone) into
        arena head ``dst_head``, blocks from ``blk0``.  Does not move
        ``n_blocks``."""
        _C.require_cuda(k, v)
        B, N, D = k.shape[0], (k.shape[2] if tok_idx is None else tok_idx.shape[-1]), k.shape[3]
        ti = None if tok_idx is None else tok_idx.contiguous()
        tsb = 0 if ti is None or ti.dim() == 1 else ti.stride(0)
        rec = self.rec
        sb, sh = self.H * self.max_blocks * rec, self.max_blocks * rec
        for x, is_key, bits in ((k, True, self.key_bits), (v, False, self.value_bits)):
            xh = x[:, src_head:src_head + 1]
            if xh.stride(-1) != 1:
                xh = xh.contiguous()
            dest = record_dest(self.layout, self._base(blk0) + dst_head * sh, sb, sh, rec, is_key)
            _C.quantize(xh.data_ptr(), xh.stride(0), xh.stride(1), xh.stride(2),
                        None if ti is None else ti.data_ptr(), tsb,
                        B, 1, N, D, bits, is_key, min(group, N), self.n_out, dest, None, x.device,
                        n_src=x.shape[2])

    def drop_slots(self, slots: torch.Tensor) -> None:
        """Drop warm tokens (slot = blk*32 + s, int64 on the device) from every
        row and head by clearing their mask bits (promotion)."""
        words = self.buf[:, :, :, self.layout.mask:self.layout.mask + 4]
        m = words.contiguous().view(torch.int32)[..., 0]
        blk = slots // BLOCK
        bit = torch.ones_like(slots, dtype=torch.int64) << (slots % BLOCK)
        clear = torch.zeros(m.shape[-1], dtype=torch.int64, device=m.device).index_add_(0, blk, bit)
        m &= (~clear).to(torch.int32)
        words.copy_(m.unsqueeze(-1).view(torch.uint8).view(words.shape))

    def clear_slots(self, blk: torch.Tensor, slot_mask: torch.Tensor) -> None:
        """Drop tokens from the warm tier by clearing their mask bits (promotion)."""
        L = self.layout
        m = self.buf[:, :, :, L.mask:L.mask + 4].view(torch.int32)[..., 0]
        m[:, :, blk] &= ~slot_mask.to(torch.int32)

    def packed_bytes(self) -> int:
        """Bytes a reference quantiser would report for the stored blocks (codes+scale+zero)."""
        D, H, B = self.D, self.H, self.B
        per_tok = packed_width(D, self.key_bits) + packed_width(D, self.value_bits) + 4
        return B * H * (self.n_blocks * BLOCK * per_tok + self.n_blocks * 4 * D)

    def resident_bytes(self) -> int:
        return self.buf.numel()


class HeadGroupArena:
    """Warm tier of a layer whose KV heads have their own bit widths
    (reference drop_in.py:315-374, ``per_head_bits``): one ``WarmArena`` per
    distinct width over that width's heads (K and V at the head's width, as
    the reference's per-width quantiser pool), every head quantised on its
    own like the reference's per-head quantiser calls.  Block j of every
    group's arena holds the same tokens, so slots and masks agree across
    groups.  Offers the ``WarmArena`` surface the cache uses, and ``decode``:
    one mixed-tier decode launch per width group over that group's query
    heads."""

    def __init__(self, batch: int, per_head_bits: list, head_dim: int, outlier_fraction: float = 0.0,
                 max_blocks: int = 64, device="cuda"):
        self.B, self.H, self.D = batch, len(per_head_bits), head_dim
        self.per_head_bits = list(per_head_bits)
        self.groups = []  # (bits, model heads, arena)
        for bits in sorted(set(per_head_bits)):
            heads = [h for h, b in enumerate(per_head_bits) if b == bits]
            self.groups.append((bits, heads, WarmArena(batch, len(heads), head_dim, bits, bits, outlier_fraction,
                                                       max_blocks=max_blocks, device=device)))
        self.max_blocks = max_blocks
        self.n_blocks = 0
        self._idx: dict = {}

    @property
    def device(self):
        return self.groups[0][2].device

    def _index(self, key, values) -> torch.Tensor:
        t = self._idx.get(key)
        if t is None:
            t = self._idx[key] = torch.tensor(values, dtype=torch.int64, device=self.device)
        return t

    def grow(self, min_blocks: int) -> None:
        for _, _, a in self.groups:
            a.grow(min_blocks)
        self.max_blocks = self.groups[0][2].max_blocks

    def append(self, k: torch.Tensor, v: torch.Tensor, group: int = BLOCK, tok_idx: torch.Tensor | None = None) -> int:
        N = k.shape[2] if tok_idx is None else tok_idx.shape[-1]
        nblk = (N + BLOCK - 1) // BLOCK
        if self.n_blocks + nblk > self.max_blocks:
            raise RuntimeError(f"warm arena full ({self.n_blocks}+{nblk} > {self.max_blocks} blocks)")
        blk0 = self.n_blocks
        for _, heads, a in self.groups:
            for j, h in enumerate(heads):
                a.write_head(k, v, h, j, blk0, group, tok_idx)
            a.n_blocks = blk0 + nblk
        self.n_blocks = blk0 + nblk
        return blk0

    def dequantize(self, tok_idx: torch.Tensor | None = None, n_tokens: int | None = None) -> tuple:
        N = tok_idx.shape[-1] if tok_idx is not None else (n_tokens if n_tokens is not None
                                                            else self.n_blocks * BLOCK)
        out_k = torch.empty(self.B, self.H, N, self.D, dtype=torch.float16, device=self.device)
        out_v = torch.empty_like(out_k)
        for bits, heads, a in self.groups:
            dk, dv = a.dequantize(tok_idx=tok_idx, n_tokens=n_tokens)
            idx = self._index(("kv", bits), heads)
            out_k.index_copy_(1, idx, dk)
            out_v.index_copy_(1, idx, dv)
        return out_k, out_v

    def masks(self) -> torch.Tensor:
        out = torch.empty(self.B, self.H, self.n_blocks, dtype=torch.int64, device=self.device)
        for bits, heads, a in self.groups:
            out.index_copy_(1, self._index(("kv", bits), heads), a.masks())
        return out

    def drop_slots(self, slots: torch.Tensor) -> None:
        for _, _, a in self.groups:
            a.drop_slots(slots)

    def select_batch(self, index: torch.Tensor) -> None:
        for _, _, a in self.groups:
            a.select_batch(index)
        self.B = self.groups[0][2].B

    def packed_bytes(self) -> int:
        return sum(a.packed_bytes() for _, _, a in self.groups)

    def resident_bytes(self) -> int:
        return sum(a.resident_bytes() for _, _, a in self.groups)

    def decode(self, query: torch.Tensor, hot_keys: torch.Tensor, hot_values: torch.Tensor,
               sm_scale: float | None = None) -> torch.Tensor:
        """query (B, Hq, 1, D) over the hot tier and every group's records ->
        (B, Hq, 1, D): each width group attends its own query heads (GQA
        head h // (Hq / H)) in one launch."""
        from .fused_attention import mixed_tier_decode_attention
        Hq = query.shape[1]
        g = Hq // self.H
        out = torch.empty_like(query)
        for bits, heads, a in self.groups:
            qi = self._index(("q", bits, g), [h * g + i for h in heads for i in range(g)])
            ki = self._index(("kv", bits), heads)
            o = mixed_tier_decode_attention(query.index_select(1, qi), hot_keys.index_select(1, ki),
                                            hot_values.index_select(1, ki), a, sm_scale=sm_scale)
            out.index_copy_(1, qi, o)
        return out
