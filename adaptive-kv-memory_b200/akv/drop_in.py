"""HuggingFace drop-in: ``AKVCache`` / ``AKVLayer`` (reference akv/drop_in.py).

``AKVCache`` subclasses ``transformers.DynamicCache`` and ``AKVLayer``
subclasses ``DynamicLayer``, with the reference's constructor arguments,
presets, tier policy and bookkeeping (drop_in.py:131-878, :885-1318):

* every ``update()`` appends the new tokens to the FP16 hot tier, decays
  the recency importance (x0.3, new tokens 1.0, :376-390), optionally
  promotes warm tokens (attention weights, :415-484, or the key-similarity
  proxy, :486-589), and demotes the lowest-importance hot tokens beyond the
  budget (:676-751);
* a demote event is quantised as ONE scale group per batch row, exactly the
  reference's single ``AffineQuantizer`` call per event (:699-701), by the
  sm_100a quantiser reading the hot rows in place through the demote indices
  (fused gather) and writing packed warm block records (``WarmArena``, the
  source of truth for the warm tier);
* the returned K/V is the chronologically sorted [warm; hot] FP16 view
  (:753-787); the warm part is the exact dequantisation of the packed
  records, produced by the dequantise kernel once per demoted token and kept
  as the working copy, as the reference does.

Demote selection uses ``torch.topk`` on the CPU importance vector like the
reference (:392-413): the recency scores are full of ties and the reference's
tier indices are defined by that call's tie order.  ``akv.tiering`` offers
the GPU bottom-k kernel for callers whose scores need no such tie parity.

Everything that touches K/V runs on CUDA; a demotion on CPU tensors raises
(no CPU fallback).  Layers that never demote (large budget, protected
layers) only concatenate tensors and work on any device, like the
reference.
"""
from __future__ import annotations

import ctypes
import logging
import math
from typing import Any, Optional, Tuple

import numpy as np
import torch

from . import _C
from .bitpack import packed_width
from .packed_layout import BLOCK, HeadGroupArena, WarmArena
from .fused_attention import KERNEL_HEAD_DIMS as _KERNEL_HEAD_DIMS
from .tiering import gather_rows, scatter_rows

logger = logging.getLogger(__name__)

try:
    from transformers.cache_utils import DynamicCache as _CacheBase
    from transformers.cache_utils import DynamicLayer as _LayerBase
except ImportError:  # transformers absent: plain containers with the same surface
    class _CacheBase:  # type: ignore[no-redef]
        def __init__(self, *args, **kwargs):
            self.layers = []

    class _LayerBase:  # type: ignore[no-redef]
        def __init__(self):
            self.keys = None
            self.values = None
            self.is_initialized = False

        def get_seq_length(self) -> int:
            return 0 if self.keys is None else self.keys.shape[-2]


def _to_device(t: torch.Tensor, device: torch.device) -> torch.Tensor:
    """A small CPU index tensor on ``device`` without a stream sync: staged in
    pinned memory and copied asynchronously (a copy from pageable memory
    waits for the stream first)."""
    if t.device == device:
        return t
    if device.type == "cuda":
        return t.pin_memory().to(device, non_blocking=True)
    return t.to(device)


# presets of the reference (drop_in.py:89-126)
class _GapVec:
    """A host vector kept as the live slice [lo, hi) of a larger numpy
    buffer: removing the element at logical index i moves the shorter side
    (O(min(i, n - i))), appending writes one slot (amortised O(1)).  The hot
    tier's logical-order vectors (positions, importance, buffer rows) live
    here, so a decode step that demotes a token near the front and appends
    one at the end rewrites neither vector."""

    __slots__ = ("buf", "lo", "hi")

    def __init__(self, arr, dtype):
        a = np.asarray(arr, dtype=dtype).reshape(-1)
        n = a.shape[0]
        self.buf = np.empty(max(2 * n, 64), dtype=dtype)
        self.buf[:n] = a
        self.lo, self.hi = 0, n

    def __len__(self) -> int:
        return self.hi - self.lo

    def view(self) -> np.ndarray:
        return self.buf[self.lo:self.hi]

    def remove(self, i: int) -> None:
        lo, hi, b = self.lo, self.hi, self.buf
        if i < (hi - lo) // 2:
            b[lo + 1:lo + 1 + i] = b[lo:lo + i].copy()
            self.lo = lo + 1
        else:
            b[lo + i:hi - 1] = b[lo + i + 1:hi].copy()
            self.hi = hi - 1

    def append(self, x) -> None:
        if self.hi == self.buf.shape[0]:
            n = self.hi - self.lo
            nb = np.empty(max(2 * (n + 1), 64), dtype=self.buf.dtype)
            nb[:n] = self.buf[self.lo:self.hi]
            self.buf, self.lo, self.hi = nb, 0, n
        self.buf[self.hi] = x
        self.hi += 1


_PRESETS = {
    "quality": {"warm_bits": 4, "hot_budget": 256, "description": "Near-lossless 4-bit. +1-2% PPL."},
    "balanced": {"warm_bits": 3, "hot_budget": 128, "description": "Block-affine 3-bit. +3.3% PPL, 5x compression."},
    "compact": {"warm_bits": 2, "hot_budget": 64, "description": "Block-affine 2-bit. +11% PPL, 8x compression."},
    "k4v2": {"warm_bits": 4, "warm_key_bits": 4, "warm_value_bits": 2, "hot_budget": 128,
             "description": "Asymmetric K4/V2. Keys preserved, values aggressively compressed."},
    "k4v3": {"warm_bits": 4, "warm_key_bits": 4, "warm_value_bits": 3, "hot_budget": 128,
             "description": "Asymmetric K4/V3. Near-quality keys with balanced value compression."},
}


class AKVLayer(_LayerBase):
    """Per-layer tiered KV state (reference drop_in.py:131-878)."""

    is_compileable: bool = False
    is_sliding: bool = False

    def __init__(self, warm_bits: int = 3, hot_budget: int = 128, group_size: int = 64, protect: bool = False,
                 enable_promotion: bool = True, promotion_threshold: float = 0.05,
                 per_head_bits: Optional[list] = None, enable_promotion_proxy: bool = True,
                 proxy_decay: float = 0.7, adaptive_hot_frac: float = 0.0,
                 warm_key_bits: Optional[int] = None, warm_value_bits: Optional[int] = None,
                 outlier_fraction: float = 0.0, fused_decode: bool = False):
        try:
            super().__init__()
        except TypeError:
            self.keys = None
            self.values = None
            self.is_initialized = False
        self.warm_bits = warm_bits
        self.hot_budget = hot_budget
        self.group_size = group_size
        self.protect = protect
        self.enable_promotion = enable_promotion
        self.promotion_threshold = promotion_threshold
        self.enable_promotion_proxy = enable_promotion_proxy
        self.proxy_decay = proxy_decay
        self.adaptive_hot_frac = adaptive_hot_frac
        self.warm_key_bits = warm_key_bits or warm_bits
        self.warm_value_bits = warm_value_bits or warm_bits
        self.outlier_fraction = outlier_fraction
        # bit width per KV head (calibrated caches, drop_in.py:315-374): K and V
        # of head h at per_head_bits[h], each head quantised on its own; used
        # when the list matches the head count, else the layer's widths apply
        self.per_head_bits = list(per_head_bits) if per_head_bits is not None else None
        # decode steps (one new token) return a placeholder instead of the
        # chronological FP16 view; the "akv" attention function
        # (akv.hf_attention) attends over the packed warm records and the hot
        # tier in place
        self.fused_decode = fused_decode

        # hot tier storage: ring buffers (B, H, cap, D) whose rows [0, _hn) are
        # the live tokens; _phys maps logical hot order (arrival order, promoted
        # tokens first) to buffer rows (None: identity).  A decode step writes
        # its token into the row its demoted token leaves, so no step copies
        # the hot tier; the logical-order tensors (_hot_keys / _hot_values) are
        # rebuilt only where order matters (the view, promotion, batch ops).
        self._hk: Optional[torch.Tensor] = None
        self._hv: Optional[torch.Tensor] = None
        self._hn = 0
        self._phys: Optional[np.ndarray] = None
        self._warm_keys_fp16: Optional[torch.Tensor] = None  # exact dequantisation of the warm records
        self._warm_values_fp16: Optional[torch.Tensor] = None
        # capacity buffers behind the two tensors above: appends write in place
        # (doubling on overflow) instead of re-concatenating the whole warm copy
        self._warm_kbuf: Optional[torch.Tensor] = None
        self._warm_vbuf: Optional[torch.Tensor] = None
        self._nan: Optional[torch.Tensor] = None  # one-element source of the fused-decode placeholder
        self._warm: Optional[WarmArena] = None  # packed warm block records (source of truth)
        # arena slot (blk*32 + s) of each warm token, in warm order (host; the
        # device copy _warm_slots is built when a dequantisation needs it)
        self._wslots_buf = np.zeros(64, dtype=np.int64)
        self._wslots_n = 0
        self._wslots_dev: Optional[torch.Tensor] = None
        # int32 position of the token in each arena slot (host mirror; uploaded
        # for the prefill kernel); slots a demote event leaves empty are never
        # read (their record mask bit is clear)
        self._slot_pos_np: Optional[np.ndarray] = None
        self._slot_pos_dev: Optional[torch.Tensor] = None
        self._warm_len = 0
        self._total_len = 0
        self._warm_bytes_packed = 0
        self._proxy_score: Optional[torch.Tensor] = None
        self._hot_positions: Optional[torch.Tensor] = None
        # positions of the warm tokens in warm order: the front of a host
        # capacity buffer (an append writes only the new entries)
        self._wpos_buf = np.zeros(64, dtype=np.int64)
        self._wpos_n = 0
        self._importance: Optional[torch.Tensor] = None
        self._decay = 0.3
        self._n_anchors = 16
        self._step = 0

    # ------------------------------------------------------------------ hot-tier order vectors
    # Logical-order (arrival order, promoted tokens first) host vectors of the
    # hot tier, kept in _GapVec buffers.  Reads return copies (numpy / CPU
    # torch, as before); assignments replace the vector.
    @property
    def _phys(self) -> Optional[np.ndarray]:
        """Buffer row of each logical hot token (None: identity)."""
        g = self.__dict__.get("_phys_g")
        return None if g is None else g.view().copy()

    @_phys.setter
    def _phys(self, a) -> None:
        self.__dict__["_phys_g"] = None if a is None else _GapVec(a, np.int64)

    @property
    def _hot_positions(self) -> Optional[torch.Tensor]:
        g = self.__dict__.get("_hpos_g")
        return None if g is None else torch.from_numpy(g.view().copy())

    @_hot_positions.setter
    def _hot_positions(self, t) -> None:
        self.__dict__["_hpos_g"] = None if t is None else _GapVec(
            t.numpy() if isinstance(t, torch.Tensor) else t, np.int64)

    @property
    def _importance(self) -> Optional[torch.Tensor]:
        g = self.__dict__.get("_imp_g")
        return None if g is None else torch.from_numpy(g.view().copy())

    @_importance.setter
    def _importance(self, t) -> None:
        self.__dict__["_imp_g"] = None if t is None else _GapVec(
            t.numpy() if isinstance(t, torch.Tensor) else t, np.float32)

    # ------------------------------------------------------------------ hot ring
    def _hot_view(self, buf: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
        if buf is None:
            return None
        if self._phys is None:
            return buf[:, :, :self._hn]
        return buf.index_select(2, _to_device(torch.from_numpy(self._phys), buf.device))

    @property
    def _hot_keys(self) -> Optional[torch.Tensor]:
        """Hot keys (B, H, hot_len, D) in logical order (a view when rows are in order)."""
        return self._hot_view(self._hk)

    @property
    def _hot_values(self) -> Optional[torch.Tensor]:
        return self._hot_view(self._hv)

    def _set_hot(self, which: int, x: Optional[torch.Tensor]) -> None:
        """Replace the keys (0) or values (1) with logical-order tensor x; the
        other buffer is first rewritten in logical order, so the two stay aligned."""
        if self._phys is not None:
            other = self._hv if which == 0 else self._hk
            if other is not None:
                o = self._hot_view(other)
                if which == 0:
                    self._hv = o.contiguous()
                else:
                    self._hk = o.contiguous()
            self._phys = None
        if x is None:
            if which == 0:
                self._hk = None
            else:
                self._hv = None
            self._hn = 0
            return
        buf = x.contiguous() if x.stride(-1) != 1 else x
        if which == 0:
            self._hk = buf
        else:
            self._hv = buf
        self._hn = x.shape[2]

    @_hot_keys.setter
    def _hot_keys(self, x: Optional[torch.Tensor]) -> None:
        self._set_hot(0, x)

    @_hot_values.setter
    def _hot_values(self, x: Optional[torch.Tensor]) -> None:
        self._set_hot(1, x)

    def _hot_reserve(self, n: int) -> None:
        """Room for n live rows (capacity doubles; live rows are copied)."""
        cap = self._hk.shape[2]
        if n <= cap and self._hk.stride(2) == self._hk.shape[3] and self._hk.is_contiguous():
            return
        new_cap = max(n, 2 * cap, self.hot_budget + 64)
        B, H, _, D = self._hk.shape
        for name in ("_hk", "_hv"):
            old = getattr(self, name)
            nb = torch.empty(B, H, new_cap, D, dtype=old.dtype, device=old.device)
            nb[:, :, :self._hn].copy_(old[:, :, :self._hn])
            setattr(self, name, nb)

    def _hot_append(self, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append new tokens at the end of the logical order (rows _hn .. _hn + N)."""
        N = k.shape[2]
        if self._hk is None:
            self._hk, self._hv, self._hn, self._phys = k, v, 0, None
            self._hk = None
            B, H, _, D = k.shape
            cap = max(N, self.hot_budget) + 64
            self._hk = torch.empty(B, H, cap, D, dtype=k.dtype, device=k.device)
            self._hv = torch.empty(B, H, cap, D, dtype=v.dtype, device=v.device)
        self._hot_reserve(self._hn + N)
        self._hk[:, :, self._hn:self._hn + N].copy_(k)
        self._hv[:, :, self._hn:self._hn + N].copy_(v)
        if self._phys is not None:
            self._phys = np.concatenate([self._phys, np.arange(self._hn, self._hn + N, dtype=np.int64)])
        self._hn += N

    def _hot_remove(self, rows: np.ndarray, kept_logical: np.ndarray) -> None:
        """Drop buffer rows ``rows``; the live rows of the tail move into the
        holes, and the logical order becomes the kept logical indices."""
        phys = self._phys if self._phys is not None else np.arange(self._hn, dtype=np.int64)
        new_n = self._hn - rows.size
        gone = np.zeros(self._hn, dtype=bool)
        gone[rows] = True
        holes = rows[rows < new_n]
        movers = np.nonzero(~gone[new_n:])[0] + new_n  # live rows past the new end
        if holes.size:
            dev = self._hk.device
            if holes.size == 1:
                h, m = int(holes[0]), int(movers[0])
                self._hk[:, :, h].copy_(self._hk[:, :, m])
                self._hv[:, :, h].copy_(self._hv[:, :, m])
            else:
                idx = _to_device(torch.from_numpy(np.concatenate([movers, holes])), dev)
                self._move_rows(idx[:movers.size], idx[movers.size:])
            remap = np.arange(self._hn, dtype=np.int64)
            remap[movers] = holes
            new_phys = remap[phys[kept_logical]]
        else:
            new_phys = phys[kept_logical]
        self._hn = new_n
        self._phys = None if np.array_equal(new_phys, np.arange(new_n)) else new_phys

    def _move_rows(self, src: torch.Tensor, dst: torch.Tensor) -> None:
        """Ring rows src -> rows dst (disjoint sets) in both buffers, one row-scatter launch each."""
        if self._hk.stride(-1) == 1 and (self._hk.shape[-1] * self._hk.element_size()) % 16 == 0:
            scatter_rows(self._hk, self._hk, dst, src)
            scatter_rows(self._hv, self._hv, dst, src)
        else:
            self._hk.index_copy_(2, dst, self._hk.index_select(2, src))
            self._hv.index_copy_(2, dst, self._hv.index_select(2, src))

    def _hot_phys_positions(self) -> np.ndarray:
        """Position of the token in each buffer row [0, _hn)."""
        hp = self._hot_positions.numpy()
        if self._phys is None:
            return hp
        out = np.empty(self._hn, dtype=hp.dtype)
        out[self._phys] = hp
        return out

    # ------------------------------------------------------------------ importance / selection
    def _update_importance(self, n_new: int, hot_len: int) -> None:
        """Recency importance on the CPU (drop_in.py:376-390)."""
        if self._importance is None or self._importance.shape[0] != hot_len - n_new:
            self._importance = torch.ones(hot_len, dtype=torch.float32)
        else:  # host bookkeeping in numpy: the same float32 multiply, far less dispatch
            imp = self._importance.numpy()
            self._importance = torch.from_numpy(
                np.concatenate([imp * np.float32(self._decay), np.ones(n_new, dtype=np.float32)]))

    def _select_demote_indices(self, n_demote: int, hot_len: int) -> torch.Tensor:
        """Lowest importance, first 4 / last min(16, budget//4) protected, ascending (drop_in.py:392-413)."""
        protect_initial = 4
        protect_recent = min(16, self.hot_budget // 4)
        if self._importance is None or self._importance.shape[0] != hot_len:
            return torch.arange(n_demote)
        scores = self._importance.numpy().copy()
        scores[:protect_initial] = np.inf
        scores[max(0, hot_len - protect_recent):] = np.inf
        _, idx = torch.from_numpy(scores).topk(n_demote, largest=False)  # torch's tie order, as the reference
        return torch.from_numpy(np.sort(idx.numpy()))

    # ------------------------------------------------------------------ warm tier
    def _demote(self, rows: np.ndarray, positions: np.ndarray) -> None:
        """Quantise hot buffer rows ``rows`` (the demote event, in logical
        order) into new warm records, one scale group per batch row, reading
        the rows in place (a single row by pointer, several through the fused
        gather); ``positions`` are the demoted tokens' positions."""
        hk, hv = self._hk[:, :, :self._hn], self._hv[:, :, :self._hn]
        _C.require_cuda(hk, hv)
        B, H, _, D = hk.shape
        n = int(rows.size)
        if self._warm is None:
            cap = max(4, (n + BLOCK - 1) // BLOCK)
            if self.per_head_bits is not None and len(self.per_head_bits) == H:
                self._warm = HeadGroupArena(B, self.per_head_bits, D, self.outlier_fraction, max_blocks=cap,
                                            device=hk.device)
            else:
                self._warm = WarmArena(B, H, D, self.warm_key_bits, self.warm_value_bits, self.outlier_fraction,
                                       max_blocks=cap, device=hk.device)
        arena = self._warm
        nblk = (n + BLOCK - 1) // BLOCK
        arena.grow(arena.n_blocks + nblk)
        if n == 1:
            r = int(rows[0])
            blk0 = arena.append(hk[:, :, r:r + 1], hv[:, :, r:r + 1], group=1)
        else:
            blk0 = arena.append(hk, hv, group=n, tok_idx=_to_device(torch.from_numpy(rows), hk.device))
        slots = np.arange(blk0 * BLOCK, blk0 * BLOCK + n, dtype=np.int64)
        self._wslots_append(slots)
        self._record_slot_pos(blk0 * BLOCK, positions)
        # the reference's measure_packed_bytes of this event's K and V dicts (drop_in.py:331-336)
        if isinstance(arena, HeadGroupArena):  # one K and one V dict per head, at that head's width
            self._warm_bytes_packed += B * sum(2 * n * packed_width(D, b) + 4 * D + 4 * n for b in self.per_head_bits)
        else:
            kb, vb = self.warm_key_bits, self.warm_value_bits
            self._warm_bytes_packed += B * (H * n * packed_width(D, kb) + 4 * H * D + H * n * packed_width(D, vb)
                                            + 4 * H * n)
        if not self._no_fp16_copy:
            self._append_warm_fp16(*arena.dequantize(tok_idx=_to_device(torch.from_numpy(slots), hk.device)))

    @property
    def _warm_positions(self) -> Optional[torch.Tensor]:
        """Positions of the warm tokens in warm order (CPU int64, a view of the host buffer)."""
        return torch.from_numpy(self._wpos_buf[:self._wpos_n]) if self._wpos_n else None

    @_warm_positions.setter
    def _warm_positions(self, t: Optional[torch.Tensor]) -> None:
        arr = np.zeros(0, np.int64) if t is None else np.asarray(t.numpy() if isinstance(t, torch.Tensor) else t,
                                                                  dtype=np.int64)
        self._wpos_buf = np.array(arr, dtype=np.int64)
        self._wpos_n = arr.shape[0]

    def _wpos_append(self, pos: np.ndarray) -> None:
        n = self._wpos_n + pos.shape[0]
        if n > self._wpos_buf.shape[0]:
            nb = np.empty(max(2 * n, 64), dtype=np.int64)
            nb[:self._wpos_n] = self._wpos_buf[:self._wpos_n]
            self._wpos_buf = nb
        self._wpos_buf[self._wpos_n:n] = pos
        self._wpos_n = n

    @property
    def _wslots(self) -> np.ndarray:
        return self._wslots_buf[:self._wslots_n]

    @_wslots.setter
    def _wslots(self, arr: np.ndarray) -> None:
        self._wslots_buf = np.array(arr, dtype=np.int64)
        self._wslots_n = self._wslots_buf.shape[0]
        self._wslots_dev = None

    def _wslots_append(self, slots: np.ndarray) -> None:
        """Amortised append: the slot list is the front of a capacity buffer."""
        n = self._wslots_n + slots.shape[0]
        if n > self._wslots_buf.shape[0]:
            nb = np.empty(max(2 * n, 64), dtype=np.int64)
            nb[:self._wslots_n] = self._wslots_buf[:self._wslots_n]
            self._wslots_buf = nb
        self._wslots_buf[self._wslots_n:n] = slots
        self._wslots_n = n
        self._wslots_dev = None

    @property
    def _warm_slots(self) -> Optional[torch.Tensor]:
        """Device copy of the warm tokens' arena slots (built when needed)."""
        if self._warm is None:
            return None
        if self._wslots_dev is None or self._wslots_dev.shape[0] != self._wslots.shape[0]:
            self._wslots_dev = _to_device(torch.from_numpy(self._wslots), self._warm.device)
        return self._wslots_dev

    def _record_slot_pos(self, slot0: int, positions: np.ndarray) -> None:
        """Positions of the tokens written at arena slots slot0 .. slot0 + n - 1."""
        need = self._warm.max_blocks * BLOCK
        buf = self._slot_pos_np
        if buf is None or buf.shape[0] < need:
            nb = np.zeros(need, dtype=np.int32)
            if buf is not None:
                nb[:buf.shape[0]] = buf
            self._slot_pos_np = buf = nb
        buf[slot0:slot0 + positions.shape[0]] = positions
        self._slot_pos_dev = None

    @property
    def _slot_pos(self) -> Optional[torch.Tensor]:
        """Device int32 slot positions for the prefill kernel (uploaded when they changed)."""
        if self._slot_pos_np is None or self._warm is None:
            return None
        if self._slot_pos_dev is None:
            self._slot_pos_dev = _to_device(torch.from_numpy(self._slot_pos_np.copy()), self._warm.device)
        return self._slot_pos_dev

    @property
    def _no_fp16_copy(self) -> bool:
        """A fused cache that never promotes keeps no FP16 working copy of the
        warm tier: nothing reads it at decode, and the view for a prefill or a
        masked step is dequantised from the records when asked for."""
        return self.fused_decode and not self.enable_promotion and not self.enable_promotion_proxy

    def warm_fp16(self) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
        """FP16 K/V of the warm tokens in warm order (the working copy, or the
        records dequantised on demand when no copy is kept)."""
        if self._warm_keys_fp16 is not None or self._warm is None or self._warm_slots is None:
            return self._warm_keys_fp16, self._warm_values_fp16
        return self._warm.dequantize(tok_idx=self._warm_slots)

    def _append_1d(self, name: str, new: torch.Tensor) -> None:
        """``self.<name> = cat([self.<name>, new])`` for the warm tier's
        per-token vectors (positions on the host, record slots on the device),
        amortised: the vector is the front of a capacity buffer and an append
        that fits writes only the new entries.  A vector rebuilt elsewhere
        (promotion) is moved into a new buffer first."""
        cur = getattr(self, name)
        bufs = self.__dict__.setdefault("_vec_bufs", {})
        buf = bufs.get(name)
        n_old = 0 if cur is None else cur.shape[0]
        n = n_old + new.shape[0]
        in_buf = cur is None or (buf is not None and cur.data_ptr() == buf.data_ptr() and cur.device == buf.device)
        if buf is None or not in_buf or n > buf.shape[0] or buf.device != new.device or buf.dtype != new.dtype:
            nb = torch.empty(max(2 * n, 64), dtype=new.dtype, device=new.device)
            if n_old:
                nb[:n_old].copy_(cur)
            bufs[name] = buf = nb
        buf[n_old:n].copy_(new)
        setattr(self, name, buf[:n])

    def _append_warm_fp16(self, dk: torch.Tensor, dv: torch.Tensor) -> None:
        """Append dequantised warm rows to the FP16 working copy.

        The copy lives at the front of capacity buffers; an append that fits
        writes only the new rows.  A copy that is no longer a view of the
        buffers (after promotion or a batch op rebuilt it) is moved into new
        buffers of twice the needed capacity first."""
        old_k, old_v = self._warm_keys_fp16, self._warm_values_fp16
        n_old = 0 if old_k is None else old_k.shape[2]
        n = n_old + dk.shape[2]
        kb = self._warm_kbuf
        in_buf = (old_k is None or (kb is not None and old_k.data_ptr() == kb.data_ptr()
                                    and old_k.shape[:2] == kb.shape[:2]))
        if kb is None or not in_buf or n > kb.shape[2] or kb.shape[:2] != dk.shape[:2]:
            cap = max(2 * n, 64)
            B, H, _, D = dk.shape
            kb = torch.empty(B, H, cap, D, dtype=dk.dtype, device=dk.device)
            vb = torch.empty(B, H, cap, D, dtype=dv.dtype, device=dv.device)
            if n_old:
                kb[:, :, :n_old].copy_(old_k)
                vb[:, :, :n_old].copy_(old_v)
            self._warm_kbuf, self._warm_vbuf = kb, vb
        self._warm_kbuf[:, :, n_old:n].copy_(dk)
        self._warm_vbuf[:, :, n_old:n].copy_(dv)
        self._warm_keys_fp16 = self._warm_kbuf[:, :, :n]
        self._warm_values_fp16 = self._warm_vbuf[:, :, :n]

    def _remove_warm(self, promote_mask: torch.Tensor, n_promote: int, warm_len: int) -> None:
        """Drop promoted tokens from the warm tier (records keep the bytes, mask bits cleared)."""
        keep = ~promote_mask
        pm = promote_mask.detach().cpu().numpy()
        gone = self._wslots[pm]
        if self._warm is not None and gone.size:
            self._warm.drop_slots(_to_device(torch.from_numpy(gone), self._warm.device))
        self._warm_keys_fp16 = self._warm_keys_fp16[:, :, keep, :]
        self._warm_values_fp16 = self._warm_values_fp16[:, :, keep, :]
        self._wslots = self._wslots[~pm]
        if self._warm_positions is not None:
            self._warm_positions = self._warm_positions[keep.detach().to("cpu")]
        if warm_len > 0:
            keep_frac = max(0, warm_len - n_promote) / warm_len
            self._warm_bytes_packed = int(self._warm_bytes_packed * keep_frac)
        self._warm_len -= n_promote

    def _promote(self, promote_mask: torch.Tensor, n_promote: int, filter_proxy: bool) -> None:
        """Move warm tokens to the front of the hot tier with importance 2.0.

        The proxy path keeps its scores aligned with the warm tier; the
        attention path leaves them as they are, like the reference (the next
        proxy update then restarts the EMA on the length mismatch)."""
        warm_len = self._warm_keys_fp16.shape[2]
        promote_idx = promote_mask.nonzero(as_tuple=True)[0]
        promoted_pos = self._warm_positions[promote_idx.detach().to("cpu")] if self._warm_positions is not None else None
        wk = self._warm_keys_fp16
        if self._hk is not None and wk.stride(-1) == 1 and (wk.shape[-1] * wk.element_size()) % 16 == 0:
            # promoted rows go to free ring rows [hn, hn + n) by the row
            # gather and to the front of the logical order
            hn = self._hn
            self._hot_reserve(hn + n_promote)
            gather_rows(self._warm_keys_fp16, promote_idx, out=self._hk[:, :, hn:hn + n_promote])
            gather_rows(self._warm_values_fp16, promote_idx, out=self._hv[:, :, hn:hn + n_promote])
            old = self._phys if self._phys is not None else np.arange(hn, dtype=np.int64)
            self._phys = np.concatenate([np.arange(hn, hn + n_promote, dtype=np.int64), old])
            self._hn = hn + n_promote
        else:
            promoted_k = self._warm_keys_fp16[:, :, promote_idx, :]
            promoted_v = self._warm_values_fp16[:, :, promote_idx, :]
            nk = torch.cat([promoted_k, self._hot_keys], dim=2)
            nv = torch.cat([promoted_v, self._hot_values], dim=2)
            self._hot_keys, self._hot_values = nk, nv
        if filter_proxy:
            self._proxy_score = self._proxy_score[~promote_mask]
        self._remove_warm(promote_mask, n_promote, warm_len)
        if promoted_pos is not None and self._hot_positions is not None:
            self._hot_positions = torch.cat([promoted_pos, self._hot_positions])
        if self._importance is not None:
            self._importance = torch.cat([torch.ones(n_promote) * 2.0, self._importance])

    def _cap_promotion(self, score: torch.Tensor, promote_mask: torch.Tensor) -> Tuple[torch.Tensor, int]:
        n_promote = int(promote_mask.sum().item())
        max_promote = max(1, self.hot_budget // 8)
        if n_promote > max_promote:
            _, top_idx = score.topk(max_promote)
            promote_mask = torch.zeros_like(promote_mask)
            promote_mask[top_idx] = True
            n_promote = max_promote
        return promote_mask, n_promote

    def _promote_from_warm(self, attention_weights: torch.Tensor) -> None:
        """Promotion by mean attention to warm tokens (drop_in.py:415-484)."""
        if self._warm_keys_fp16 is None or self._warm_keys_fp16.shape[2] == 0 or self._hk is None:
            return
        warm_len = self._warm_keys_fp16.shape[2]
        hot_len = self._hn
        if attention_weights.dim() == 4 and attention_weights.shape[-1] >= warm_len + hot_len:
            warm_attn = attention_weights[:, :, :, :warm_len].mean(dim=(0, 1, 2))
            promote_mask = warm_attn > self.promotion_threshold
            if int(promote_mask.sum().item()) > 0:
                promote_mask, n_promote = self._cap_promotion(warm_attn, promote_mask)
                self._promote(promote_mask, n_promote, filter_proxy=False)

    def _update_proxy_score(self, key_states: torch.Tensor) -> None:
        """EMA of |cos(mean new key, warm key)| per warm token (drop_in.py:486-525)."""
        if self._warm_keys_fp16 is None or self._warm_keys_fp16.shape[2] == 0:
            self._proxy_score = None
            return
        probe = key_states.detach().float().mean(dim=(0, 1, 2))
        probe = probe / (probe.norm() + 1e-6)
        wk = self._warm_keys_fp16.detach().float().mean(dim=(0, 1))
        wk = wk / (wk.norm(dim=-1, keepdim=True) + 1e-6)
        sim = wk @ probe
        if self._proxy_score is None or self._proxy_score.shape[0] != sim.shape[0]:
            self._proxy_score = sim.abs()
        else:
            d = self.proxy_decay
            self._proxy_score = d * self._proxy_score + (1 - d) * sim.abs()

    def _promote_from_proxy(self) -> None:
        """Attention-free promotion (drop_in.py:527-589)."""
        if (self._proxy_score is None or self._warm_keys_fp16 is None or self._warm_keys_fp16.shape[2] == 0
                or self._hk is None):
            return
        if self._proxy_score.shape[0] != self._warm_keys_fp16.shape[2]:
            return
        promote_mask = self._proxy_score > self.promotion_threshold
        if int(promote_mask.sum().item()) == 0:
            return
        promote_mask, n_promote = self._cap_promotion(self._proxy_score, promote_mask)
        self._promote(promote_mask, n_promote, filter_proxy=True)

    # ------------------------------------------------------------------ update
    def _publish(self, k: torch.Tensor, v: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        self.keys, self.values = k, v
        self.dtype, self.device = k.dtype, k.device
        self.is_initialized = True
        return k, v

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor,
               cache_kwargs: Optional[dict] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """Append, migrate, return the chronological full view (drop_in.py:591-787)."""
        if self._steady_decode_step(key_states, value_states):
            if self.fused_decode and self._warm is not None:
                return self._publish(*self._placeholder())
            return self._publish(*self.full_view())
        N = key_states.shape[2]
        new_positions = np.arange(self._total_len, self._total_len + N, dtype=np.int64)
        first = self._hk is None
        budget = self.hot_budget
        if self.adaptive_hot_frac > 0.0:
            budget = max(self.hot_budget, int(self.adaptive_hot_frac * (self._total_len + N)))
        # a decode step of a layer that demotes one token and promotes nothing:
        # its token goes straight into the row the demoted token leaves
        fast = (N == 1 and not first and not self.protect and not self.enable_promotion
                and not self.enable_promotion_proxy and self._hn + 1 - budget == 1 and key_states.is_cuda)
        if first:
            self._hot_append(key_states, value_states)
            self._hot_positions = torch.from_numpy(new_positions)
        else:
            if not fast:
                self._hot_append(key_states, value_states)
            self._hot_positions = torch.from_numpy(np.concatenate([self._hot_positions.numpy(), new_positions]))
        self._total_len += N
        if self.protect:
            return self._publish(self._hot_keys, self._hot_values)
        self._step += 1

        hot_len = self._hn + (1 if fast else 0)
        self._update_importance(N, hot_len)
        if self.enable_promotion_proxy:
            self._update_proxy_score(key_states)
        if self.enable_promotion and cache_kwargs and "attention_weights" in cache_kwargs:
            self._promote_from_warm(cache_kwargs["attention_weights"])
            hot_len = self._hn
        elif self.enable_promotion and self.enable_promotion_proxy:
            self._promote_from_proxy()
            hot_len = self._hn

        if hot_len > budget:
            n_demote = hot_len - budget
            d_np = self._select_demote_indices(n_demote, hot_len).numpy()
            if n_demote == 1:  # one index: two slices are much cheaper than np.delete
                v0 = int(d_np[0])
                kept_np = np.concatenate((np.arange(v0, dtype=np.int64), np.arange(v0 + 1, hot_len, dtype=np.int64)))
            else:
                kept_np = np.delete(np.arange(hot_len, dtype=np.int64), d_np)
            hp = self._hot_positions.numpy()
            phys = self._phys if self._phys is not None else np.arange(self._hn, dtype=np.int64)
            if fast and int(d_np[0]) == hot_len - 1:  # the new token itself: append it, then demote
                self._hot_append(key_states, value_states)
                phys = self._phys if self._phys is not None else np.arange(self._hn, dtype=np.int64)
                fast = False
            rows = phys[d_np]
            self._demote(rows, hp[d_np])
            self._wpos_append(hp[d_np])
            self._warm_len += n_demote
            if self._proxy_score is not None:
                pad = torch.zeros(n_demote, dtype=self._proxy_score.dtype, device=self._warm_keys_fp16.device)
                self._proxy_score = torch.cat([self._proxy_score.to(pad.device), pad])
            if fast:  # the new token takes the demoted token's row
                r = int(rows[0])
                self._hk[:, :, r:r + 1].copy_(key_states)
                self._hv[:, :, r:r + 1].copy_(value_states)
                new_phys = np.concatenate((phys[:v0], phys[v0 + 1:], np.array([r], dtype=np.int64)))
                self._phys = None if np.array_equal(new_phys, np.arange(self._hn)) else new_phys
            else:
                self._hot_remove(rows, kept_np)
            if n_demote == 1:
                self._hot_positions = torch.from_numpy(np.concatenate((hp[:v0], hp[v0 + 1:])))
                if self._importance is not None:
                    imp = self._importance.numpy()
                    self._importance = torch.from_numpy(np.concatenate((imp[:v0], imp[v0 + 1:])))
            else:
                self._hot_positions = torch.from_numpy(hp[kept_np])
                if self._importance is not None:
                    self._importance = torch.from_numpy(self._importance.numpy()[kept_np])
        elif fast:  # nothing to demote after all (a promotion path made room): append normally
            self._hot_append(key_states, value_states)

        if self.fused_decode and self._warm is not None:
            return self._publish(*self._placeholder())
        return self._publish(*self.full_view())

    def _steady_decode_step(self, key_states: torch.Tensor, value_states: torch.Tensor) -> bool:
        """The steady-state decode step (one new token, hot tier full, recency
        importance, no promotion) in O(1) host work; False when it does not
        apply (update() then runs the general path).

        Same result as the general path: the recency update imp * 0.3 (fp32)
        with 1.0 for the new token (drop_in.py:376-390), the demoted token is
        the reference's torch.topk(1, largest=False) over the scores with the
        first 4 and last min(16, budget // 4) positions protected
        (drop_in.py:392-413) — for 64 or more scores torch's CPU top-1 is the
        first index of the minimum, which np.argmin returns — then that
        token's row is quantised into a new warm record and the new token is
        written into the row it leaves."""
        if (key_states.shape[2] != 1 or self.protect or self.enable_promotion or self.enable_promotion_proxy
                or self.adaptive_hot_frac > 0.0 or self._hk is None or not key_states.is_cuda):
            return False
        d = self.__dict__
        ig, hg = d.get("_imp_g"), d.get("_hpos_g")
        hn = self._hn
        pr = min(16, self.hot_budget // 4)
        hot_len = hn + 1
        if (hn != self.hot_budget or hot_len < 64 or ig is None or hg is None or len(ig) != hn or len(hg) != hn
                or hot_len - pr <= 4):
            return False
        pg = d.get("_phys_g")
        if pg is None:
            pg = d["_phys_g"] = _GapVec(np.arange(hn, dtype=np.int64), np.int64)
        if (type(self._warm) is WarmArena and self._no_fp16_copy and key_states.dtype == torch.float16
                and self._native_decode_step(key_states, value_states, ig, hg, pg, pr)):
            return True
        # recency importance and the new token's position
        imp = ig.view()
        imp *= np.float32(self._decay)
        ig.append(1.0)
        hg.append(self._total_len)
        self._total_len += 1
        self._step += 1
        # the demoted token: first minimum of the unprotected scores
        v0 = 4 + int(np.argmin(ig.view()[4:hot_len - pr]))
        r = int(pg.view()[v0])
        pos = np.array([hg.view()[v0]], dtype=np.int64)
        self._demote(np.array([r], dtype=np.int64), pos)
        self._wpos_append(pos)
        self._warm_len += 1
        # the new token takes the demoted token's buffer row
        self._hk[:, :, r:r + 1].copy_(key_states)
        self._hv[:, :, r:r + 1].copy_(value_states)
        ig.remove(v0)
        hg.remove(v0)
        pg.remove(v0)
        pg.append(r)
        return True

    def _native_decode_step(self, key_states, value_states, ig: "_GapVec", hg: "_GapVec", pg: "_GapVec",
                            pr: int) -> bool:
        """_steady_decode_step in one library call (akv_layer_decode_step): the
        host vectors are handed over by pointer, the launches issued there.
        The three hot order vectors share one buffer capacity and [lo, hi)."""
        arena = self._warm
        hn = self._hn
        # one capacity and window for the three order vectors, room for one more entry
        if not (ig.lo == hg.lo == pg.lo and ig.hi == hg.hi == pg.hi and ig.hi < ig.buf.shape[0]
                and ig.buf.shape[0] == hg.buf.shape[0] == pg.buf.shape[0]):
            cap = max(2 * (hn + 1), 64)
            for g in (ig, hg, pg):
                nb = np.empty(cap, dtype=g.buf.dtype)
                nb[:hn] = g.view()
                g.buf, g.lo, g.hi = nb, 0, hn
        if arena.n_blocks + 1 > arena.max_blocks:
            arena.grow(arena.n_blocks + 1)
        if self._wslots_n + 1 > self._wslots_buf.shape[0]:
            nb = np.empty(max(2 * (self._wslots_n + 1), 64), dtype=np.int64)
            nb[:self._wslots_n] = self._wslots_buf[:self._wslots_n]
            self._wslots_buf = nb
        if self._wpos_n + 1 > self._wpos_buf.shape[0]:
            nb = np.empty(max(2 * (self._wpos_n + 1), 64), dtype=np.int64)
            nb[:self._wpos_n] = self._wpos_buf[:self._wpos_n]
            self._wpos_buf = nb
        if self._slot_pos_np is None or self._slot_pos_np.shape[0] < arena.max_blocks * BLOCK:
            self._record_slot_pos(0, np.zeros(0, dtype=np.int64))
        hk, hv = self._hk, self._hv
        if hk.stride() != hv.stride() or hk.stride(-1) != 1 or key_states.stride(-1) != 1 \
                or value_states.stride(-1) != 1:
            return False
        c = self.__dict__.get("_step_ctx")
        key = self.__dict__.get("_step_key")
        fresh = (c is not None and key is not None and key[0] is hk and key[1] is arena.buf and key[2] is ig.buf
                 and key[3] is self._wslots_buf and key[4] is self._wpos_buf and key[5] is self._slot_pos_np
                 and c.lo == ig.lo and c.hi == ig.hi and c.n_blocks == arena.n_blocks
                 and c.n_wslots == self._wslots_n and c.n_wpos == self._wpos_n and c.total_len == self._total_len
                 and c.step == self._step and c.warm_len == self._warm_len
                 and c.warm_bytes_packed == self._warm_bytes_packed and key[6] is hg.buf and key[7] is pg.buf)
        if not fresh:
            c = self._refresh_step_ctx(c, hk, hv, arena, ig, hg, pg, pr)
        ks, vs = key_states.stride(), value_states.stride()
        _C.check(_C.load().akv_layer_decode_step(ctypes.byref(c), key_states.data_ptr(), ks[0], ks[1],
                                                 value_states.data_ptr(), vs[0], vs[1], _C.stream_of(hk)),
                 "akv_layer_decode_step")
        for g in (ig, hg, pg):
            g.lo, g.hi = c.lo, c.hi
        arena.n_blocks = c.n_blocks
        self._wslots_n, self._wpos_n = c.n_wslots, c.n_wpos
        self._wslots_dev = None
        self._slot_pos_dev = None
        self._total_len, self._step, self._warm_len = c.total_len, c.step, c.warm_len
        self._warm_bytes_packed = c.warm_bytes_packed
        return True

    def _refresh_step_ctx(self, c, hk, hv, arena, ig, hg, pg, pr):
        """(Re)fill the akv_layer_step struct from the layer's current state."""
        if c is None:
            c = self.__dict__["_step_ctx"] = _C.LayerStep()
            kb, vb, D, H, B = self.warm_key_bits, self.warm_value_bits, arena.D, arena.H, arena.B
            c.layout = arena.layout
            c.B, c.H = B, H
            c.protect_first, c.protect_recent = 4, pr
            c.decay = self._decay
            c.bytes_per_event = B * (H * packed_width(D, kb) + 4 * H * D + H * packed_width(D, vb) + 4 * H)
        c.hot_k, c.hot_v = hk.data_ptr(), hv.data_ptr()
        c.h_sb, c.h_sh, c.h_sn = hk.stride(0), hk.stride(1), hk.stride(2)
        c.hot_rows = hk.shape[2]
        buf = arena.buf
        c.arena, c.a_sb, c.a_sh = buf.data_ptr(), buf.stride(0), buf.stride(1)
        c.n_blocks, c.max_blocks = arena.n_blocks, arena.max_blocks
        c.phys, c.hpos, c.imp = pg.buf.ctypes.data, hg.buf.ctypes.data, ig.buf.ctypes.data
        c.lo, c.hi, c.cap = ig.lo, ig.hi, ig.buf.shape[0]
        c.wslots, c.n_wslots, c.cap_wslots = self._wslots_buf.ctypes.data, self._wslots_n, self._wslots_buf.shape[0]
        c.wpos, c.n_wpos, c.cap_wpos = self._wpos_buf.ctypes.data, self._wpos_n, self._wpos_buf.shape[0]
        c.slot_pos, c.cap_slot_pos = self._slot_pos_np.ctypes.data, self._slot_pos_np.shape[0]
        c.total_len, c.step, c.warm_len = self._total_len, self._step, self._warm_len
        c.warm_bytes_packed = self._warm_bytes_packed
        self.__dict__["_step_key"] = (hk, buf, ig.buf, self._wslots_buf, self._wpos_buf, self._slot_pos_np, hg.buf,
                                      pg.buf)
        return c

    def full_view(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """The chronologically sorted [warm; hot] FP16 K/V (drop_in.py:753-787)."""
        wk, wv = self.warm_fp16()
        if wk is None:
            return self._hot_keys, self._hot_values
        full_k = torch.cat([wk, self._hot_keys], dim=2)
        full_v = torch.cat([wv, self._hot_values], dim=2)
        order = torch.cat([self._warm_positions, self._hot_positions]).argsort().to(full_k.device)
        return full_k.index_select(2, order), full_v.index_select(2, order)

    def _placeholder(self) -> Tuple[torch.Tensor, torch.Tensor]:
        """What a fused decode step returns instead of the view: NaN-filled
        zero-stride tensors of the view's shape, the key tagged with this
        layer.  Only the "akv" attention function reads the tag; any other
        attention over them produces NaN, never a silently wrong result."""
        hk = self._hk
        if self._nan is None or self._nan.dtype != hk.dtype or self._nan.device != hk.device:
            self._nan = torch.full((1, 1, 1, 1), float("nan"), dtype=hk.dtype, device=hk.device)
        B, H, _, D = hk.shape
        n = self._hn + self._warm_len
        k = self._nan.expand(B, H, n, D)
        v = self._nan.expand(B, H, n, D)
        k._akv_layer = self
        return k, v

    def can_prefill_fused(self) -> bool:
        """Prefill attention can read this layer's tiers in place (one bit
        width for every head, and a position recorded for every warm slot)."""
        return (self._warm is not None and not isinstance(self._warm, HeadGroupArena)
                and self._slot_pos_np is not None and self._hk is not None)

    def prefill_attention(self, query: torch.Tensor, sm_scale: Optional[float] = None) -> torch.Tensor:
        """The newest q_len tokens' queries (B, Hq, q_len, D), causal by
        position over the packed warm records and the FP16 hot tier in place
        (akv_prefill_attention) -- the SDPA over the chronological view of the
        reference's prefill (drop_in.py:753-787).  Returns (B, Hq, q_len, D)."""
        from .fused_attention import prefill_attention
        M = query.shape[2]
        dev = query.device
        q_pos = torch.arange(self._total_len - M, self._total_len, dtype=torch.int32, device=dev)
        # the hot rows in buffer order, each with its token's position (order does not matter)
        hot_pos = _to_device(torch.from_numpy(self._hot_phys_positions().astype(np.int32)), dev)
        hn = self._hn
        return prefill_attention(query, q_pos, self._hk[:, :, :hn], self._hv[:, :, :hn], hot_pos, self._warm,
                                 self._slot_pos[: self._warm.n_blocks * BLOCK], sm_scale=sm_scale)

    def decode_attention(self, query: torch.Tensor, sm_scale: Optional[float] = None,
                         reuse_out: bool = False) -> torch.Tensor:
        """One decode query (B, Hq, 1, D) over the packed warm records and the
        FP16 hot tier, in place (akv_mixed_decode).  Returns (B, Hq, 1, D).
        reuse_out: write into a buffer the layer keeps and reuses at its next
        step (for a caller that consumes the result before then)."""
        warm = self._warm
        hk_all = self._hk
        if (type(warm) is WarmArena and self._hn > 0 and query.dtype == torch.float16 and query.dim() == 4
                and query.stride(-1) == 1 and query.shape[-1] in _KERNEL_HEAD_DIMS
                and hk_all.stride() == self._hv.stride()):
            return self._decode_args_call(query, hk_all, self._hv, warm, sm_scale, reuse_out)
        from .fused_attention import mixed_tier_decode_attention
        hk, hv = hk_all[:, :, :self._hn], self._hv[:, :, :self._hn]  # buffer order: attention is order-free
        if isinstance(warm, HeadGroupArena):
            return warm.decode(query, hk, hv, sm_scale=sm_scale)
        return mixed_tier_decode_attention(query, hk, hv, warm, sm_scale=sm_scale)

    def _decode_args_call(self, query, hk, hv, warm, sm_scale, reuse_out: bool = False) -> torch.Tensor:
        """mixed_tier_decode_attention through akv_mixed_decode_args: the
        layer keeps the argument struct and its workspace; a step rewrites
        the query pointer and the lengths, the rest only when the tensors
        behind it (hot buffer, warm arena, query shape, scale) changed."""
        B, Hq, _, D = query.shape
        d = self.__dict__
        a = d.get("_dec_args")
        if a is None:
            a = d["_dec_args"] = _C.DecodeArgs()
            d["_dec_need"] = ctypes.c_size_t(0)
            a.workspace_need = ctypes.addressof(d["_dec_need"])
            d["_dec_ws"] = None
            d["_dec_key"] = None
        buf = warm.buf
        qs = query.stride()
        objs, vals = (hk, hv, buf, warm.layout), (B, Hq, D, qs[0], qs[1], sm_scale)
        old = d["_dec_key"]
        if old is None or any(x is not y for x, y in zip(objs, old[0])) or vals != old[1]:
            d["_dec_key"] = (objs, vals)
            a.q_sb, a.q_sh = qs[0], qs[1]
            a.hot_k, a.hot_v = hk.data_ptr(), hv.data_ptr()
            a.h_sb, a.h_sh, a.h_sn = hk.stride(0), hk.stride(1), hk.stride(2)
            a.warm, a.w_sb, a.w_sh = buf.data_ptr(), buf.stride(0), buf.stride(1)
            a.layout = ctypes.addressof(warm.layout)
            a.B, a.Hq, a.Hkv, a.D = B, Hq, warm.H, D
            a.sm_scale = (1.0 / math.sqrt(D)) if sm_scale is None else float(sm_scale)
            d["_dec_out"] = None
        a.q = query.data_ptr()
        a.n_hot = self._hn
        a.n_warm_blocks = warm.n_blocks
        out = d["_dec_out"] if reuse_out else None
        if out is None or out.device != query.device:
            out = torch.empty(B, Hq, 1, D, dtype=torch.float16, device=query.device)
            if reuse_out:
                d["_dec_out"] = out
            a.out, a.o_sb, a.o_sh = out.data_ptr(), Hq * D, D
        elif a.out != out.data_ptr():
            a.out, a.o_sb, a.o_sh = out.data_ptr(), Hq * D, D
        lib = _C.load()
        stream = _C.stream_of(query)
        rc = lib.akv_mixed_decode_args(ctypes.byref(a), stream)
        if rc == _C.AKV_ERR_WORKSPACE:  # first call or a longer context: a larger workspace, then again
            need = int(d["_dec_need"].value)
            ws = torch.empty(max(2 * need, 1 << 20), dtype=torch.uint8, device=query.device)
            d["_dec_ws"] = ws
            a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
            rc = lib.akv_mixed_decode_args(ctypes.byref(a), stream)
        _C.check(rc, "akv_mixed_decode")
        return out

    # ------------------------------------------------------------------ accounting
    def memory_usage_bytes(self) -> dict:
        """Per-layer byte accounting with the reference's keys (drop_in.py:794-878)."""
        H, D = 1, 128
        hot = 0
        if self._hk is not None:
            B_, H, _, D = self._hk.shape
            hot = 2 * self._hk.element_size() * B_ * H * self._hn * D
        live = 0
        if self._warm_keys_fp16 is not None:
            live = (self._warm_keys_fp16.element_size() * self._warm_keys_fp16.numel()
                    + self._warm_values_fp16.element_size() * self._warm_values_fp16.numel())
        packed = int(self._warm_bytes_packed)
        formula = 0
        if self._warm_len > 0:
            groups = (D + self.group_size - 1) // self.group_size
            formula = self._warm_len * (((H * D * self.warm_bits + 7) // 8) + groups * H * 4) * 2
        total = hot + packed
        fp16_equiv = self._total_len * H * D * 2 * 2
        return {"hot_bytes": hot, "warm_bytes": packed, "warm_bytes_live": live, "warm_bytes_packed": packed,
                "warm_bytes_formula": formula, "total_bytes": total, "fp16_equivalent_bytes": fp16_equiv,
                "savings_ratio": fp16_equiv / max(total, 1),
                "warm_bytes_resident": 0 if self._warm is None else self._warm.resident_bytes()}

    # ------------------------------------------------------------------ batch ops
    def _select_batch(self, fn) -> None:
        if self._hk is not None:
            self._hot_keys, self._hot_values = fn(self._hot_keys), fn(self._hot_values)
        if self._warm_keys_fp16 is not None:
            self._warm_keys_fp16, self._warm_values_fp16 = fn(self._warm_keys_fp16), fn(self._warm_values_fp16)


class AKVCache(_CacheBase):
    """Drop-in ``DynamicCache`` with a packed warm tier (reference drop_in.py:885-1318)."""

    def __init__(self, preset: Optional[str] = None, warm_bits: Optional[int] = None,
                 warm_key_bits: Optional[int] = None, warm_value_bits: Optional[int] = None,
                 hot_budget: Optional[int] = None, group_size: int = 64, outlier_fraction: float = 0.0,
                 protect_first: int = 0, protect_last: int = 0, protect_layers: Optional[list] = None,
                 num_hidden_layers: Optional[int] = None, enable_promotion: bool = True,
                 promotion_threshold: float = 0.05, enable_promotion_proxy: bool = True,
                 proxy_decay: float = 0.7, adaptive_hot_frac: float = 0.0, fused_decode: bool = False):
        if preset is not None:
            if preset not in _PRESETS:
                raise ValueError(f"Unknown preset {preset!r}. Choose from: {sorted(_PRESETS.keys())}")
            if warm_bits is not None or hot_budget is not None:
                raise ValueError("preset= is mutually exclusive with warm_bits/hot_budget. "
                                 "Pick a preset OR pass explicit params.")
            p = _PRESETS[preset]
            self.warm_bits, self.hot_budget = p["warm_bits"], p["hot_budget"]
        else:
            self.warm_bits = warm_bits or 3
            self.hot_budget = hot_budget or 128
        if preset and "warm_key_bits" in _PRESETS[preset]:
            self.warm_key_bits = _PRESETS[preset]["warm_key_bits"]
            self.warm_value_bits = _PRESETS[preset]["warm_value_bits"]
        else:
            self.warm_key_bits = warm_key_bits or self.warm_bits
            self.warm_value_bits = warm_value_bits or self.warm_bits
        self.group_size = group_size
        self.outlier_fraction = outlier_fraction
        self.num_hidden_layers = num_hidden_layers
        self.enable_promotion = enable_promotion
        self.promotion_threshold = promotion_threshold
        self.enable_promotion_proxy = enable_promotion_proxy
        self.proxy_decay = proxy_decay
        self.adaptive_hot_frac = adaptive_hot_frac
        self.fused_decode = fused_decode
        self._protect_first = protect_first
        self._protect_last = protect_last
        self._protect_explicit = list(protect_layers) if protect_layers else []
        if protect_last > 0 and num_hidden_layers is None:
            raise ValueError("protect_last requires num_hidden_layers. "
                             "Use AKVCache.for_model(model, ...) or pass num_hidden_layers=.")
        self._protected_set: set = set(range(protect_first))
        if num_hidden_layers is not None:
            for i in range(protect_last):
                self._protected_set.add(num_hidden_layers - 1 - i)
            for p in self._protect_explicit:
                self._protected_set.add(p if p >= 0 else num_hidden_layers + p)
        else:
            for p in self._protect_explicit:
                if p < 0:
                    raise ValueError("Negative protect_layers indices require num_hidden_layers. "
                                     "Use AKVCache.for_model(model, ...).")
                self._protected_set.add(p)
        super().__init__()
        self._seen_tokens = 0
        self._calibration_per_head_bits: dict = {}

    @classmethod
    def from_calibration(cls, calibration_path, **overrides) -> "AKVCache":
        """Cache from a calibration report JSON (reference drop_in.py:1281-1313):
        protect window and layer count from the report, ``warm_bits`` from its
        average bits when in [2, 4] (else its preset), the per-(layer, head)
        bit widths applied to each layer; ``overrides`` win."""
        import json
        with open(calibration_path) as f:
            rep = json.load(f)
        kwargs = dict(protect_first=rep["recommended_protect_first"], protect_last=rep["recommended_protect_last"],
                      num_hidden_layers=rep["num_layers"])
        avg = float(rep["recommended_average_bits"])
        if 2.0 <= avg <= 4.0:
            kwargs["warm_bits"] = int(round(avg))
        else:
            kwargs["preset"] = rep["recommended_preset"]
        kwargs.update(overrides)
        cache = cls(**kwargs)
        cache._calibration_per_head_bits = {int(k): list(v) for k, v in rep.get("per_head_bits", {}).items()}
        return cache

    @classmethod
    def for_model(cls, model, **kwargs) -> "AKVCache":
        """Cache sized from ``model.config.num_hidden_layers`` (drop_in.py:1011-1054, no adapter registry)."""
        config = getattr(model, "config", None)
        if config is None:
            raise ValueError("model has no .config attribute")
        n_layers = getattr(config, "num_hidden_layers", None) or getattr(config, "n_layer", None)
        if n_layers is None:
            raise ValueError("Could not find num_hidden_layers in model.config. Pass num_hidden_layers= explicitly.")
        return cls(num_hidden_layers=n_layers, **kwargs)

    def _is_protected(self, layer_idx: int) -> bool:
        return layer_idx in self._protected_set

    def _new_layer(self, idx: int) -> AKVLayer:
        return AKVLayer(warm_bits=self.warm_bits, hot_budget=self.hot_budget, group_size=self.group_size,
                        protect=self._is_protected(idx), enable_promotion=self.enable_promotion,
                        promotion_threshold=self.promotion_threshold,
                        enable_promotion_proxy=self.enable_promotion_proxy, proxy_decay=self.proxy_decay,
                        adaptive_hot_frac=self.adaptive_hot_frac, warm_key_bits=self.warm_key_bits,
                        warm_value_bits=self.warm_value_bits, outlier_fraction=self.outlier_fraction,
                        fused_decode=self.fused_decode,
                        per_head_bits=self._calibration_per_head_bits.get(idx))

    def update(self, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               cache_kwargs: Optional[dict[str, Any]] = None, *args, **kwargs) -> Tuple[torch.Tensor, torch.Tensor]:
        """``DynamicCache.update`` contract (drop_in.py:1059-1096)."""
        while len(self.layers) <= layer_idx:
            self.layers.append(self._new_layer(len(self.layers)))
        if layer_idx == 0:
            self._seen_tokens += key_states.shape[2]
        return self.layers[layer_idx].update(key_states, value_states, cache_kwargs)

    def get_seq_length(self, layer_idx: int = 0, *args, **kwargs) -> int:
        if layer_idx < len(self.layers):
            return self.layers[layer_idx].get_seq_length()
        return 0

    def get_usable_length(self, max_length: int, layer_idx: int = 0) -> int:
        return self.get_seq_length(layer_idx)

    def get_max_length(self) -> Optional[int]:
        return None

    @property
    def seen_tokens(self) -> int:
        return self._seen_tokens

    @seen_tokens.setter
    def seen_tokens(self, value: int):
        self._seen_tokens = value

    # ------------------------------------------------------------------ batch / beam ops
    def _each_batch(self, fn, arena_index=None) -> None:
        for layer in self.layers:
            layer._select_batch(fn)
            if layer._warm is not None and arena_index is not None:
                layer._warm.select_batch(arena_index)
            if layer.keys is not None and layer._hk is not None:
                if getattr(layer.keys, "_akv_layer", None) is not None:
                    layer.keys, layer.values = layer._placeholder()
                else:
                    layer.keys, layer.values = fn(layer.keys), fn(layer.values)

    def reorder_cache(self, beam_idx: torch.LongTensor):
        self._each_batch(lambda t: t.index_select(0, beam_idx.to(t.device)), beam_idx)

    def batch_repeat_interleave(self, repeats: int):
        idx = None
        if self.layers and self.layers[0]._hk is not None:
            B = self.layers[0]._hk.shape[0]
            idx = torch.arange(B).repeat_interleave(repeats)
        self._each_batch(lambda t: t.repeat_interleave(repeats, dim=0), idx)
        return self

    def batch_select_indices(self, indices: torch.LongTensor):
        self._each_batch(lambda t: t.index_select(0, indices.to(t.device)), indices)
        return self

    def crop(self, max_length: int):
        """Trim the hot tier from the end (drop_in.py:1231-1243)."""
        for layer in self.layers:
            if layer._hk is not None:
                cur = layer._hn + layer._warm_len
                if cur > max_length:
                    keep = max(0, layer._hn - (cur - max_length))
                    nk, nv = layer._hot_keys[:, :, :keep, :], layer._hot_values[:, :, :keep, :]
                    layer._hot_keys, layer._hot_values = nk, nv
                    layer._total_len = max_length

    def reset(self):
        self.layers.clear()
        self._seen_tokens = 0

    # ------------------------------------------------------------------ accounting
    def memory_usage(self) -> dict:
        keys = ("hot_bytes", "warm_bytes", "warm_bytes_live", "warm_bytes_packed", "warm_bytes_formula",
                "total_bytes", "fp16_equivalent_bytes", "warm_bytes_resident")
        totals = {k: 0 for k in keys}
        for layer in self.layers:
            stats = layer.memory_usage_bytes()
            for k in keys:
                totals[k] += stats.get(k, 0)
        totals["savings_ratio"] = totals["fp16_equivalent_bytes"] / max(totals["total_bytes"], 1)
        totals["num_layers"] = len(self.layers)
        return totals

    def memory_report(self) -> dict:
        stats = self.memory_usage()
        return {"compressed_bytes": stats["total_bytes"], "fp16_equiv_bytes": stats["fp16_equivalent_bytes"],
                "savings_ratio": round(stats["savings_ratio"], 2), "key_bits": self.warm_key_bits,
                "value_bits": self.warm_value_bits, "num_layers": stats["num_layers"],
                "seq_length": self.get_seq_length(0)}

    # ------------------------------------------------------------------ legacy accessors
    def __len__(self) -> int:
        return len(self.layers)

    def __getitem__(self, layer_idx: int):
        if layer_idx < len(self.layers):
            layer = self.layers[layer_idx]
            if layer._hk is not None:
                wk, wv = layer.warm_fp16()
                if wk is not None:
                    return (torch.cat([wk, layer._hot_keys], dim=2), torch.cat([wv, layer._hot_values], dim=2))
                return (layer._hot_keys, layer._hot_values)
        return (torch.tensor([]), torch.tensor([]))

    def __iter__(self):
        for i in range(len(self.layers)):
            yield self[i]

    def to_legacy_cache(self):
        return tuple(self[i] for i in range(len(self.layers)))

    @property
    def key_cache(self):
        return [self[i][0] for i in range(len(self.layers))]

    @property
    def value_cache(self):
        return [self[i][1] for i in range(len(self.layers))]

    @classmethod
    def from_legacy_cache(cls, past_key_values=None):
        cache = cls()
        if past_key_values is not None:
            for layer_idx, (k, v) in enumerate(past_key_values):
                cache.update(k, v, layer_idx)
        return cache


def recommend_preset(model, tokenizer=None, sample_text: str = None) -> dict:
    """Preset heuristic from the model config (reference drop_in.py:1321-1366)."""
    config = getattr(model, "config", None)
    if config is None:
        return {"preset": "balanced", "reason": "No config found, using default"}
    n_layers = getattr(config, "num_hidden_layers", 32)
    n_heads = getattr(config, "num_key_value_heads", getattr(config, "num_attention_heads", 32))
    head_dim = getattr(config, "head_dim",
                       getattr(config, "hidden_size", 4096) // getattr(config, "num_attention_heads", 32))
    est = n_layers * n_heads * head_dim * head_dim * 4
    if est > 5e9:
        return {"preset": "balanced", "warm_bits": 3, "hot_budget": 128, "protect_first": 2, "protect_last": 2,
                "reason": f"Large model ({est/1e9:.0f}B est.) — robust to 3-bit"}
    if est > 1e9:
        return {"preset": "quality", "warm_bits": 4, "hot_budget": 256, "protect_first": 1, "protect_last": 1,
                "reason": f"Medium model ({est/1e9:.1f}B est.) — use 4-bit for safety"}
    return {"preset": "quality", "warm_bits": 4, "hot_budget": 512, "protect_first": 2, "protect_last": 2,
            "reason": f"Small model ({est/1e9:.1f}B est.) — protect more layers"}
