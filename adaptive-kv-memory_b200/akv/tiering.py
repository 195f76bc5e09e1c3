"""Tier management on the GPU: importance update, demote selection, row
gather/compaction and cold-tier (pinned host) copies.

  fused_importance_update   reference akv/triton_ops.py:604-650
  select_demote_indices     reference akv/drop_in.py:392-413
  select_bottomk            reference akv/vmm.py:221-242 (bottom-k, protected ends)
  gather_rows               reference akv/drop_in.py:684-685, :739-751 (gather / keep-mask)
  cold_copy_blocks /        reference akv/async_migration.py:303-349, with pinned host
  cold_restore_blocks       memory and a side stream (the reference declares
                            pin_memory but never uses it, :102)
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _C


def fused_importance_update(attention_weights: torch.Tensor, scores: torch.Tensor,
                            decay: float = 0.95) -> torch.Tensor:
    """scores = scores*decay + sum_M mean_{B,H} attn, in place (two roundings, no FMA)."""
    _C.require_cuda(attention_weights, scores)
    a = attention_weights
    if a.dtype != torch.float32:
        a = a.float()
    a = a.contiguous()
    if scores.dtype != torch.float32 or not scores.is_contiguous():
        raise TypeError("scores must be a contiguous fp32 tensor (updated in place)")
    B, H, M, Na = a.shape
    _C.check(_C.load().akv_importance_update(a.data_ptr(), B, H, M, Na, scores.data_ptr(), scores.shape[0],
                                             float(decay), _C.stream_of(scores)), "akv_importance_update")
    return scores


_select_ws: dict = {}  # device -> selection workspace (histograms, threshold state, per-CTA counts)


def select_bottomk(scores: torch.Tensor, k: int, protect_first: int = 4, protect_last: int = 16) -> torch.Tensor:
    """Ascending int64 indices of the k lowest scores, protected ends excluded; ties lowest index first."""
    _C.require_cuda(scores)
    s = scores.float().contiguous()
    n = s.shape[0]
    out = torch.empty(k, dtype=torch.int64, device=s.device)
    if k == 0:
        return out
    need = _C.workspace_bytes("akv_select_workspace_bytes", n)
    key = (s.device.type, s.device.index)
    ws = _select_ws.get(key)
    if ws is None or ws.numel() < need:
        ws = _select_ws[key] = torch.empty(need, dtype=torch.uint8, device=s.device)
    _C.check(_C.load().akv_select_bottomk(s.data_ptr(), n, k, protect_first, protect_last, out.data_ptr(),
                                          ws.data_ptr(), ws.numel(), _C.stream_of(s)), "akv_select_bottomk")
    return out


def select_demote_indices(scores: torch.Tensor, n_demote: int, hot_budget: int,
                          protect_initial: int = 4) -> torch.Tensor:
    """AKVLayer demote choice: first 4 and last min(16, budget//4) positions are never demoted."""
    return select_bottomk(scores, n_demote, protect_initial, min(16, hot_budget // 4))


def gather_rows(x: torch.Tensor, idx: torch.Tensor, out: torch.Tensor | None = None,
                status: torch.Tensor | None = None) -> torch.Tensor:
    """out[b, h, i] = x[b, h, idx[i]] for (B, H, N, D) tensors (rows of D elements).

    An index outside [0, N) records AKV_ERR_SHAPE in ``status`` (an int32
    device word, when given) and copies row 0 instead."""
    _C.require_cuda(x, idx)
    B, H, N, D = x.shape
    n = idx.shape[0]
    if out is None:
        out = torch.empty(B, H, n, D, dtype=x.dtype, device=x.device)
    es = x.element_size()
    if x.stride(-1) != 1 or out.stride(-1) != 1:
        raise ValueError("rows must be contiguous")
    i64 = idx.to(torch.int64).contiguous()
    _C.check(_C.load().akv_gather_rows(x.data_ptr(), x.stride(0) * es, x.stride(1) * es, x.stride(2) * es, N,
                                       i64.data_ptr(), n, B, H, D * es,
                                       out.data_ptr(), out.stride(0) * es, out.stride(1) * es, out.stride(2) * es,
                                       _C.ptr(status), _C.stream_of(x)), "akv_gather_rows")
    return out


def scatter_rows(src: torch.Tensor, dst: torch.Tensor, dst_idx: torch.Tensor, src_idx: torch.Tensor | None = None,
                 status: torch.Tensor | None = None) -> torch.Tensor:
    """dst[b, h, dst_idx[i]] = src[b, h, src_idx[i] if given else i] for (B, H, N, D) tensors.

    Rows read and rows written must not overlap (src may be dst).  An index
    outside its tensor's rows records AKV_ERR_SHAPE in ``status`` and uses
    row 0."""
    _C.require_cuda(src, dst, dst_idx, src_idx)
    B, H, n_src, D = src.shape
    if dst.shape[:2] != (B, H) or dst.shape[3] != D or dst.dtype != src.dtype:
        raise ValueError("src and dst need the same (B, H, *, D) shape and dtype")
    if src.stride(-1) != 1 or dst.stride(-1) != 1:
        raise ValueError("rows must be contiguous")
    es = src.element_size()
    di = dst_idx.to(torch.int64).contiguous()
    si = src_idx.to(torch.int64).contiguous() if src_idx is not None else None
    n = di.shape[0]
    if si is not None and si.shape[0] != n:
        raise ValueError("src_idx and dst_idx lengths differ")
    _C.check(_C.load().akv_scatter_rows(src.data_ptr(), src.stride(0) * es, src.stride(1) * es, src.stride(2) * es,
                                        n_src, _C.ptr(si), di.data_ptr(), n, B, H, D * es, dst.data_ptr(),
                                        dst.stride(0) * es, dst.stride(1) * es, dst.stride(2) * es, dst.shape[2],
                                        _C.ptr(status), _C.stream_of(src)), "akv_scatter_rows")
    return dst


def cold_copy_blocks(arena_buf: torch.Tensor, blk0: int, nblk: int, host: torch.Tensor,
                     stream: torch.cuda.Stream | None = None) -> torch.cuda.Event:
    """Copy warm records [blk0, blk0+nblk) of every (b, h) to a pinned host buffer (B, H, nblk, rec)."""
    B, H, maxb, rec = arena_buf.shape
    if not host.is_pinned():
        raise ValueError("cold tier buffers must be pinned host memory")
    st = stream or torch.cuda.current_stream(arena_buf.device)
    st.wait_stream(torch.cuda.current_stream(arena_buf.device))
    src = arena_buf.data_ptr() + blk0 * rec
    _C.check(_C.load().akv_cold_copy(host.data_ptr(), nblk * rec, src, maxb * rec, nblk * rec, B * H, 0,
                                     st.cuda_stream, None), "akv_cold_copy")
    ev = torch.cuda.Event()
    ev.record(st)
    return ev


def cold_restore_blocks(host: torch.Tensor, arena_buf: torch.Tensor, blk0: int,
                        stream: torch.cuda.Stream | None = None) -> torch.cuda.Event:
    """Copy pinned host records (B, H, nblk, rec) back into arena blocks [blk0, blk0+nblk)."""
    B, H, maxb, rec = arena_buf.shape
    nblk = host.shape[2]
    st = stream or torch.cuda.current_stream(arena_buf.device)
    st.wait_stream(torch.cuda.current_stream(arena_buf.device))
    dst = arena_buf.data_ptr() + blk0 * rec
    _C.check(_C.load().akv_cold_copy(dst, maxb * rec, host.data_ptr(), nblk * rec, nblk * rec, B * H, 1,
                                     st.cuda_stream, None), "akv_cold_copy")
    ev = torch.cuda.Event()
    ev.record(st)
    return ev


class ImportanceMigrator:
    """GPU state and scoring of the reference's ``ImportanceBasedMigrator``
    (akv/vmm.py:113-245): per layer, fp32 attention scores, int64 last-access
    steps and fp32 retrieval flags, grown as the sequence grows.

    ``update`` and ``compute_importance`` run in the CUDA library
    (``akv_migrator_update``, ``akv_migrator_importance``), eviction candidates
    come from the bottom-k kernel.  Defaults follow the reference's VMMConfig.
    """

    def __init__(self, importance_decay: float = 0.95, attention_weight: float = 0.6,
                 recency_weight: float = 0.2, retrieval_weight: float = 0.2, protect_initial: int = 4,
                 protect_recent: int = 32, device="cuda"):
        self.decay = importance_decay
        self.w = (attention_weight, recency_weight, retrieval_weight)
        self.protect_initial, self.protect_recent = protect_initial, protect_recent
        self.device = torch.device(device)
        self._state: dict = {}  # layer -> [scores, access, retrieval, length]
        self._step = 0
        self._ws = torch.empty(64, dtype=torch.uint8, device=self.device)

    def _grow(self, layer: int, n: int):
        st = self._state.get(layer)
        if st is None:
            cap = max(n, 64)
            st = [torch.zeros(cap, device=self.device), torch.zeros(cap, dtype=torch.int64, device=self.device),
                  torch.zeros(cap, device=self.device), 0]
            self._state[layer] = st
        elif st[0].shape[0] < n:
            cap = max(n, 2 * st[0].shape[0])
            for i in range(3):
                t = torch.zeros(cap, dtype=st[i].dtype, device=self.device)
                t[: st[i].shape[0]] = st[i]
                st[i] = t
        return st

    def update(self, layer_idx: int, attention_weights: torch.Tensor, seq_len: Optional[int] = None) -> None:
        """Fold one step's (B, H, Q, KV) attention into the layer's scores (vmm.py:121-164)."""
        _C.require_cuda(attention_weights)
        a = attention_weights.float().contiguous()
        B, H, M, Na = a.shape
        st = self._grow(layer_idx, Na)
        n_prev = min(st[3], Na)
        _C.check(_C.load().akv_migrator_update(a.data_ptr(), B, H, M, Na, st[0].data_ptr(), st[1].data_ptr(),
                                               st[2].data_ptr(), n_prev, self._step, float(self.decay),
                                               _C.stream_of(a)), "akv_migrator_update")
        st[3] = max(st[3], Na)

    def mark_promoted(self, layer_idx: int, indices: torch.Tensor) -> None:
        st = self._state.get(layer_idx)
        if st is not None and indices.numel() > 0:
            st[2][indices.to(self.device)] = 1.0

    def compact(self, layer_idx: int, keep: torch.Tensor) -> None:
        """Keep only positions ``keep`` (ascending int64 on the device), in that
        order: the tier manager's hot compaction after a demotion."""
        st = self._state.get(layer_idx)
        if st is None:
            return
        m = keep.numel()
        for i in range(3):
            st[i][:m] = st[i][keep]
        st[3] = m

    def advance_step(self) -> None:
        self._step += 1
        for st in self._state.values():
            st[2].mul_(0.9)

    def compute_importance(self, layer_idx: int, seq_len: int) -> torch.Tensor:
        """(seq_len,) composite importance, protected ends +inf (vmm.py:175-219)."""
        st = self._state.get(layer_idx)
        if st is None:
            return torch.arange(seq_len, dtype=torch.float32, device=self.device)
        out = torch.empty(seq_len, dtype=torch.float32, device=self.device)
        wa, wr, wt = self.w
        _C.check(_C.load().akv_migrator_importance(st[0].data_ptr(), st[1].data_ptr(), st[2].data_ptr(), seq_len,
                                                   self._step, float(wa), float(wr), float(wt),
                                                   self.protect_initial, self.protect_recent, out.data_ptr(),
                                                   self._ws.data_ptr(), self._ws.numel(), _C.stream_of(out)),
                 "akv_migrator_importance")
        return out

    def get_eviction_candidates(self, layer_idx: int, seq_len: int, num_to_evict: int) -> torch.Tensor:
        """Ascending indices of the least important positions (vmm.py:221-242)."""
        if num_to_evict <= 0:
            return torch.empty(0, dtype=torch.int64, device=self.device)
        imp = self.compute_importance(layer_idx, seq_len)
        protected = min(seq_len, min(self.protect_initial, seq_len) + min(self.protect_recent, seq_len))
        k = min(num_to_evict, seq_len - protected)
        if k <= 0:
            return torch.empty(0, dtype=torch.int64, device=self.device)
        return select_bottomk(imp, k, 0, 0)

    def reset(self) -> None:
        self._state.clear()
        self._step = 0
