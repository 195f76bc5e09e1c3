"""Multi-GPU partitioning of the warm-tier hot path.

One process per GPU with ``torch.distributed`` (NCCL); three partitions:

* ``batch``    batch rows split over the GPUs.  Every GPU holds all KV heads
               of its rows, so quantisation (outlier selection averages over
               all heads) and attention are local: no collective at all.
* ``head``     KV heads (and their query heads) split over the GPUs.
               Attention is local.  The one exchange step is the outlier
               score of quantisation: the reference picks outlier channels by
               the mean over ALL heads of the per-(head, channel) L2 norms
               (affine_quantizer.py:79 / :146), so each GPU computes its
               heads' norm sums per (batch row, scale group) with the CUDA
               kernel and an all-reduce (SUM) of those D floats per group
               precedes the quantiser (``quantize_head_sharded``).
* ``sequence`` the warm blocks of one sequence split contiguously over the
               GPUs (batch 1 at very long context).  Each GPU's decode writes
               the split-K partial record (acc, m, l) of its tokens; an
               all-gather over NVLink and the same LSE combine kernel that
               merges intra-GPU splits give the output on every GPU
               (``sequence_split_decode``).

The compute steps are CUDA kernels; the orchestration functions take them as
arguments (defaulting to the kernels) so the collective pattern can also be
driven by CPU ``gloo`` ranks in tests.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

import torch

from . import _C


@dataclass(frozen=True)
class ShardPlan:
    mode: str   # "single" | "batch" | "head" | "sequence"
    world: int
    rank: int

    def span(self, n: int) -> tuple:
        """This rank's contiguous [lo, hi) share of n items (the first n % world ranks get one more)."""
        base, extra = divmod(n, self.world)
        lo = self.rank * base + min(self.rank, extra)
        return lo, lo + base + (1 if self.rank < extra else 0)


def plan(batch: int, kv_heads: int, world: int, rank: int, prefer: str = "batch") -> ShardPlan:
    """Batch rows when they divide evenly (no collective), else KV heads, else the sequence."""
    if world == 1:
        return ShardPlan("single", 1, 0)
    order = ("batch", "head") if prefer == "batch" else ("head", "batch")
    for mode in order:
        if mode == "batch" and batch % world == 0:
            return ShardPlan("batch", world, rank)
        if mode == "head" and kv_heads % world == 0:
            return ShardPlan("head", world, rank)
    return ShardPlan("sequence", world, rank)


def _all_reduce_sum(t: torch.Tensor, group=None) -> torch.Tensor:
    import torch.distributed as dist
    dist.all_reduce(t, op=dist.ReduceOp.SUM, group=group)
    return t


def quantize_head_sharded(arena, k: torch.Tensor, v: torch.Tensor, total_heads: int, group: int = 32,
                          tok_idx: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None,
                          process_group=None, norm_sums: Optional[Callable] = None,
                          all_reduce: Optional[Callable] = None) -> int:
    """Append this GPU's heads of (B, H_local, N, D) K/V to its arena with outlier
    channels chosen over all ``total_heads`` heads (reference semantics).

    Without outlier channels nothing crosses GPUs.  Returns the first block written."""
    if arena.n_out == 0:
        return arena.append(k, v, group=group, tok_idx=tok_idx, status=status)
    N = k.shape[2] if tok_idx is None else tok_idx.shape[-1]
    g = min(group, N)
    norm_sums = norm_sums or (lambda x: _C.outlier_norm_sums(x, tok_idx, N, g))
    all_reduce = all_reduce or (lambda t: _all_reduce_sum(t, process_group))
    sums = []
    for x in (k, v):  # same order on every rank
        s = norm_sums(x)
        all_reduce(s)
        sums.append(s)
    return arena.append(k, v, group=group, tok_idx=tok_idx, status=status, score_sums=tuple(sums),
                        score_heads=total_heads)


def _empty_partial(rows: int, D: int, device) -> torch.Tensor:
    p = torch.zeros(rows, D + 2, dtype=torch.float32, device=device)
    p[:, D] = float("-inf")
    return p


def local_partial(query: torch.Tensor, hot_keys: Optional[torch.Tensor], hot_values: Optional[torch.Tensor],
                  warm, sm_scale: Optional[float] = None) -> torch.Tensor:
    """(B*Hq, D+2) partial record of this GPU's tokens (the decode kernel's ``partial_out``)."""
    from .fused_attention import mixed_tier_decode_attention
    q3 = query.reshape(query.shape[0], query.shape[1], query.shape[-1])
    B, Hq, D = q3.shape
    has_hot = hot_keys is not None and hot_keys.shape[2] > 0
    has_warm = warm is not None and warm.n_blocks > 0
    if not has_hot and not has_warm:
        return _empty_partial(B * Hq, D, q3.device)
    p = torch.empty(B * Hq, D + 2, dtype=torch.float32, device=q3.device)
    mixed_tier_decode_attention(q3, hot_keys if has_hot else None, hot_values if has_hot else None,
                                warm if has_warm else None, sm_scale=sm_scale, partial_out=p)
    return p


def combine_partials(part: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """(rows, splits, D+2) partial records -> (rows, D) fp16 via the LSE combine kernel.

    Any row / split strides with a contiguous last dim are read in place, so
    the all-gather's (world, rows, D+2) buffer passes as
    ``gathered.permute(1, 0, 2)`` without a copy."""
    _C.require_cuda(part)
    if part.stride(-1) != 1:
        part = part.contiguous()
    rows, splits, D2 = part.shape
    D = D2 - 2
    if out is None:
        out = torch.empty(rows, D, dtype=torch.float16, device=part.device)
    _C.check(_C.load().akv_lse_combine(part.data_ptr(), part.stride(1), part.stride(0), rows, splits, D,
                                       out.data_ptr(), out.stride(0), None, None, _C.stream_of(part)),
             "akv_lse_combine")
    return out


def _all_gather(t: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """(world, *t.shape): one all_gather_into_tensor on NCCL, a list all_gather elsewhere."""
    import torch.distributed as dist
    t = t.contiguous()
    if t.is_cuda:
        out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
        dist.all_gather_into_tensor(out, t, group=group)
        return out
    outs = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(outs, t, group=group)
    return torch.stack(outs)


class PeerExchange:
    """The cross-GPU step of a sequence split over NVLink peer memory.

    Every rank allocates one exchange buffer (``akv_peer_alloc``: a gather
    area for two epochs of the world's merged partial records, a flag per
    rank, a counter), exports it as a CUDA IPC handle, and maps every other
    rank's buffer (handles exchanged once with ``all_gather_object``).  Then
    ``exchange(part)`` per decode step: ``akv_peer_publish`` stores this
    rank's records into every rank's buffer and raises its flag there,
    ``akv_peer_combine`` waits for the world's flags of the step in local
    memory and merges — no collective call on the data path.  Every rank
    calls ``exchange`` the same number of times, in the same order.
    ``close()`` is collective too."""

    HANDLE_BYTES = 64

    def __init__(self, rows: int, D: int, group=None, device=None):
        import ctypes
        import torch.distributed as dist
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rows, self.D = rows, D
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        lib = _C.load()
        rec = D + 2
        self.n_gather = 2 * self.world * rows * rec
        nbytes = 4 * self.n_gather + 4 * self.world + 8
        p = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _C.check(lib.akv_peer_alloc(nbytes, ctypes.byref(p)), "akv_peer_alloc")
            self.base = p.value
            h = ctypes.create_string_buffer(self.HANDLE_BYTES)
            _C.check(lib.akv_ipc_export(self.base, h), "akv_ipc_export")
            handles = [None] * self.world
            dist.all_gather_object(handles, h.raw, group=group)
            self._opened = []
            bases = []
            for r, hb in enumerate(handles):
                if r == self.rank:
                    bases.append(self.base)
                    continue
                q = ctypes.c_void_p()
                _C.check(lib.akv_ipc_open(ctypes.create_string_buffer(hb, self.HANDLE_BYTES), ctypes.byref(q)),
                         "akv_ipc_open")
                self._opened.append(q.value)
                bases.append(q.value)
        self.flags = self.base + 4 * self.n_gather
        self.counter = self.flags + 4 * self.world
        self.peer_gather = torch.tensor(bases, dtype=torch.int64, device=self.device)
        self.peer_flags = torch.tensor([b + 4 * self.n_gather for b in bases], dtype=torch.int64, device=self.device)
        self.epoch = 0
        dist.barrier(group=group)  # every rank has mapped every buffer before the first publish

    def exchange(self, part: torch.Tensor, out: Optional[torch.Tensor] = None, lse: Optional[torch.Tensor] = None,
                 status: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Merge this rank's (rows, D+2) partial records with every other rank's: (rows, D) fp16."""
        if part.shape != (self.rows, self.D + 2) or part.dtype != torch.float32 or part.stride(-1) != 1:
            raise ValueError("partial records must be fp32 (rows, D+2) with a contiguous last dim")
        if out is None:
            out = torch.empty(self.rows, self.D, dtype=torch.float16, device=part.device)
        lib = _C.load()
        st = _C.stream_of(part)
        self.epoch += 1
        _C.check(lib.akv_peer_publish(part.data_ptr(), part.stride(0), self.rows, self.D, self.peer_gather.data_ptr(),
                                      self.peer_flags.data_ptr(), self.world, self.rank, self.epoch, self.counter, st),
                 "akv_peer_publish")
        _C.check(lib.akv_peer_combine(self.base, self.flags, self.rows, self.D, self.world, self.epoch,
                                      out.data_ptr(), out.stride(0), _C.ptr(lse), _C.ptr(status), st),
                 "akv_peer_combine")
        return out

    def close(self) -> None:
        """Collective: after every rank's work is done, unmap the peers' buffers and free this one."""
        import torch.distributed as dist
        if self.base is None:
            return
        lib = _C.load()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)  # nobody still stores into a buffer about to go
        with torch.cuda.device(self.device):
            for q in self._opened:
                lib.akv_ipc_close(q)
            dist.barrier(group=self.group)
            lib.akv_peer_free(self.base)
        self.base = None


def sequence_split_decode(query: torch.Tensor, hot_keys: Optional[torch.Tensor],
                          hot_values: Optional[torch.Tensor], warm, world: int,
                          sm_scale: Optional[float] = None, process_group=None,
                          partial: Optional[Callable] = None, all_gather: Optional[Callable] = None,
                          combine: Optional[Callable] = None,
                          exchange: Optional[PeerExchange] = None) -> torch.Tensor:
    """Decode attention of one sequence whose tokens are spread over ``world`` GPUs.

    Each GPU passes the tokens it holds (its contiguous share of warm blocks,
    and the hot window on whichever GPU keeps it; others pass None).  Returns
    (B, Hq, D) fp16 on every GPU."""
    partial = partial or local_partial
    if exchange is not None:  # NVLink peer memory: publish + wait-and-merge, no collective call
        p = partial(query, hot_keys, hot_values, warm, sm_scale)
        q3 = query.reshape(query.shape[0], query.shape[1], query.shape[-1])
        return exchange.exchange(p).reshape(q3.shape)
    all_gather = all_gather or (lambda t: _all_gather(t, world, process_group))
    combine = combine or combine_partials
    p = partial(query, hot_keys, hot_values, warm, sm_scale)
    gathered = all_gather(p)           # (world, rows, D+2)
    part = gathered.permute(1, 0, 2)   # (rows, world, D+2), a strided view
    q3 = query.reshape(query.shape[0], query.shape[1], query.shape[-1])
    return combine(part).reshape(q3.shape)
