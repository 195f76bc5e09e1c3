"""Three-tier KV manager with an INT2 cold tier in pinned host memory.

The reference moves tokens between tiers in two places: ``AdaptiveKVCache``
demotes hot tokens to a quantised warm tier and to a CPU cold tier that
attention skips (akv/cache.py:243-327, get_kv :197-227), and
``AsyncMigrator`` queues hot->warm / warm->cold / cold->warm moves on side
CUDA streams (akv/async_migration.py:163-241, :303-349; its ``pin_memory``
flag, :102, is never used).  ``TierManager`` is that manager for the packed
warm tier of this build, per layer:

* hot:   FP16 rows (B, H, cap, D) with an int64 position per row and GPU
         importance scores (``tiering.ImportanceMigrator``: decay x old score
         + attention sum + recency, akv/vmm.py:121-219);
* warm:  a ``WarmArena`` of 32-token block records (2-bit by default, the
         compact preset), live blocks kept dense in [0, n_blocks) so the
         decode kernel streams exactly the live records; an int64 position
         per record slot;
* cold:  the same records byte for byte in a pinned host arena
         (B, H, cold_blocks, rec), never attended (as the reference's cold
         tier).

Moves:

* ``demote(layer, n)``: the n least important hot tokens are quantised in
  place (fused gather) into new warm records, one scale group per 32-token
  block, and the hot tier is compacted (rows, positions, scores);
* ``evict(layer, k)``: the k oldest warm blocks are copied to the cold arena
  with ``cudaMemcpy2DAsync`` on a side stream after an event from the compute
  stream; the compute stream waits on the copy's event before the holes are
  refilled by moving the last live blocks into them (no host synchronisation);
* ``restore(layer, k)``: the k most recently evicted cold blocks are copied
  back to the end of the warm arena on the side stream, and the compute stream
  waits on that copy before its next attention.

The record bytes never change on the way (no requantisation: the records
already hold the 2-bit codes), so a cold round trip is bit-exact.  No batched
memcpy call is used: one ``cudaMemcpy2DAsync`` per block move.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional

import numpy as np
import torch

from . import _C, tiering
from .packed_layout import BLOCK, WarmArena


@dataclass
class MigrationStats:
    """Counters in the reference's MigrationStats vocabulary (async_migration.py:58-78)."""
    hot_to_warm_count: int = 0
    warm_to_cold_count: int = 0
    cold_to_warm_count: int = 0
    total_demotions: int = 0
    total_promotions: int = 0
    total_tokens_migrated: int = 0
    cold_bytes_d2h: int = 0
    cold_bytes_h2d: int = 0


@dataclass
class _Layer:
    hot_k: torch.Tensor
    hot_v: torch.Tensor
    hot_pos: torch.Tensor          # int64 (cap,)
    hot_len: int
    next_pos: int                  # position of the next appended token
    arena: WarmArena
    slot_pos: torch.Tensor         # int64 (max_blocks * 32,) position of each warm slot
    blk_age: List[int] = field(default_factory=list)  # demote pass that created warm block j
    cold: Optional[torch.Tensor] = None               # pinned (B, H, cold_cap, rec) uint8
    cold_pos: Optional[torch.Tensor] = None           # pinned int64 (cold_cap, 32)
    cold_used: List[int] = field(default_factory=list)  # cold slots in eviction order (oldest first)
    cold_free: List[int] = field(default_factory=list)


class TierManager:
    """Hot FP16 ring + packed warm arena + pinned INT2 cold arena, per layer."""

    def __init__(self, batch: int, kv_heads: int, head_dim: int = 128, hot_capacity: int = 4096,
                 warm_blocks: int = 1024, cold_blocks: int = 256, key_bits: int = 2, value_bits: int = 2,
                 outlier_fraction: float = 0.0, importance_decay: float = 0.9, device="cuda"):
        self.B, self.H, self.D = batch, kv_heads, head_dim
        self.hot_capacity, self.warm_blocks, self.cold_blocks = hot_capacity, warm_blocks, cold_blocks
        self.key_bits, self.value_bits, self.outlier_fraction = key_bits, value_bits, outlier_fraction
        self.device = torch.device(device)
        self.layers: List[_Layer] = []
        self.importance = tiering.ImportanceMigrator(importance_decay=importance_decay, device=self.device)
        self.side = torch.cuda.Stream(device=self.device)  # cold-tier copies
        self.stats = MigrationStats()
        self._pass = 0

    # ------------------------------------------------------------------ state
    def _layer(self, idx: int) -> _Layer:
        while len(self.layers) <= idx:
            B, H, D = self.B, self.H, self.D
            cap = self.hot_capacity
            arena = WarmArena(B, H, D, self.key_bits, self.value_bits, self.outlier_fraction,
                              max_blocks=self.warm_blocks, device=self.device)
            lay = _Layer(hot_k=torch.zeros(B, H, cap, D, dtype=torch.float16, device=self.device),
                         hot_v=torch.zeros(B, H, cap, D, dtype=torch.float16, device=self.device),
                         hot_pos=torch.zeros(cap, dtype=torch.int64, device=self.device), hot_len=0, next_pos=0,
                         arena=arena,
                         slot_pos=torch.full((self.warm_blocks * BLOCK,), -1, dtype=torch.int64,
                                             device=self.device))
            if self.cold_blocks > 0:
                lay.cold = torch.zeros(B, H, self.cold_blocks, arena.rec, dtype=torch.uint8).pin_memory()
                lay.cold_pos = torch.full((self.cold_blocks, BLOCK), -1, dtype=torch.int64).pin_memory()
                lay.cold_free = list(range(self.cold_blocks - 1, -1, -1))
            self.layers.append(lay)
        return self.layers[idx]

    def hot_len(self, layer: int) -> int:
        return self._layer(layer).hot_len

    def warm_len_blocks(self, layer: int) -> int:
        return self._layer(layer).arena.n_blocks

    def cold_len_blocks(self, layer: int) -> int:
        return len(self._layer(layer).cold_used)

    # ------------------------------------------------------------------ append / attend
    def append(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Append (B, H, n, D) fp16 K/V rows to the hot tier at the layer's next n positions."""
        _C.require_cuda(k, v)
        lay = self._layer(layer)
        n = k.shape[2]
        if lay.hot_len + n > self.hot_capacity:
            raise RuntimeError(f"hot tier full ({lay.hot_len}+{n} > {self.hot_capacity}); demote first")
        lay.hot_k[:, :, lay.hot_len:lay.hot_len + n].copy_(k)
        lay.hot_v[:, :, lay.hot_len:lay.hot_len + n].copy_(v)
        lay.hot_pos[lay.hot_len:lay.hot_len + n] = torch.arange(lay.next_pos, lay.next_pos + n, device=self.device)
        lay.hot_len += n
        lay.next_pos += n

    def load_warm(self, layer: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Quantise (B, H, n, D) K/V straight into warm records at the layer's
        next n positions (a prefill demotion; one scale group per 32 tokens)."""
        _C.require_cuda(k, v)
        lay = self._layer(layer)
        n = k.shape[2]
        nblk = (n + BLOCK - 1) // BLOCK
        arena = lay.arena
        if arena.n_blocks + nblk > arena.max_blocks:
            raise RuntimeError("warm tier full")
        blk0 = arena.append(k, v, group=BLOCK)
        lay.slot_pos[blk0 * BLOCK:(blk0 + nblk) * BLOCK] = -1
        lay.slot_pos[blk0 * BLOCK:blk0 * BLOCK + n] = torch.arange(lay.next_pos, lay.next_pos + n, device=self.device)
        lay.blk_age += [self._pass] * nblk
        lay.next_pos += n

    def update_importance(self, layer: int, attention_weights: torch.Tensor) -> None:
        """Fold one step's (B, H, Q, hot_len) attention over the hot tier into its scores."""
        self.importance.update(layer, attention_weights, self._layer(layer).hot_len)

    def advance_step(self) -> None:
        self.importance.advance_step()

    def attend(self, layer: int, query: torch.Tensor, sm_scale: Optional[float] = None,
               out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Decode attention (B, Hq, D) over the hot rows and the live warm records (cold is not attended)."""
        from .fused_attention import mixed_tier_decode_attention
        lay = self._layer(layer)
        hk = lay.hot_k[:, :, :lay.hot_len] if lay.hot_len else None
        hv = lay.hot_v[:, :, :lay.hot_len] if lay.hot_len else None
        warm = lay.arena if lay.arena.n_blocks else None
        return mixed_tier_decode_attention(query, hk, hv, warm, sm_scale=sm_scale, out=out)

    # ------------------------------------------------------------------ moves
    def demote(self, layer: int, n: int) -> int:
        """Move the n least important hot tokens into new warm records.  Returns tokens moved."""
        lay = self._layer(layer)
        n = min(n, lay.hot_len)
        if n <= 0:
            return 0
        idx = self.importance.get_eviction_candidates(layer, lay.hot_len, n)
        n = idx.numel()
        if n == 0:
            return 0
        arena = lay.arena
        nblk = (n + BLOCK - 1) // BLOCK
        if arena.n_blocks + nblk > arena.max_blocks:
            raise RuntimeError("warm tier full; evict to the cold tier first")
        blk0 = arena.n_blocks
        hk, hv = lay.hot_k[:, :, :lay.hot_len], lay.hot_v[:, :, :lay.hot_len]
        arena.append(hk, hv, group=BLOCK, tok_idx=idx)
        lay.slot_pos[blk0 * BLOCK:(blk0 + nblk) * BLOCK] = -1  # slots past n stay empty
        lay.slot_pos[blk0 * BLOCK:blk0 * BLOCK + n].copy_(lay.hot_pos[idx])
        lay.blk_age += [self._pass] * nblk
        # compact the hot tier: rows, positions and scores of the kept tokens
        keep = torch.ones(lay.hot_len, dtype=torch.bool, device=self.device)
        keep[idx] = False
        kidx = keep.nonzero().squeeze(1)
        m = kidx.numel()
        lay.hot_k[:, :, :m] = tiering.gather_rows(hk, kidx)
        lay.hot_v[:, :, :m] = tiering.gather_rows(hv, kidx)
        lay.hot_pos[:m] = lay.hot_pos[kidx]
        self.importance.compact(layer, kidx)
        lay.hot_len = m
        self.stats.hot_to_warm_count += 1
        self.stats.total_demotions += 1
        self.stats.total_tokens_migrated += n
        return n

    def evict(self, layer: int, k: int) -> int:
        """Move the k oldest warm blocks to the pinned cold arena.  Returns blocks moved."""
        lay = self._layer(layer)
        arena = lay.arena
        k = min(k, arena.n_blocks, len(lay.cold_free))
        if k <= 0:
            return 0
        ages = np.asarray(lay.blk_age[:arena.n_blocks])
        victims = sorted(np.argsort(ages, kind="stable")[:k].tolist())
        cur = torch.cuda.current_stream(self.device)
        self.side.wait_stream(cur)  # the records and positions are final on the compute stream
        rec, maxb = arena.rec, arena.max_blocks
        with torch.cuda.stream(self.side):
            for j in victims:
                c = lay.cold_free.pop()
                _C.check(_C.load().akv_cold_copy(lay.cold.data_ptr() + c * rec, self.cold_blocks * rec,
                                                 arena.buf.data_ptr() + j * rec, maxb * rec, rec,
                                                 self.B * self.H, 0, self.side.cuda_stream, None), "akv_cold_copy")
                lay.cold_pos[c].copy_(lay.slot_pos[j * BLOCK:(j + 1) * BLOCK], non_blocking=True)
                lay.cold_used.append(c)
        done = torch.cuda.Event()
        done.record(self.side)
        cur.wait_event(done)  # holes are refilled only after the copies have read them
        # refill holes with the last live blocks (dense [0, n_blocks) again)
        live = arena.n_blocks
        gone = set(victims)
        movers = [j for j in range(live - 1, -1, -1) if j not in gone][: sum(1 for j in victims if j < live - k)]
        holes = [j for j in victims if j < live - k]
        for dst, src in zip(holes, movers):
            arena.buf[:, :, dst].copy_(arena.buf[:, :, src])
            lay.slot_pos[dst * BLOCK:(dst + 1) * BLOCK].copy_(lay.slot_pos[src * BLOCK:(src + 1) * BLOCK])
            lay.blk_age[dst] = lay.blk_age[src]
        arena.n_blocks = live - k
        del lay.blk_age[arena.n_blocks:]
        nb = k * self.B * self.H * rec
        self.stats.warm_to_cold_count += 1
        self.stats.total_demotions += 1
        self.stats.total_tokens_migrated += k * BLOCK
        self.stats.cold_bytes_d2h += nb
        return k

    def restore(self, layer: int, k: int) -> int:
        """Bring the k most recently evicted cold blocks back to the end of the warm arena."""
        lay = self._layer(layer)
        arena = lay.arena
        k = min(k, len(lay.cold_used), arena.max_blocks - arena.n_blocks)
        if k <= 0:
            return 0
        cur = torch.cuda.current_stream(self.device)
        self.side.wait_stream(cur)  # the destination blocks are free on the compute stream
        rec, maxb = arena.rec, arena.max_blocks
        with torch.cuda.stream(self.side):
            for _ in range(k):
                c = lay.cold_used.pop()
                j = arena.n_blocks
                _C.check(_C.load().akv_cold_copy(arena.buf.data_ptr() + j * rec, maxb * rec,
                                                 lay.cold.data_ptr() + c * rec, self.cold_blocks * rec, rec,
                                                 self.B * self.H, 1, self.side.cuda_stream, None), "akv_cold_copy")
                lay.slot_pos[j * BLOCK:(j + 1) * BLOCK].copy_(lay.cold_pos[c], non_blocking=True)
                lay.cold_free.append(c)
                arena.n_blocks += 1
                lay.blk_age.append(self._pass)
        done = torch.cuda.Event()
        done.record(self.side)
        cur.wait_event(done)  # attention after this point sees the restored records
        self.stats.cold_to_warm_count += 1
        self.stats.total_promotions += 1
        self.stats.total_tokens_migrated += k * BLOCK
        self.stats.cold_bytes_h2d += k * self.B * self.H * rec
        return k

    def end_pass(self) -> None:
        """Close one demote / evict / restore pass (block ages count passes)."""
        self._pass += 1

    def flush(self) -> None:
        """Wait for every cold-tier copy issued so far (reference AsyncMigrator.flush)."""
        self.side.synchronize()

    # ------------------------------------------------------------------ reference-style names
    def schedule_demotion(self, layer_idx: int, num_tokens: int, target_tier: str = "warm") -> int:
        """hot -> warm (``num_tokens`` least important) or warm -> cold (whole oldest blocks)."""
        if target_tier == "warm":
            return self.demote(layer_idx, num_tokens)
        return self.evict(layer_idx, (num_tokens + BLOCK - 1) // BLOCK) * BLOCK

    def schedule_promotion(self, layer_idx: int, num_tokens: int, source_tier: str = "cold") -> int:
        """cold -> warm of whole blocks (the most recently evicted first)."""
        if source_tier != "cold":
            raise NotImplementedError("warm -> hot promotion lives in AKVCache (attention or proxy scores)")
        return self.restore(layer_idx, (num_tokens + BLOCK - 1) // BLOCK) * BLOCK

    @property
    def is_idle(self) -> bool:
        return self.side.query()

    # ------------------------------------------------------------------ inspection
    def positions(self, layer: int) -> dict:
        """Host copies of the positions held by each tier (after a flush)."""
        lay = self._layer(layer)
        torch.cuda.current_stream(self.device).synchronize()
        self.flush()
        n = lay.arena.n_blocks * BLOCK
        masks = lay.arena.masks()[0, 0].cpu().numpy() if lay.arena.n_blocks else np.zeros(0, np.int64)
        valid = ((masks[:, None] >> np.arange(BLOCK)) & 1).astype(bool).reshape(-1)
        warm = lay.slot_pos[:n].cpu().numpy()[valid]
        cold = np.concatenate([lay.cold_pos[c].numpy() for c in lay.cold_used]) if lay.cold_used else np.zeros(0, np.int64)
        cold = cold[cold >= 0]
        return {"hot": lay.hot_pos[:lay.hot_len].cpu().numpy(), "warm": warm, "cold": cold}
