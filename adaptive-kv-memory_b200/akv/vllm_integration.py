"""vLLM-style engine over the paged warm pool (reference akv/vllm_integration.py).

The reference's ``AdaptiveCacheEngine`` keeps one cache object per sequence
and its ``AdaptiveAttentionBackend.forward(query, seq_id, layer_idx,
sm_scale)`` (vllm_integration.py:304-343) attends one sequence at a time.
Here the engine keeps, per layer,

* a slot-indexed FP16 hot pool ``(max_seqs, Hkv, hot_budget_per_seq, D)``
  with a per-slot length, and
* one ``PagedWarmPool`` of block records shared by all sequences, with a
  per-slot block table (int32 ``(max_seqs, max_blocks)``) and block count,

so ``AdaptiveAttentionBackend.forward_batch`` attends a whole batch of
sequences, each over its own hot window and its own warm pages, in one
``akv_mixed_decode_paged`` launch.  ``forward`` keeps the reference
signature for one sequence.

Tier policy (``update``): new tokens join the hot window; when a sequence's
hot window would exceed ``hot_budget_per_seq``, its oldest tokens after the
``initial_tokens_protected`` first ones are demoted, at least
``eviction_batch_size`` at a time (as many as the recent-token protection
allows), quantised into freshly allocated pages with one K scale per
32-token block.  The hot rows of a slot are kept in any order (attention
over them is order-free) with each row's token position on the host: a
demotion quantises the oldest rows straight from the hot pool (the
quantiser gathers them by index) and moves only as many of the newest rows
into the freed rows, so the valid rows stay a prefix; nothing else of the
window is copied.  The first ``initial_tokens_protected`` rows never move.  Warm pages per sequence are bounded by
``warm_budget_per_seq``; this engine has no cold tier (the INT2 cold tier of
``akv.tiering`` serves ``AKVCache``), so a sequence that outgrows its warm
budget raises.  ``AdaptiveKVLLM`` / ``patch_vllm_model_runner`` of the
reference wrap a vLLM ``LLM`` object (serving layer) and are not part of
this package.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np
import torch

from . import _C
from .fused_attention import KERNEL_HEAD_DIM, prefill_attention
from .paged import PagedWarmPool, paged_decode_attention
from .packed_layout import BLOCK


def _pinned(values: list, dtype) -> torch.Tensor:
    """Host values staged in pinned memory, so their copy to the device is
    asynchronous (a copy from pageable memory waits for the stream)."""
    return torch.tensor(values, dtype=dtype).pin_memory()


@dataclass
class AdaptiveVLLMConfig:
    """Engine configuration; fields and defaults of the reference
    (vllm_integration.py:48-75) plus the B200 engine's own sizes."""
    hot_budget_per_seq: int = 1024
    warm_budget_per_seq: int = 4096
    cold_budget_per_seq: int = 8192
    warm_bits: int = 4
    cold_bits: int = 2
    group_size: int = 128
    eviction_trigger_ratio: float = 0.9
    eviction_batch_size: int = 64
    initial_tokens_protected: int = 4
    recent_tokens_protected: int = 32
    importance_decay: float = 0.95
    enable_cold_tier: bool = True
    enable_async_migration: bool = True
    migration_stream: bool = True
    prefetch_cold_tokens: int = 16
    # B200 engine
    max_seqs: int = 64
    warm_key_bits: Optional[int] = None
    warm_value_bits: Optional[int] = None
    outlier_fraction: float = 0.0
    pool_pages: Optional[int] = None  # pages per layer (default: max_seqs x warm budget in blocks)


class _LayerState:
    def __init__(self, cfg: AdaptiveVLLMConfig, kv_heads: int, head_dim: int, dtype, device):
        S = cfg.max_seqs
        self.max_blocks = (cfg.warm_budget_per_seq + BLOCK - 1) // BLOCK + 1
        kb = cfg.warm_key_bits or cfg.warm_bits
        vb = cfg.warm_value_bits or cfg.warm_bits
        pages = cfg.pool_pages or S * self.max_blocks
        self.pool = PagedWarmPool(pages, kv_heads, head_dim, kb, vb, cfg.outlier_fraction, device=device)
        self.hot_k = torch.zeros(S, kv_heads, cfg.hot_budget_per_seq, head_dim, dtype=dtype, device=device)
        self.hot_v = torch.zeros_like(self.hot_k)
        self.hot_len = [0] * S
        self.row_pos = np.zeros((S, cfg.hot_budget_per_seq), dtype=np.int64)  # token position of each hot row
        self.seen = [0] * S                      # tokens fed so far (the next position)
        self.pages = [[] for _ in range(S)]      # block table rows (host)
        self.events = [[] for _ in range(S)]     # (first block, tokens) of each demote event
        self.table = torch.zeros(S, self.max_blocks, dtype=torch.int32, device=device)
        self.hot_len_dev = torch.zeros(S, dtype=torch.int32, device=device)
        self.warm_len_dev = torch.zeros(S, dtype=torch.int32, device=device)

    def sync_lengths(self, slot: int) -> None:
        self.hot_len_dev[slot:slot + 1].copy_(_pinned([self.hot_len[slot]], torch.int32),
                                              non_blocking=True)
        self.warm_len_dev[slot:slot + 1].copy_(_pinned([len(self.pages[slot])], torch.int32),
                                               non_blocking=True)

    def reset(self, slot: int) -> None:
        self.pool.release(self.pages[slot])
        self.pages[slot], self.events[slot], self.hot_len[slot], self.seen[slot] = [], [], 0, 0
        self.sync_lengths(slot)

    def chronological(self, slot: int) -> np.ndarray:
        """The slot's hot rows in token order."""
        h = self.hot_len[slot]
        return np.argsort(self.row_pos[slot, :h], kind="stable")


class AdaptiveCacheEngine:
    """Per-layer slot-indexed hot pools and paged warm pools for up to
    ``config.max_seqs`` sequences (reference vllm_integration.py:96-290)."""

    def __init__(self, config: AdaptiveVLLMConfig, num_layers: int, num_heads: int, head_dim: int,
                 dtype: torch.dtype = torch.float16, device: str = "cuda"):
        self.config = config
        self.num_layers, self.num_heads, self.head_dim = num_layers, num_heads, head_dim
        self.dtype, self.device = dtype, torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("AdaptiveCacheEngine keeps its tiers on a CUDA device (no CPU fallback)")
        self._layers = [_LayerState(config, num_heads, head_dim, dtype, self.device) for _ in range(num_layers)]
        self._slot: dict = {}
        self._free_slots = list(range(config.max_seqs - 1, -1, -1))
        self._total_sequences = 0
        self._total_migrations = 0

    # ------------------------------------------------------------------ sequences
    @property
    def _active_sequences(self) -> int:
        return len(self._slot)

    def allocate(self, seq_id: int) -> None:
        """A slot for a new sequence (an existing one is reset)."""
        if seq_id in self._slot:
            for L in self._layers:
                L.reset(self._slot[seq_id])
            return
        if not self._free_slots:
            raise RuntimeError(f"all {self.config.max_seqs} sequence slots are in use")
        slot = self._free_slots.pop()
        self._slot[seq_id] = slot
        for L in self._layers:
            L.reset(slot)
        self._total_sequences += 1

    def free(self, seq_id: int) -> None:
        """Release a finished sequence's slot and warm pages."""
        slot = self._slot.pop(seq_id, None)
        if slot is None:
            return
        for L in self._layers:
            L.reset(slot)
        self._free_slots.append(slot)

    def get_cache(self, seq_id: int) -> Optional[int]:
        """The sequence's slot (None if it has none)."""
        return self._slot.get(seq_id)

    # ------------------------------------------------------------------ tiers
    def update(self, seq_id: int, key_states: torch.Tensor, value_states: torch.Tensor, layer_idx: int,
               attention_weights: Optional[torch.Tensor] = None):
        """Append (1, Hkv, N, D) K/V of one sequence at one layer and demote
        beyond the hot budget.  Returns the sequence's hot window (1, Hkv,
        hot_len, D) K and V, its rows in pool order (not token order); its
        warm tokens stay packed in the pool."""
        _C.require_cuda(key_states, value_states)
        if seq_id not in self._slot:
            self.allocate(seq_id)
        slot = self._slot[seq_id]
        L = self._layers[layer_idx]
        cfg = self.config
        h, N = L.hot_len[slot], key_states.shape[2]
        total = h + N
        budget = cfg.hot_budget_per_seq
        pos0 = L.seen[slot]
        L.seen[slot] = pos0 + N
        if total <= budget:
            L.hot_k[slot, :, h:total] = key_states[0]
            L.hot_v[slot, :, h:total] = value_states[0]
            L.row_pos[slot, h:total] = np.arange(pos0, pos0 + N)
            L.hot_len[slot] = total
        else:
            init = min(cfg.initial_tokens_protected, budget)
            movable = max(0, total - init - cfg.recent_tokens_protected)
            n_dem = min(max(total - budget, cfg.eviction_batch_size), max(movable, total - budget))
            nblk = (n_dem + BLOCK - 1) // BLOCK
            if len(L.pages[slot]) + nblk > L.max_blocks:
                raise RuntimeError(f"sequence {seq_id} exceeds its warm budget of "
                                   f"{cfg.warm_budget_per_seq} tokens at layer {layer_idx}")
            pages = L.pool.alloc(nblk)
            dev = L.hot_k.device
            if n_dem <= h - init:  # the demoted tokens are all in the window: gather, no copy of it
                pos = L.row_pos[slot]
                cand = np.argpartition(pos[init:h], n_dem - 1)[:n_dem] + init if n_dem < h - init \
                    else np.arange(init, h)
                dem = cand[np.argsort(pos[cand], kind="stable")]  # the n_dem oldest rows, in token order
                L.pool.write(L.hot_k[slot:slot + 1], L.hot_v[slot:slot + 1], pages, group=BLOCK,
                             tok_idx=_pinned(dem.tolist(), torch.int64).to(dev, non_blocking=True))
                new_h = h - n_dem
                is_dem = np.zeros(h, dtype=bool)
                is_dem[dem] = True
                holes = dem[dem < new_h]
                movers = np.nonzero(~is_dem[new_h:h])[0] + new_h
                if holes.size:
                    both = _pinned(np.concatenate([movers, holes]).tolist(), torch.int64).to(dev, non_blocking=True)
                    src, dst = both[:holes.size], both[holes.size:]
                    for buf in (L.hot_k, L.hot_v):
                        buf[slot].index_copy_(1, dst, buf[slot].index_select(1, src))
                    pos[holes] = pos[movers]
                L.hot_k[slot, :, new_h:new_h + N] = key_states[0]
                L.hot_v[slot, :, new_h:new_h + N] = value_states[0]
                pos[new_h:new_h + N] = np.arange(pos0, pos0 + N)
                L.hot_len[slot] = new_h + N
            else:  # a prompt chunk longer than the window: some new tokens go straight to the warm tier
                order = _pinned(L.chronological(slot).tolist(), torch.int64).to(dev, non_blocking=True)
                ck = torch.cat([L.hot_k[slot, :, :h].index_select(1, order), key_states[0]], dim=1)
                cv = torch.cat([L.hot_v[slot, :, :h].index_select(1, order), value_states[0]], dim=1)
                cpos = np.concatenate([np.sort(L.row_pos[slot, :h]), np.arange(pos0, pos0 + N)])
                L.pool.write(ck[None, :, init:init + n_dem], cv[None, :, init:init + n_dem], pages, group=BLOCK)
                keep = total - n_dem
                L.hot_k[slot, :, :init] = ck[:, :init]
                L.hot_v[slot, :, :init] = cv[:, :init]
                L.hot_k[slot, :, init:keep] = ck[:, init + n_dem:]
                L.hot_v[slot, :, init:keep] = cv[:, init + n_dem:]
                L.row_pos[slot, :init] = cpos[:init]
                L.row_pos[slot, init:keep] = cpos[init + n_dem:]
                L.hot_len[slot] = keep
            first = len(L.pages[slot])
            L.table[slot, first:first + nblk].copy_(_pinned(pages, torch.int32), non_blocking=True)
            L.pages[slot].extend(pages)
            L.events[slot].append((first, n_dem))
            self._total_migrations += 1
        L.sync_lengths(slot)
        return L.hot_k[slot:slot + 1, :, :L.hot_len[slot]], L.hot_v[slot:slot + 1, :, :L.hot_len[slot]]

    def get_kv_for_attention(self, seq_id: int, layer_idx: int):
        """Full FP16 K/V (1, Hkv, T, D) of a sequence in token order: protected
        prefix, dequantised warm tokens, then the rest of the hot window."""
        slot = self._slot.get(seq_id)
        if slot is None or layer_idx >= self.num_layers:
            return None, None
        L = self._layers[layer_idx]
        init = min(self.config.initial_tokens_protected, self.config.hot_budget_per_seq)
        hl = L.hot_len[slot]
        order = torch.from_numpy(L.chronological(slot)).to(L.hot_k.device)
        hk, hv = L.hot_k[slot:slot + 1].index_select(2, order), L.hot_v[slot:slot + 1].index_select(2, order)
        ks, vs = [hk[:, :, :min(init, hl)]], [hv[:, :, :min(init, hl)]]
        for first, n in L.events[slot]:
            nb = (n + BLOCK - 1) // BLOCK
            k, v = L.pool.dequantize(L.pages[slot][first:first + nb], n_tokens=n)
            ks.append(k)
            vs.append(v)
        ks.append(hk[:, :, min(init, hl):hl])
        vs.append(hv[:, :, min(init, hl):hl])
        return torch.cat(ks, 2), torch.cat(vs, 2)

    # ------------------------------------------------------------------ accounting
    def memory_usage(self) -> dict:
        """Aggregate tier sizes (reference keys, MB)."""
        mb = 1 / (1024 * 1024)
        hot = warm = 0
        for L in self._layers:
            for slot in self._slot.values():
                hot += L.hot_len[slot] * self.num_heads * self.head_dim * 2 * 2
                warm += len(L.pages[slot]) * self.num_heads * L.pool.rec
        return {"active_sequences": self._active_sequences, "total_hot_mb": round(hot * mb, 2),
                "total_warm_mb": round(warm * mb, 2), "total_cold_mb": 0.0,
                "total_mb": round((hot + warm) * mb, 2), "total_migrations": self._total_migrations}

    def stats(self) -> dict:
        return {"active_sequences": self._active_sequences, "total_sequences_served": self._total_sequences,
                "total_migrations": self._total_migrations, "memory": self.memory_usage()}


class AdaptiveAttentionBackend:
    """Decode attention over the engine's tiers (reference vllm_integration.py:293-343)."""

    def __init__(self, cache_engine: AdaptiveCacheEngine):
        self.cache_engine = cache_engine

    def forward_batch(self, query: torch.Tensor, seq_ids: Sequence[int], layer_idx: int,
                      sm_scale: Optional[float] = None) -> torch.Tensor:
        """One decode query per sequence, (S, Hq, D) fp16 -> (S, Hq, D) fp16,
        every sequence over its hot window and its warm pages, one launch."""
        eng = self.cache_engine
        L = eng._layers[layer_idx]
        slots = [eng._slot[s] for s in seq_ids]
        S = len(slots)
        if slots == list(range(S)):
            rows, q = S, query
        else:
            rows = max(slots) + 1
            q = torch.zeros(rows, *query.shape[1:], dtype=query.dtype, device=query.device)
            idx = _pinned(slots, torch.int64).to(query.device, non_blocking=True)
            q.index_copy_(0, idx, query)
        out = paged_decode_attention(q, L.hot_k[:rows], L.hot_v[:rows], L.hot_len_dev[:rows], L.pool,
                                     L.table[:rows], L.warm_len_dev[:rows], sm_scale=sm_scale)
        if rows != S or slots != list(range(S)):
            out = out.index_select(0, _pinned(slots, torch.int64).to(query.device, non_blocking=True))
        return out

    def forward(self, query: torch.Tensor, seq_id: int, layer_idx: int,
                sm_scale: Optional[float] = None) -> torch.Tensor:
        """Reference signature: query (1, Hq, M, D) -> (1, Hq, M, D).  M = 1
        runs the paged decode kernel; M > 1 attends every query over the
        sequence's full K/V without a mask, as the reference's fallback does
        (vllm_integration.py:331-343): the tcgen05 prefill kernel with every
        key visible to every query at head dim 128, else fp32 torch."""
        eng = self.cache_engine
        if eng.get_cache(seq_id) is None:
            raise ValueError(f"No cache for seq_id={seq_id}")
        if query.shape[2] == 1:
            return self.forward_batch(query[:, :, 0], [seq_id], layer_idx, sm_scale).unsqueeze(2)
        k, v = eng.get_kv_for_attention(seq_id, layer_idx)
        if query.shape[-1] == KERNEL_HEAD_DIM and query.dtype == torch.float16:
            M, T = query.shape[2], k.shape[2]
            q_pos = torch.full((M,), T, dtype=torch.int32, device=query.device)  # sees keys 0 .. T
            k_pos = torch.arange(T, dtype=torch.int32, device=query.device)
            return prefill_attention(query, q_pos, k, v, k_pos, sm_scale=sm_scale)
        g = query.shape[1] // k.shape[1]
        k, v = k.repeat_interleave(g, dim=1), v.repeat_interleave(g, dim=1)
        if sm_scale is None:
            sm_scale = 1.0 / math.sqrt(query.shape[-1])
        p = torch.softmax(torch.matmul(query.float(), k.float().transpose(-2, -1)) * sm_scale, dim=-1)
        return torch.matmul(p, v.float()).to(query.dtype)
