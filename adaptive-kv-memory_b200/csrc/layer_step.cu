// Steady-state decode step of one AKVLayer in a single host call.
//
// Once a layer's hot tier is full and only recency importance decides what
// leaves it (no promotion), every decode step does the same bookkeeping:
// decay the hot tokens' importance, pick the least important unprotected
// token, quantise its K / V rows into a new warm record, write the new
// token into the ring row it leaves, and update the host vectors that keep
// the hot tier's logical order and the warm tier's slots and positions.
// Issued from Python this costs tens of microseconds per layer; here it is
// one call that does the host arithmetic in place and issues the launches.
#include <cuda_runtime.h>

#include "akv_b200.h"

extern "C" int akv_layer_decode_step(akv_layer_step* c, const uint16_t* new_k, int64_t nk_sb, int64_t nk_sh,
                                     const uint16_t* new_v, int64_t nv_sb, int64_t nv_sh, void* stream) {
  if (!c || !new_k || !new_v || !c->hot_k || !c->hot_v || !c->arena || !c->phys || !c->hpos || !c->imp ||
      !c->wslots || !c->wpos || !c->slot_pos)
    return AKV_ERR_NULL;
  const int64_t lo = c->lo, hi = c->hi, n = hi - lo;
  const int64_t hot_len = n + 1;
  const int64_t lim = hot_len - c->protect_recent;
  // capacities the caller guarantees (checked, never exceeded)
  if (n <= 0 || hi + 1 > c->cap || c->protect_first < 0 || lim <= c->protect_first) return AKV_ERR_SHAPE;
  if (c->n_blocks + 1 > c->max_blocks || c->n_wslots + 1 > c->cap_wslots || c->n_wpos + 1 > c->cap_wpos ||
      (static_cast<int64_t>(c->n_blocks) + 1) * AKV_BLOCK_TOKENS > c->cap_slot_pos)
    return AKV_ERR_SHAPE;
  float* imp = c->imp;
  int64_t* pos = c->hpos;
  int64_t* phys = c->phys;

  // recency importance (AKVLayer._update_importance: scores * decay, the new
  // token at 1.0; one fp32 rounding each) and the new token's position
  const float decay = c->decay;
  for (int64_t i = lo; i < hi; ++i) imp[i] = imp[i] * decay;
  imp[hi] = 1.0f;
  pos[hi] = c->total_len;

  // the demoted token: first index of the minimum over the unprotected
  // scores (torch.topk(1, largest=False) on the CPU for 64+ scores)
  int64_t v0 = c->protect_first;
  float best = imp[lo + v0];
  for (int64_t i = v0 + 1; i < lim; ++i)
    if (imp[lo + i] < best) {
      best = imp[lo + i];
      v0 = i;
    }
  const int64_t r = phys[lo + v0];
  const int64_t vpos = pos[lo + v0];
  if (r < 0 || r >= c->hot_rows) return AKV_ERR_SHAPE;

  // its K / V rows into a new record (one group of one token), and the new
  // token written over them in ring row r: one launch (the record is read
  // before the row is overwritten inside each CTA)
  const int blk = c->n_blocks;
  uint16_t* kr = c->hot_k + r * c->h_sn;
  uint16_t* vr = c->hot_v + r * c->h_sn;
  const int rc = akv_warm_demote_install(c->arena, c->a_sb, c->a_sh, &c->layout, blk, kr, c->h_sb, c->h_sh, vr,
                                         c->h_sb, c->h_sh, new_k, nk_sb, nk_sh, new_v, nv_sb, nv_sh, c->B, c->H,
                                         c->status, stream);
  if (rc != AKV_OK) return rc;

  // warm-side host vectors
  c->wslots[c->n_wslots++] = static_cast<int64_t>(blk) * AKV_BLOCK_TOKENS;
  c->wpos[c->n_wpos++] = vpos;
  c->slot_pos[static_cast<int64_t>(blk) * AKV_BLOCK_TOKENS] = static_cast<int32_t>(vpos);
  c->n_blocks = blk + 1;
  c->warm_len += 1;
  c->warm_bytes_packed += c->bytes_per_event;
  c->total_len += 1;
  c->step += 1;

  // logical order: drop entry v0 of importance / positions (n + 1 entries
  // with the new token) and of the rows (n entries), the new token's row r
  // last; the shorter side moves, so all three keep one [lo, hi)
  if (v0 < n / 2) {
    for (int64_t i = v0; i > 0; --i) {
      imp[lo + i] = imp[lo + i - 1];
      pos[lo + i] = pos[lo + i - 1];
      phys[lo + i] = phys[lo + i - 1];
    }
    phys[hi] = r;
    c->lo = lo + 1;
    c->hi = hi + 1;
  } else {
    for (int64_t i = v0; i < n; ++i) {
      imp[lo + i] = imp[lo + i + 1];
      pos[lo + i] = pos[lo + i + 1];
    }
    for (int64_t i = v0; i < n - 1; ++i) phys[lo + i] = phys[lo + i + 1];
    phys[hi - 1] = r;
  }
  return AKV_OK;
}
