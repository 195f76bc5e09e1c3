"""GPU: the three-tier manager (akv.migration.TierManager) through a
config-4-style cycle: per-step importance from attention in which 5 % of the
hot tokens carry 80 % of the mass, a demote pass every 32 steps (hot -> warm
by importance, oldest warm blocks -> pinned INT2 cold tier, cold -> warm
restores), decode attention over hot + warm throughout.

Checks:
* every position sits in exactly one tier;
* attention equals fp32 attention over the dequantised warm tier and the hot
  tier (the cold tier is not attended, as in the reference's AdaptiveKVCache,
  akv/cache.py:197-227);
* after every cold block is restored, every warm record dequantises bit for
  bit to the oracle's quantisation of the original tokens at its slots: the
  cold round trip (device -> pinned host -> device, side stream) is exact.
"""
import numpy as np
import pytest
import torch

import oracle.akv_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _attention(g, B, H, N, hot_frac=0.05, mass=0.8):
    k = max(1, int(N * hot_frac))
    idx = torch.randperm(N, generator=g, device=DEV)[:k]
    p = torch.rand(B, H, 1, N, generator=g, device=DEV)
    p[..., idx] = 0.0
    p = p / p.sum(-1, keepdim=True) * (1 - mass)
    p[..., idx] += mass / k
    return p


def _warm_tokens(tm, layer):
    """(slots, positions) of the live warm tokens."""
    lay = tm.layers[layer]
    n = lay.arena.n_blocks
    masks = lay.arena.masks()[0, 0].cpu().numpy()
    valid = ((masks[:, None] >> np.arange(32)) & 1).astype(bool).reshape(-1)
    slots = np.arange(n * 32)[valid]
    pos = lay.slot_pos[: n * 32].cpu().numpy()[valid]
    return slots, pos


def _check_attention(tm, gt_k, gt_v, q):
    lay = tm.layers[0]
    out = tm.attend(0, q)
    slots, pos = _warm_tokens(tm, 0)
    keys, vals = [], []
    if slots.size:
        wk, wv = lay.arena.dequantize(tok_idx=torch.from_numpy(slots).to(DEV))
        keys.append(wk.cpu().numpy())
        vals.append(wv.cpu().numpy())
    keys.append(lay.hot_k[:, :, :lay.hot_len].cpu().numpy())
    vals.append(lay.hot_v[:, :, :lay.hot_len].cpu().numpy())
    ref = O.decode_attention(q.cpu().numpy(), np.concatenate(keys, 2), np.concatenate(vals, 2))
    return float(np.abs(out.float().cpu().numpy() - ref).max())


def test_tier_manager_cycle():
    from akv.migration import TierManager
    B, H, Hq, D = 2, 4, 8, 128
    g = torch.Generator(device=DEV).manual_seed(0)
    tm = TierManager(B, H, D, hot_capacity=512, warm_blocks=32, cold_blocks=24, key_bits=2, value_bits=2,
                     device=DEV)
    N0, steps, every = 384, 256, 32
    total = N0 + steps
    gt_k = torch.randn(B, H, total, D, generator=g, device=DEV).half()
    gt_v = torch.randn(B, H, total, D, generator=g, device=DEV).half()
    tm.append(0, gt_k[:, :, :N0], gt_v[:, :, :N0])
    errs = []
    for step in range(steps):
        t = N0 + step
        tm.append(0, gt_k[:, :, t:t + 1], gt_v[:, :, t:t + 1])
        tm.update_importance(0, _attention(g, B, H, tm.hot_len(0)))
        tm.advance_step()
        if (step + 1) % every == 0:
            pas = (step + 1) // every
            tm.demote(0, 96)
            if tm.warm_len_blocks(0) > 12:
                tm.evict(0, tm.warm_len_blocks(0) - 10)
            if pas % 2 == 0:
                tm.restore(0, 2)
            tm.end_pass()
            q = torch.randn(B, Hq, D, generator=g, device=DEV).half()
            errs.append(_check_attention(tm, gt_k, gt_v, q))
    assert tm.stats.warm_to_cold_count > 0 and tm.stats.cold_to_warm_count > 0
    assert tm.cold_len_blocks(0) > 0
    # every position in exactly one tier
    pos = tm.positions(0)
    allpos = np.sort(np.concatenate([pos["hot"], pos["warm"], pos["cold"]]))
    np.testing.assert_array_equal(allpos, np.arange(total))
    assert max(errs) <= 2e-3, errs
    # restore everything, then every warm record is the oracle's quantisation of its tokens
    tm.restore(0, tm.cold_len_blocks(0))
    tm.flush()
    torch.cuda.synchronize()
    lay = tm.layers[0]
    n = lay.arena.n_blocks
    slot_pos = lay.slot_pos[: n * 32].cpu().numpy()
    masks = lay.arena.masks()[0, 0].cpu().numpy()
    gk, gv = gt_k.cpu().numpy(), gt_v.cpu().numpy()
    for j in range(n):
        m = int(masks[j])
        cnt = bin(m).count("1")
        assert m == (1 << cnt) - 1  # demoted blocks fill their slots from 0
        p = slot_pos[j * 32:j * 32 + cnt]
        wk, wv = lay.arena.dequantize(tok_idx=torch.arange(j * 32, j * 32 + cnt, device=DEV))
        rk = O.dequantize_groups(O.quantize_groups(gk[:, :, p], 2, 32, True))
        rv = O.dequantize_groups(O.quantize_groups(gv[:, :, p], 2, 32, False))
        np.testing.assert_array_equal(wk.cpu().numpy().view(np.uint16), rk.view(np.uint16))
        np.testing.assert_array_equal(wv.cpu().numpy().view(np.uint16), rv.view(np.uint16))
    pos = tm.positions(0)
    assert pos["cold"].size == 0
    np.testing.assert_array_equal(np.sort(np.concatenate([pos["hot"], pos["warm"]])), np.arange(total))
    q = torch.randn(B, Hq, D, generator=g, device=DEV).half()
    assert _check_attention(tm, gt_k, gt_v, q) <= 2e-3
