"""Config-4-style migration stress, scaled down: per-step importance from
attention in which 5 % of tokens carry 80 % of the mass, a demote pass every
64 steps (importance bottom-k -> fused gather + 2-bit quantise into the warm
arena -> hot compaction), the oldest warm blocks moved to a pinned INT2 cold
tier on a side stream and restored, and a decode over what is left.

Checks: every token is in exactly one tier, the cold round trip is
byte-exact, the warm tier dequantises to the oracle's quantisation of the
demoted rows, and attention over [warm; hot] matches the fp32 oracle.
"""
import numpy as np
import pytest
import torch

import oracle.akv_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _attention(g, B, H, N, hot_frac=0.05, mass=0.8):
    """(B, H, 1, N) probabilities: a seeded 5 % of positions share 80 % of the mass."""
    k = max(1, int(N * hot_frac))
    idx = torch.randperm(N, generator=g, device=DEV)[:k]
    p = torch.rand(B, H, 1, N, generator=g, device=DEV)
    p[..., idx] = 0.0
    p = p / p.sum(-1, keepdim=True) * (1 - mass)
    p[..., idx] += mass / k
    return p


def test_migration_stress_cycle():
    import akv
    from akv import tiering
    B, H, D = 2, 4, 128
    g = torch.Generator(device=DEV).manual_seed(0)
    N0, steps, every, n_demote, cold_after = 512, 256, 64, 96, 4
    hot_k = torch.randn(B, H, N0, D, generator=g, device=DEV).half()
    hot_v = torch.randn(B, H, N0, D, generator=g, device=DEV).half()
    hot_pos = torch.arange(N0, device=DEV)
    arena = akv.WarmArena(B, H, D, 2, 2, 0.0, max_blocks=64, device=DEV)
    warm_pos, demoted_k, demoted_v = [], [], []
    cold = []  # (blk0, pinned host records)
    mig = tiering.ImportanceMigrator(importance_decay=0.9, device=DEV)
    side = torch.cuda.Stream(device=DEV)
    total = N0
    for step in range(steps):
        nk = torch.randn(B, H, 1, D, generator=g, device=DEV).half()
        nv = torch.randn(B, H, 1, D, generator=g, device=DEV).half()
        hot_k, hot_v = torch.cat([hot_k, nk], 2), torch.cat([hot_v, nv], 2)
        hot_pos = torch.cat([hot_pos, torch.tensor([total], device=DEV)])
        total += 1
        mig.update(0, _attention(g, B, H, hot_k.shape[2]), hot_k.shape[2])
        if (step + 1) % every == 0:
            n = hot_k.shape[2]
            idx = mig.get_eviction_candidates(0, n, n_demote)
            assert idx.numel() == n_demote and torch.all(idx[1:] > idx[:-1])
            demoted_k.append(hot_k[:, :, idx].clone())
            demoted_v.append(hot_v[:, :, idx].clone())
            arena.append(hot_k, hot_v, group=32, tok_idx=idx)
            warm_pos.append(hot_pos[idx])
            keep = torch.ones(n, dtype=torch.bool, device=DEV)
            keep[idx] = False
            kidx = keep.nonzero().squeeze(1)
            hot_k = tiering.gather_rows(hot_k, kidx)
            hot_v = tiering.gather_rows(hot_v, kidx)
            hot_pos = hot_pos[kidx]
            mig.reset()  # scores are per hot position; restart them after compaction
            if arena.n_blocks >= cold_after + 3 and not cold:
                host = torch.empty(B, H, 3, arena.rec, dtype=torch.uint8).pin_memory()
                ev = tiering.cold_copy_blocks(arena.buf, 0, 3, host, stream=side)
                cold.append((0, host, ev))
        mig.advance_step()

    # every token sits in exactly one tier
    wp = torch.cat(warm_pos)
    allpos = torch.cat([wp, hot_pos]).sort().values
    assert torch.equal(allpos.cpu(), torch.arange(total))
    # cold tier: byte-exact round trip of the first three blocks
    blk0, host, ev = cold[0]
    ev.synchronize()
    saved = arena.buf[:, :, :3].clone()
    arena.buf[:, :, :3].zero_()
    tiering.cold_restore_blocks(host, arena.buf, 0, stream=side).synchronize()
    assert torch.equal(arena.buf[:, :, :3], saved)
    # warm tier == the oracle's per-32-token-group quantisation of the demoted rows
    dk_all = torch.cat(demoted_k, 2).cpu().numpy()
    dv_all = torch.cat(demoted_v, 2).cpu().numpy()
    slots = []
    blk = 0
    for part in demoted_k:
        n = part.shape[2]
        slots.append(torch.arange(blk * 32, blk * 32 + n))
        blk += (n + 31) // 32
    slots = torch.cat(slots).to(DEV)
    wk, wv = arena.dequantize(tok_idx=slots)
    ref_k = np.concatenate([O.dequantize_groups(O.quantize_groups(p.cpu().numpy(), 2, 32, True))
                            for p in demoted_k], 2)
    ref_v = np.concatenate([O.dequantize_groups(O.quantize_groups(p.cpu().numpy(), 2, 32, False))
                            for p in demoted_v], 2)
    np.testing.assert_array_equal(wk.cpu().numpy().view(np.uint16), ref_k.view(np.uint16))
    np.testing.assert_array_equal(wv.cpu().numpy().view(np.uint16), ref_v.view(np.uint16))
    assert dk_all.shape[2] == wk.shape[2]
    # decode over [warm arena; hot] == fp32 oracle over the dequantised tiers
    q = torch.randn(B, 2 * H, D, generator=g, device=DEV).half()
    out = akv.mixed_tier_decode_attention(q, hot_k.contiguous(), hot_v.contiguous(), arena)
    ref = O.decode_attention(q.cpu().numpy(), np.concatenate([ref_k, hot_k.cpu().numpy()], 2),
                             np.concatenate([ref_v, hot_v.cpu().numpy()], 2))
    assert np.abs(out.float().cpu().numpy() - ref).max() <= 2e-3
