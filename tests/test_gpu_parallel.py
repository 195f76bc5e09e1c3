"""akv.parallel with the CUDA kernels, ranks emulated in one process on one
GPU (the collectives are replaced by their arithmetic: a sum for the
all-reduce, a stack for the all-gather; tests/test_parallel_gloo.py runs the
real collectives on CPU ranks).
"""
import numpy as np
import pytest
import torch

import oracle.akv_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _np(t):
    return t.detach().cpu().numpy()


def test_outlier_norm_sums_vs_oracle():
    from akv import _C
    rng = np.random.default_rng(0)
    B, H, N, D, G = 2, 4, 96, 128, 32
    x = rng.standard_normal((B, H, N, D)).astype(np.float16)
    x[..., 9] *= 12
    got = _np(_C.outlier_norm_sums(torch.from_numpy(x).to(DEV), None, N, G))
    for b in range(B):
        for g in range(N // G):
            ref = O.outlier_norm_sum(x[b, :, g * G:(g + 1) * G])
            np.testing.assert_allclose(got[b, g], ref, rtol=2e-6, atol=0)


@pytest.mark.parametrize("group,N", [(32, 96), (700, 700)])
def test_head_sharded_quantise_equals_unsharded(group, N):
    """Two 'ranks' holding 4 heads each == one arena over all 8 heads, bit for bit."""
    import akv
    from akv import parallel as P
    rng = np.random.default_rng(1)
    B, H, D = 2, 8, 128
    k = torch.from_numpy(rng.standard_normal((B, H, N, D)).astype(np.float16)).to(DEV)
    k[..., 40] *= 12
    v = torch.from_numpy(rng.standard_normal((B, H, N, D)).astype(np.float16)).to(DEV)
    nblk = (N + 31) // 32
    full = akv.WarmArena(B, H, D, 4, 2, 0.01, max_blocks=nblk, device=DEV)
    full.append(k, v, group=group)
    halves = [akv.WarmArena(B, H // 2, D, 4, 2, 0.01, max_blocks=nblk, device=DEV) for _ in range(2)]
    g = min(group, N)
    local = [[None, None], [None, None]]
    from akv import _C
    for r in range(2):  # every rank's local norm sums, then their all-reduce
        for i, x in enumerate((k, v)):
            local[r][i] = _C.outlier_norm_sums(x[:, 4 * r:4 * r + 4].contiguous(), None, N, g)
    reduced = [local[0][i] + local[1][i] for i in range(2)]
    for r in range(2):
        it = iter(reduced)
        P.quantize_head_sharded(halves[r], k[:, 4 * r:4 * r + 4].contiguous(), v[:, 4 * r:4 * r + 4].contiguous(),
                                total_heads=H, group=group, norm_sums=lambda x: next(it), all_reduce=lambda t: t)
    ref = _np(full.buf)
    for r in range(2):
        np.testing.assert_array_equal(_np(halves[r].buf), ref[:, 4 * r:4 * r + 4])


def test_sequence_split_partials_combine_to_full_decode():
    """Three 'ranks' with contiguous warm block ranges (hot on rank 0) == one decode."""
    import akv
    from akv import parallel as P
    rng = np.random.default_rng(2)
    B, Hq, Hkv, D, nblk, nh = 1, 16, 4, 128, 40, 100
    wk = torch.from_numpy(rng.standard_normal((B, Hkv, 32 * nblk, D)).astype(np.float16)).to(DEV)
    wv = torch.from_numpy(rng.standard_normal((B, Hkv, 32 * nblk, D)).astype(np.float16)).to(DEV)
    hk = torch.from_numpy(rng.standard_normal((B, Hkv, nh, D)).astype(np.float16)).to(DEV)
    hv = torch.from_numpy(rng.standard_normal((B, Hkv, nh, D)).astype(np.float16)).to(DEV)
    q = torch.from_numpy(rng.standard_normal((B, Hq, D)).astype(np.float16)).to(DEV)
    full = akv.WarmArena(B, Hkv, D, 4, 2, 0.01, max_blocks=nblk, device=DEV)
    full.append(wk, wv, group=32)
    ref = akv.mixed_tier_decode_attention(q, hk, hv, full)
    parts = []
    for r in range(3):
        lo, hi = P.ShardPlan("sequence", 3, r).span(nblk)
        a = akv.WarmArena(B, Hkv, D, 4, 2, 0.01, max_blocks=hi - lo, device=DEV)
        a.append(wk[:, :, 32 * lo:32 * hi], wv[:, :, 32 * lo:32 * hi], group=32)
        parts.append(P.local_partial(q, hk if r == 0 else None, hv if r == 0 else None, a))
    parts.append(P.local_partial(q, None, None, None))  # a rank with nothing
    out = P.sequence_split_decode(q, None, None, None, 4, partial=lambda *a: parts.pop(0),
                                  all_gather=lambda t: torch.stack([t] + parts))
    err = (out.float() - ref.float()).abs().max().item()
    assert err <= 2e-3, err
    combined = O.lse_combine(_np(torch.stack(
        [P.local_partial(q, hk, hv, full)], 1)))
    np.testing.assert_allclose(combined, _np(ref).reshape(B * Hq, D).astype(np.float32), atol=2e-3, rtol=0)
