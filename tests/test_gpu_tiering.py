"""GPU parity: importance update, demote selection, row gather, cold-tier copies."""
import os

import numpy as np
import pytest
import torch

from oracle import akv_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _np(t):
    return t.detach().cpu().numpy()


def test_importance_update_golden(golden_dir):
    from akv import tiering
    z = np.load(os.path.join(golden_dir, "importance.npz"))
    for (B, H, M, N) in ((1, 4, 1, 64), (2, 8, 3, 257), (8, 8, 1, 512)):
        t = f"imp_B{B}_H{H}_M{M}_N{N}"
        attn = torch.from_numpy(z[f"{t}/attn"]).to(DEV)
        scores = torch.from_numpy(z[f"{t}/scores_in"]).to(DEV)
        out = tiering.fused_importance_update(attn, scores, decay=float(z[f"{t}/decay"]))
        assert out.data_ptr() == scores.data_ptr()  # in place, like the reference
        np.testing.assert_array_equal(_np(out), z[f"{t}/scores_out"])
    s = torch.ones(32, device=DEV)
    out = tiering.fused_importance_update(torch.zeros(1, 1, 1, 32, device=DEV), s, decay=0.5)
    np.testing.assert_array_equal(_np(out), z["imp_zero/scores_out"])


def test_importance_update_pad_and_truncate():
    from akv import tiering
    rng = np.random.default_rng(0)
    for na, n in ((40, 64), (100, 64)):
        attn = rng.random((2, 3, 2, na)).astype(np.float32)
        scores = rng.random(n).astype(np.float32)
        ref = O.importance_update(attn, scores, 0.9, vec_width=_C_width())
        out = tiering.fused_importance_update(torch.from_numpy(attn).to(DEV), torch.from_numpy(scores).to(DEV), 0.9)
        np.testing.assert_array_equal(_np(out), ref)


def _C_width():
    from akv import _C
    return _C.cpu_reduction_width()


@pytest.mark.parametrize("width", [8, 16])
@pytest.mark.parametrize("shape", [(8, 8, 1, 512), (16, 32, 1, 1000), (4, 8, 2, 3000), (3, 5, 17, 100),
                                   (5, 7, 3, 33), (32, 16, 1, 2000), (8, 8, 1, 131072), (2, 8, 64, 300)])
def test_importance_update_torch_order(shape, width):
    """Bit-exact against the oracle's restatement of torch's CPU reduction
    order (pinned to torch itself on the CPU) at both SIMD widths: every
    cascade level, block, single-register and scalar-tail column path."""
    from akv import _C, tiering
    rng = np.random.default_rng(sum(shape) + width)
    a = rng.random(shape).astype(np.float32)
    a /= a.sum(-1, keepdims=True)
    s = rng.random(shape[-1]).astype(np.float32)
    lib = _C.load()
    try:
        assert lib.akv_set_reduction_width(width) == 0
        out = tiering.fused_importance_update(torch.from_numpy(a).to(DEV), torch.from_numpy(s).to(DEV), 0.9)
        np.testing.assert_array_equal(_np(out), O.importance_update(a, s, 0.9, vec_width=width))
    finally:
        lib.akv_set_reduction_width(_C.cpu_reduction_width())


def test_select_golden(golden_dir):
    from akv import tiering
    z = np.load(os.path.join(golden_dir, "importance.npz"))
    for key in [k for k in z.files if k.startswith("sel_") and k.endswith("/meta")]:
        t = key[:-5]
        hot_len, budget, n_dem = (int(x) for x in z[key])
        idx = tiering.select_demote_indices(torch.from_numpy(z[f"{t}/scores"]).to(DEV), n_dem, budget)
        np.testing.assert_array_equal(_np(idx), z[f"{t}/idx"], err_msg=t)


@pytest.mark.parametrize("n,k", [(1, 1), (10, 3), (1000, 999), (4096, 3584), (131072, 8192), (131072, 1)])
def test_select_vs_oracle_ties(n, k):
    """Ties (quantised scores) resolve lowest index first, like the oracle."""
    from akv import tiering
    rng = np.random.default_rng(n + k)
    scores = (rng.integers(0, 50, n) / 7.0).astype(np.float32)
    budget = 64
    pf, pl = min(4, n), min(16, budget // 4)
    k = max(0, min(k, n - pf - pl)) if n > pf + pl else 0
    if k == 0:
        return
    idx = tiering.select_bottomk(torch.from_numpy(scores).to(DEV), k, pf, pl)
    ref = O.select_demote(scores, k, budget)
    np.testing.assert_array_equal(_np(idx), ref)


def test_gather_rows():
    from akv import tiering
    x = torch.randn(2, 3, 50, 128, device=DEV).half()
    idx = torch.tensor([0, 7, 7, 49, 3], device=DEV)
    y = tiering.gather_rows(x, idx)
    torch.testing.assert_close(y, x[:, :, idx], rtol=0, atol=0)


def test_cold_copy_roundtrip():
    from akv import tiering
    src = torch.randint(0, 255, (2, 4, 10, 3856), dtype=torch.uint8, device=DEV)
    host = torch.empty(2, 4, 3, 3856, dtype=torch.uint8).pin_memory()
    side = torch.cuda.Stream()
    ev = tiering.cold_copy_blocks(src, 5, 3, host, stream=side)
    ev.synchronize()
    np.testing.assert_array_equal(host.numpy(), _np(src[:, :, 5:8]))
    dst = torch.zeros_like(src)
    ev = tiering.cold_restore_blocks(host, dst, 2, stream=side)
    ev.synchronize()
    np.testing.assert_array_equal(_np(dst[:, :, 2:5]), _np(src[:, :, 5:8]))


@pytest.mark.parametrize("n,k,pf,pl,levels", [(131072, 64, 4, 32, 0), (131072, 640, 4, 32, 50),
                                              (100003, 1000, 0, 0, 7), (4097, 4097, 3, 5, 3), (37, 5, 2, 2, 0)])
def test_select_bottomk_large_ties_unaligned(n, k, pf, pl, levels):
    """Multi-CTA selection against a stable CPU ordering (value, then index;
    protected ends rank as +inf): many CTAs, ties spanning CTA slices, and an
    unaligned score pointer (the scalar-load path)."""
    from akv import tiering
    rng = np.random.default_rng(n + k)
    vals = rng.random(n + 1).astype(np.float32)
    if levels:
        vals = np.floor(vals * levels).astype(np.float32) / levels  # heavy ties
    for offset in (0, 1):
        base = torch.from_numpy(vals).to(DEV)
        s = base[offset:offset + n]
        got = tiering.select_bottomk(s, k, pf, pl).cpu().numpy()
        keys = vals[offset:offset + n].astype(np.float64).copy()
        keys[:pf] = np.inf
        if pl:
            keys[n - pl:] = np.inf
        want = np.sort(np.lexsort((np.arange(n), keys))[:k])
        np.testing.assert_array_equal(got, want)
