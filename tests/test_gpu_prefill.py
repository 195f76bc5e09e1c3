"""GPU parity: tcgen05 prefill attention over the FP16 hot tier and packed warm
records, causal by token position, against the fp32 oracle
(oracle.akv_oracle.prefill_attention: SDPA over the chronological view, the
reference's prefill data flow, akv/drop_in.py:753-787).

Bar (as for decode, tests/test_gpu_decode.py): max-abs error <= 2e-3 against
fp32 softmax attention over the exactly dequantised warm tier; where |ref| >= 4
the fp16 output's own half-ulp rounding plus 1e-3 of arithmetic error is
allowed instead (the kernel also rounds P to fp16 before P.V, as flash
attention and the decode kernel do).
"""
import numpy as np
import pytest
import torch

from oracle import akv_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
ATOL = 2e-3


def tolerance(ref):
    ref = np.asarray(ref, np.float32)
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)
    return np.maximum(ATOL, 0.5 * ulp + 1e-3)


def check(out, ref):
    o = out.float().cpu().numpy()
    err = np.abs(o - ref)
    tol = tolerance(ref)
    worst = np.unravel_index(np.argmax(err - tol), err.shape)
    assert np.all(err <= tol), f"prefill err {err[worst]} > {tol[worst]} at {worst} (ref {ref[worst]})"


def _kv(g, shape, outlier=(3,)):
    x = torch.randn(shape, generator=g, device=DEV)
    for c in outlier:
        x[..., c] *= 12.0
    return x.half()


def _case(seed, B, Hq, Hkv, n_warm, n_hot, kb, vb, frac, M, q_start=0):
    import akv
    g = torch.Generator(device=DEV).manual_seed(seed)
    D = 128
    n_tot = n_warm + n_hot
    perm = torch.randperm(n_tot, generator=torch.Generator().manual_seed(seed)).to(torch.int32)
    arena = None
    nblk = (n_warm + 31) // 32
    wpos = torch.full((B, max(nblk, 1) * 32), 2 ** 30, dtype=torch.int32)
    if n_warm:
        arena = akv.WarmArena(B, Hkv, D, kb, vb, outlier_fraction=frac, max_blocks=nblk, device=DEV)
        arena.append(_kv(g, (B, Hkv, n_warm, D)), _kv(g, (B, Hkv, n_warm, D), (5,)), group=32)
        wpos[:, :n_warm] = perm[:n_warm]
    hk = _kv(g, (B, Hkv, n_hot, D))
    hv = _kv(g, (B, Hkv, n_hot, D), (5,))
    hpos = perm[n_warm:].unsqueeze(0).expand(B, n_hot).contiguous()
    q = torch.randn(B, Hq, M, D, generator=g, device=DEV).half()
    qpos = (torch.arange(M, dtype=torch.int32) + q_start).unsqueeze(0).expand(B, M).contiguous()
    return q, qpos, hk, hv, hpos, arena, wpos


def _oracle(q, qpos, hk, hv, hpos, arena, wpos):
    keys, vals, kpos = [], [], []
    if arena is not None:
        n = arena.n_blocks * 32
        dk, dv = arena.dequantize(n_tokens=n)
        keys.append(dk.cpu().numpy())
        vals.append(dv.cpu().numpy())
        kp = wpos[:, :n].numpy().copy()
        masks = arena.masks().cpu().numpy()  # (B, H, n_blocks): slots the quantiser wrote
        valid = ((masks[:, 0, :, None] >> np.arange(32)) & 1).reshape(masks.shape[0], -1).astype(bool)
        kp[~valid] = 2 ** 30
        kpos.append(kp)
    if hk.shape[2]:
        keys.append(hk.cpu().numpy())
        vals.append(hv.cpu().numpy())
        kpos.append(hpos.numpy())
    return O.prefill_attention(q.cpu().numpy(), qpos.numpy(), np.concatenate(keys, 2), np.concatenate(vals, 2),
                               np.concatenate(kpos, 1))


def _run(args, **kw):
    import akv
    q, qpos, hk, hv, hpos, arena, wpos = args
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out, lse = akv.prefill_attention(q, qpos.to(DEV), hk, hv, hpos.to(DEV), arena,
                                     wpos.to(DEV) if arena is not None else None, return_lse=True,
                                     status=status, **kw)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out, lse


@pytest.mark.parametrize("kb,vb,frac", [(4, 2, 0.01), (3, 3, 0.0), (2, 4, 0.02), (4, 4, 0.0)])
def test_prefill_mixed_tiers_causal(kb, vb, frac):
    """Whole-prompt prefill: positions 0..N-1 spread at random over a warm
    tier (partial last record) and a hot tier; three query tiles, the last
    partial."""
    args = _case(1, 2, 8, 2, 32 * 12 + 16, 200, kb, vb, frac, M=600)
    out, _ = _run(args)
    check(out, _oracle(*args))


def test_prefill_chunk_after_context():
    """Chunked prefill: 130 new tokens at positions 600..729 attend over all
    600 earlier tokens and causally over each other (the chunk sits in the
    hot tier)."""
    import akv
    g = torch.Generator(device=DEV).manual_seed(2)
    B, Hq, Hkv, D = 1, 12, 2, 128
    n_warm, n_old_hot, M = 32 * 15, 120, 130
    arena = akv.WarmArena(B, Hkv, D, 3, 3, max_blocks=15, device=DEV)
    arena.append(_kv(g, (B, Hkv, n_warm, D)), _kv(g, (B, Hkv, n_warm, D)), group=32)
    wpos = torch.arange(n_warm, dtype=torch.int32).unsqueeze(0)
    hk = _kv(g, (B, Hkv, n_old_hot + M, D))
    hv = _kv(g, (B, Hkv, n_old_hot + M, D))
    hpos = torch.arange(n_warm, n_warm + n_old_hot + M, dtype=torch.int32).unsqueeze(0)
    q = torch.randn(B, Hq, M, D, generator=g, device=DEV).half()
    qpos = torch.arange(n_warm + n_old_hot, n_warm + n_old_hot + M, dtype=torch.int32).unsqueeze(0)
    args = (q, qpos, hk, hv, hpos, arena, wpos)
    out, lse = _run(args)
    check(out, _oracle(*args))


def test_prefill_hot_only_and_lse():
    args = _case(3, 2, 4, 4, 0, 257, 4, 4, 0.0, M=257)
    out, lse = _run(args)
    q, qpos, hk, hv, hpos, _, _ = args
    check(out, _oracle(*args))
    # natural-log LSE of the scaled logits, against fp64
    qf, kf = q.double().cpu(), hk.double().cpu()
    s = torch.einsum("bhmd,bhnd->bhmn", qf, kf) / np.sqrt(128)
    vis = hpos[:, None, None, :] <= qpos[:, None, :, None]
    ref_lse = torch.logsumexp(s.masked_fill(~vis, float("-inf")), -1)
    np.testing.assert_allclose(lse.cpu().numpy(), ref_lse.numpy(), rtol=0, atol=1e-4)


def test_prefill_rows_without_keys_are_zero():
    """Query rows that see no key (positions before every key) give zero rows and lse -inf."""
    q, qpos, hk, hv, hpos, arena, wpos = _case(4, 1, 4, 2, 64, 64, 4, 2, 0.01, M=40)
    qpos = qpos.clone()
    qpos[:, :8] = -5
    out, lse = _run((q, qpos, hk, hv, hpos, arena, wpos))
    assert torch.all(out[:, :, :8] == 0)
    assert torch.all(torch.isinf(lse[:, :, :8]))
    check(out, _oracle(q, qpos, hk, hv, hpos, arena, wpos))


def test_prefill_gqa_strided_query():
    """Query heads of a KV head in GQA order, q given as a (B, M, Hq, D) tensor transposed (strided heads)."""
    import akv
    q, qpos, hk, hv, hpos, arena, wpos = _case(5, 2, 16, 4, 32 * 6, 96, 4, 2, 0.01, M=150)
    qs = q.transpose(1, 2).contiguous().transpose(1, 2)  # same values, head stride D, token stride Hq*D
    out, _ = _run((qs, qpos, hk, hv, hpos, arena, wpos))
    check(out, _oracle(q, qpos, hk, hv, hpos, arena, wpos))


def test_prefill_config3_scale_vs_torch_fp32():
    """Config-3 shape per KV head: a 32K prompt after its prefill demotion
    (30,720 warm tokens at k4v2 with one outlier channel, at sorted positions
    drawn at random; 2,048 hot), every one of the 32,768 queries of 4 query
    heads, causal.  Reference: fp32 softmax attention in torch on the GPU over
    the exactly dequantised warm tier (the akv dequantiser, pinned bit-exact
    to the oracle elsewhere) and the hot tier, in query chunks."""
    import akv
    g = torch.Generator(device=DEV).manual_seed(9)
    B, Hq, Hkv, D, N, n_hot = 1, 4, 1, 128, 32768, 2048
    n_warm = N - n_hot
    perm = torch.randperm(N, generator=torch.Generator().manual_seed(9))
    wpos = perm[:n_warm].sort().values.to(torch.int32)
    hpos = perm[n_warm:].sort().values.to(torch.int32)
    arena = akv.WarmArena(B, Hkv, D, 4, 2, outlier_fraction=0.01, max_blocks=n_warm // 32, device=DEV)
    arena.append(_kv(g, (B, Hkv, n_warm, D)), _kv(g, (B, Hkv, n_warm, D), (5,)), group=32)
    hk, hv = _kv(g, (B, Hkv, n_hot, D)), _kv(g, (B, Hkv, n_hot, D), (5,))
    q = torch.randn(B, Hq, N, D, generator=g, device=DEV).half()
    qpos = torch.arange(N, dtype=torch.int32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = akv.prefill_attention(q, qpos, hk, hv, hpos.to(DEV), arena, wpos.to(DEV), status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    dk, dv = arena.dequantize(n_tokens=n_warm)
    K = torch.cat([dk, hk], 2)[0, 0].float()
    V = torch.cat([dv, hv], 2)[0, 0].float()
    kp = torch.cat([wpos, hpos]).to(DEV)
    worst = 0.0
    for m0 in range(0, N, 2048):
        qc = q[0, :, m0:m0 + 2048].float()
        s = torch.einsum("hmd,nd->hmn", qc, K) / np.sqrt(D)
        vis = kp[None, None, :] <= qpos[m0:m0 + 2048][None, :, None]
        p = torch.softmax(s.masked_fill(~vis, float("-inf")), -1)
        ref = (p @ V).cpu().numpy()
        check(out[0, :, m0:m0 + 2048], ref)
        worst = max(worst, float(np.abs(out[0, :, m0:m0 + 2048].float().cpu().numpy() - ref).max()))
    assert worst < 0.05
