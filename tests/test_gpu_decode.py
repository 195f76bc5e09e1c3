"""GPU parity: mixed-tier decode attention vs the oracle.

The oracle dequantises the warm tier exactly like the reference (one
AffineQuantizer call per 32-token group and batch row), concatenates the FP16
hot window and runs fp32 softmax attention (akv/fused_attention.py:362-366).
Bar (north star): max-abs error <= 2e-3 on the fp16 output.
"""
import math

import numpy as np
import pytest
import torch

from oracle import akv_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
ATOL = 2e-3


def tolerance(ref):
    """2e-3 max-abs; where |ref| >= 4 the fp16 output's own half-ulp rounding
    (>= 9.8e-4) plus 1e-3 of arithmetic error is allowed instead."""
    ref = np.asarray(ref, np.float32)
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)
    return np.maximum(ATOL, 0.5 * ulp + 1e-3)


def _np(t):
    return t.detach().cpu().numpy()


def _rope(x, start=0, base=10000.0):
    """Half-split rotary embedding on (..., N, D) fp16 (reference _diag_quant_rope.py recipe)."""
    D = x.shape[-1]
    half = D // 2
    inv = 1.0 / (base ** (np.arange(half, dtype=np.float32) / half))
    ang = (np.arange(start, start + x.shape[-2], dtype=np.float32)[:, None] * inv[None, :])
    cos, sin = np.cos(ang), np.sin(ang)
    xf = x.astype(np.float32)
    x1, x2 = xf[..., :half], xf[..., half:]
    return np.concatenate([x1 * cos - x2 * sin, x1 * sin + x2 * cos], -1).astype(np.float16)


def make_case(seed, B, Hq, Hkv, D, n_warm, n_hot, outlier_ch=(), rope=True):
    rng = np.random.default_rng(seed)
    N = n_warm + n_hot
    k = rng.standard_normal((B, Hkv, N, D)).astype(np.float32)
    for c in outlier_ch:
        k[..., c] *= 12.0
    k = k.astype(np.float16)
    if rope:
        k = _rope(k)
    v = rng.standard_normal((B, Hkv, N, D)).astype(np.float16)
    q = rng.standard_normal((B, Hq, D)).astype(np.float16)
    return q, k[:, :, :n_warm], v[:, :, :n_warm], k[:, :, n_warm:], v[:, :, n_warm:]


def run_case(q, wk, wv, hk, hv, kb, vb, frac, hot_len=None, warm_blocks=None):
    import akv
    B, Hkv, n_warm, D = wk.shape
    n_hot = hk.shape[2]
    arena = None
    if n_warm:
        arena = akv.WarmArena(B, Hkv, D, kb, vb, outlier_fraction=frac,
                              max_blocks=(n_warm + 31) // 32 + 1, device=DEV)
        arena.append(torch.from_numpy(wk).to(DEV), torch.from_numpy(wv).to(DEV), group=32)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    hkt = torch.from_numpy(hk).to(DEV) if n_hot else None
    hvt = torch.from_numpy(hv).to(DEV) if n_hot else None
    hl = torch.tensor(hot_len, dtype=torch.int32, device=DEV) if hot_len is not None else None
    wl = torch.tensor(warm_blocks, dtype=torch.int32, device=DEV) if warm_blocks is not None else None
    out, lse = akv.mixed_tier_decode_attention(torch.from_numpy(q).to(DEV), hkt, hvt, arena,
                                               hot_len=hl, warm_len=wl, return_lse=True, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return _np(out).astype(np.float32), _np(lse)


def oracle_case(q, wk, wv, hk, hv, kb, vb, frac, hot_len=None, warm_blocks=None):
    B, Hkv, n_warm, D = wk.shape
    outs, lses = [], []
    for b in range(B):
        nw = n_warm if warm_blocks is None else min(n_warm, 32 * warm_blocks[b])
        nh = hk.shape[2] if hot_len is None else hot_len[b]
        parts_k, parts_v = [], []
        if nw:
            parts_k.append(O.dequantize_groups(O.quantize_groups(wk[b:b + 1, :, :nw], kb, 32, True, frac)))
            parts_v.append(O.dequantize_groups(O.quantize_groups(wv[b:b + 1, :, :nw], vb, 32, False, frac)))
        parts_k.append(hk[b:b + 1, :, :nh])
        parts_v.append(hv[b:b + 1, :, :nh])
        o, l = O.decode_attention(q[b:b + 1], np.concatenate(parts_k, 2), np.concatenate(parts_v, 2),
                                  return_lse=True)
        outs.append(o)
        lses.append(l)
    return np.concatenate(outs), np.concatenate(lses)


def check(seed, B, Hq, Hkv, n_warm, n_hot, kb, vb, frac, D=128, outlier_ch=(7,), **kw):
    q, wk, wv, hk, hv = make_case(seed, B, Hq, Hkv, D, n_warm, n_hot, outlier_ch)
    out, lse = run_case(q, wk, wv, hk, hv, kb, vb, frac, **kw)
    ref, rlse = oracle_case(q, wk, wv, hk, hv, kb, vb, frac, **kw)
    err = np.abs(out - ref).max()
    print(f"[decode err] seed={seed} B={B} Hq={Hq} Hkv={Hkv} nw={n_warm} nh={n_hot} k{kb}v{vb} f={frac}: {err:.3e}")
    assert (np.abs(out - ref) <= tolerance(ref)).all(), f"max abs err {err}"
    np.testing.assert_allclose(lse, rlse, atol=2e-3, rtol=0)
    return err


def test_config1_full():
    """Config 1 (the reference's small benchmark case): B1, 12 Q / 2 KV heads, D128, 512 hot + 3584 warm
    at 3 bits, 32-token groups,
    1% of K channels x12 outliers, RoPE on K."""
    check(0, 1, 12, 2, 3584, 512, 3, 3, 0.0, outlier_ch=(100,))


def test_config3_shape_small():
    """Config-3 shape family (32 Q / 8 KV heads, k4v2, outlier_fraction 0.01) at a short context."""
    check(1, 2, 32, 8, 32 * 20 + 5, 70, 4, 2, 0.01, outlier_ch=(3, 77))


@pytest.mark.parametrize("kb", [2, 3, 4])
@pytest.mark.parametrize("vb", [2, 3, 4])
def test_bit_combinations(kb, vb):
    check(10 + kb * 5 + vb, 2, 8, 2, 32 * 6, 40, kb, vb, 0.0)


@pytest.mark.parametrize("frac", [0.01, 0.05])
def test_outlier_channels(frac):
    check(20, 1, 16, 4, 32 * 9 + 17, 33, 3, 3, frac, outlier_ch=(1, 64, 127))


def test_warm_only_mha():
    check(30, 2, 4, 4, 96, 0, 2, 2, 0.0)


def test_hot_only_gqa():
    check(31, 3, 8, 2, 0, 300, 4, 4, 0.0)


def test_group16_heads():
    """g = Hq/Hkv = 16 > 8: two head groups per KV head."""
    check(32, 1, 32, 2, 32 * 4, 64, 4, 4, 0.0)


def test_ragged_batch():
    check(33, 3, 8, 2, 32 * 5, 50, 3, 3, 0.0, hot_len=[50, 7, 0], warm_blocks=[5, 2, 3])


def test_single_token():
    check(34, 1, 8, 1, 0, 1, 4, 4, 0.0)
    check(35, 1, 8, 1, 1, 0, 4, 4, 0.0)


def test_large_logits_stable():
    """Scaled-up queries: softmax must stay finite and match (online max subtraction)."""
    q, wk, wv, hk, hv = make_case(40, 1, 8, 2, 128, 32 * 8, 64)
    q = (q.astype(np.float32) * 8).astype(np.float16)
    out, _ = run_case(q, wk, wv, hk, hv, 4, 4, 0.0)
    ref, _ = oracle_case(q, wk, wv, hk, hv, 4, 4, 0.0)
    assert np.isfinite(out).all()
    assert (np.abs(out - ref) <= tolerance(ref)).all(), np.abs(out - ref).max()


@pytest.mark.parametrize("q_mul,k_mul", [(40.0, 1.0), (1e-4, 1.0), (1.0, 300.0), (0.02, 1000.0)])
def test_extreme_magnitudes(q_mul, k_mul):
    """Query and key magnitudes far from unit scale (logits from ~1e-4 to
    ~1e4): outputs stay finite and match the oracle."""
    q, wk, wv, hk, hv = make_case(41, 1, 8, 2, 128, 32 * 6 + 9, 40, outlier_ch=(5,))
    q = (q.astype(np.float32) * q_mul).astype(np.float16)
    wk = (wk.astype(np.float32) * k_mul).astype(np.float16)
    hk = (hk.astype(np.float32) * k_mul).astype(np.float16)
    for kb, vb, frac in ((4, 2, 0.01), (2, 3, 0.0)):
        out, _ = run_case(q, wk, wv, hk, hv, kb, vb, frac)
        ref, _ = oracle_case(q, wk, wv, hk, hv, kb, vb, frac)
        assert np.isfinite(out).all()
        assert (np.abs(out - ref) <= tolerance(ref)).all(), np.abs(out - ref).max()


def test_config3_full_context():
    """Config 3 (the headline decode shape) at full size (B16, 32 Q / 8 KV heads, 30,720 warm k4v2
    tokens with 1 % outliers + 2,048 hot): every warp streams a dozen records
    through its stage ring, refilling each stage.  Reference: fp32 attention
    over the arena's dequantised tiers (the dequantisation itself is checked
    bit-exact against the oracle by the quantiser tests)."""
    import akv
    B, Hq, Hkv, D, nw, nh = 16, 32, 8, 128, 30720, 2048
    g = torch.Generator(device=DEV).manual_seed(3)
    wk = torch.randn(B, Hkv, nw, D, generator=g, device=DEV).half()
    wk[..., 3] *= 12
    wv = torch.randn(B, Hkv, nw, D, generator=g, device=DEV).half()
    arena = akv.WarmArena(B, Hkv, D, 4, 2, 0.01, max_blocks=nw // 32, device=DEV)
    arena.append(wk, wv, group=32)
    del wk, wv
    hk = torch.randn(B, Hkv, nh, D, generator=g, device=DEV).half()
    hv = torch.randn(B, Hkv, nh, D, generator=g, device=DEV).half()
    q = torch.randn(B, Hq, D, generator=g, device=DEV).half()
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = akv.mixed_tier_decode_attention(q, hk, hv, arena, status=status).float()
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    kd, vd = arena.dequantize()
    err = 0.0
    for b in range(B):
        K = torch.cat([kd[b], hk[b]], 1).float().repeat_interleave(Hq // Hkv, 0)
        V = torch.cat([vd[b], hv[b]], 1).float().repeat_interleave(Hq // Hkv, 0)
        p = torch.softmax(torch.einsum("hd,hnd->hn", q[b].float(), K) / D ** 0.5, -1)
        ref = torch.einsum("hn,hnd->hd", p, V)
        err = max(err, (out[b] - ref).abs().max().item())
    print(f"[decode err] config 3 full context: {err:.3e}")
    assert err <= ATOL


def test_reference_signature_hot_only(golden_dir):
    import os
    import akv
    z = np.load(os.path.join(golden_dir, "attention.npz"))
    t = "hot_B2_H2_N100_D128"
    out = akv.mixed_precision_decode_attention(torch.from_numpy(z[f"{t}/q"]).to(DEV),
                                               torch.from_numpy(z[f"{t}/k"]).to(DEV),
                                               torch.from_numpy(z[f"{t}/v"]).to(DEV))
    assert out.shape == (2, 2, 1, 128)
    ref = z[f"{t}/out"].astype(np.float32)
    assert (np.abs(_np(out).astype(np.float32) - ref) <= tolerance(ref)).all()


def test_affine_gqa_golden(golden_dir):
    """Golden from the reference: dequantised affine warm + hot, GQA, fp32 attention."""
    import os
    import akv
    z = np.load(os.path.join(golden_dir, "attention.npz"))
    t = "affine_gqa"
    wk, wv = z[f"{t}/wk"], z[f"{t}/wv"]
    arena = akv.WarmArena(1, 2, 128, 3, 3, max_blocks=4, device=DEV)
    arena.append(torch.from_numpy(wk).to(DEV), torch.from_numpy(wv).to(DEV), group=32)
    out = akv.mixed_tier_decode_attention(torch.from_numpy(z[f"{t}/q"]).to(DEV),
                                          torch.from_numpy(z[f"{t}/hk"]).to(DEV),
                                          torch.from_numpy(z[f"{t}/hv"]).to(DEV), arena)
    ref = z[f"{t}/out"].astype(np.float32)
    assert (np.abs(_np(out).astype(np.float32) - ref) <= tolerance(ref)).all()


@pytest.mark.parametrize("gs", [32, 128])
def test_reference_int4_layout_golden(golden_dir, gs):
    """The reference's INT4 per-token-group warm layout: dequant bit-exact, the
    fused / mixed entry points within tolerance of the reference outputs."""
    import os
    import akv
    z = np.load(os.path.join(golden_dir, "attention.npz"))
    t = f"int4_gs{gs}"
    T = {k: torch.from_numpy(z[f"{t}/{k}"]).to(DEV) for k in ("q", "hk", "hv", "wkp", "wks", "wkz",
                                                               "wvp", "wvs", "wvz")}
    D = T["q"].shape[-1]
    dk = akv.int4_group_dequant(T["wkp"], T["wks"], T["wkz"], D, gs)
    np.testing.assert_array_equal(_np(dk).view(np.uint16), z[f"{t}/deq_k"].view(np.uint16))
    warm = (T["wkp"], T["wks"], T["wkz"], T["wvp"], T["wvs"], T["wvz"])
    mixed = akv.mixed_precision_decode_attention(T["q"], T["hk"], T["hv"], *warm, group_size=gs)
    ref = z[f"{t}/mixed"].astype(np.float32)
    assert mixed.shape == T["q"].shape
    assert (np.abs(_np(mixed).astype(np.float32) - ref) <= tolerance(ref)).all()
    for tag, limit in (("int4", 512.0), ("int4_tiled", 1e-3)):  # one tile / many tiles
        out = akv.fused_int4_decode_attention(T["q"], *warm, group_size=gs, memory_limit_mb=limit)
        ref = z[f"{t}/{tag}"].astype(np.float32)
        err = np.abs(_np(out).astype(np.float32) - ref)
        assert (err <= tolerance(ref)).all(), (tag, err.max())


def test_few_units_long_context():
    """Config-5b shard shape (B1, 64 Q / 8 KV heads, 61,440 warm k4v4 + 4,096
    hot): 8 units, so the planner's one-wave target gives each CTA ~28 blocks
    and each warp several stage refills.  Reference: fp32 attention over the
    arena's dequantised tiers."""
    import akv
    B, Hq, Hkv, D, nw, nh = 1, 64, 8, 128, 61440, 4096
    g = torch.Generator(device=DEV).manual_seed(9)
    wk = torch.randn(B, Hkv, nw, D, generator=g, device=DEV).half()
    wv = torch.randn(B, Hkv, nw, D, generator=g, device=DEV).half()
    arena = akv.WarmArena(B, Hkv, D, 4, 4, 0.0, max_blocks=nw // 32, device=DEV)
    arena.append(wk, wv, group=32)
    hk = torch.randn(B, Hkv, nh, D, generator=g, device=DEV).half()
    hv = torch.randn(B, Hkv, nh, D, generator=g, device=DEV).half()
    q = torch.randn(B, Hq, D, generator=g, device=DEV).half()
    out = akv.mixed_tier_decode_attention(q, hk, hv, arena).float()
    kd, vd = arena.dequantize()
    K = torch.cat([kd[0], hk[0]], 1).float().repeat_interleave(Hq // Hkv, 0)
    V = torch.cat([vd[0], hv[0]], 1).float().repeat_interleave(Hq // Hkv, 0)
    p = torch.softmax(torch.einsum("hd,hnd->hn", q[0].float(), K) / D ** 0.5, -1)
    ref = torch.einsum("hn,hnd->hd", p, V)
    err = (out[0] - ref).abs().max().item()
    print(f"[decode err] few units, long context: {err:.3e}")
    assert err <= ATOL


def test_config5a_full_shape():
    """Config 5a at its full shape (B32, 64 Q / 8 KV heads, 61,440 warm k4v4
    tokens + 4,096 hot, ~10 GB of fp16 inputs): every row against fp32
    attention over the arena's dequantised tiers (GQA groups, no repeat)."""
    import akv
    B, Hq, Hkv, D, nw, nh = 32, 64, 8, 128, 61440, 4096
    g = torch.Generator(device=DEV).manual_seed(5)
    arena = akv.WarmArena(B, Hkv, D, 4, 4, 0.0, max_blocks=nw // 32, device=DEV)
    wk = torch.randn(B, Hkv, nw, D, generator=g, device=DEV).half()
    wv = torch.randn(B, Hkv, nw, D, generator=g, device=DEV).half()
    arena.append(wk, wv, group=32)
    del wk, wv
    hk = torch.randn(B, Hkv, nh, D, generator=g, device=DEV).half()
    hv = torch.randn(B, Hkv, nh, D, generator=g, device=DEV).half()
    q = torch.randn(B, Hq, D, generator=g, device=DEV).half()
    out = akv.mixed_tier_decode_attention(q, hk, hv, arena).float()
    gq = Hq // Hkv
    worst = 0.0
    kd, vd = arena.dequantize()
    for b in range(B):
        K = torch.cat([kd[b], hk[b]], 1).float()  # (Hkv, N, D)
        V = torch.cat([vd[b], hv[b]], 1).float()
        qb = q[b].float().view(Hkv, gq, D)
        p = torch.softmax(torch.einsum("hgd,hnd->hgn", qb, K) / D ** 0.5, -1)
        ref = torch.einsum("hgn,hnd->hgd", p, V).reshape(Hq, D)
        worst = max(worst, (out[b] - ref).abs().max().item())
    print(f"[decode err] config 5a full shape: {worst:.3e}")
    assert worst <= ATOL
    del arena, kd, vd
    torch.cuda.empty_cache()


# ---------------------------------------------------------------------------- head dims 64 and 256
@pytest.mark.parametrize("D", [64, 256])
@pytest.mark.parametrize("kb,vb", [(2, 2), (3, 3), (4, 4), (4, 2), (2, 3), (3, 4)])
def test_head_dims_bit_pairs(D, kb, vb):
    """The decode kernel built for head dim 64 (half a 32-channel record
    chunk per K thread column, 8 V channels per thread row) and 256 (two
    chunks, two 16-channel V groups), warm + hot, against the oracle."""
    check(60 + D + 3 * kb + vb, 2, 8, 2, 32 * 6 + 9, 45, kb, vb, 0.0, D=D, outlier_ch=(5,))


@pytest.mark.parametrize("D", [64, 256])
@pytest.mark.parametrize("n_out", [1, 3, 8])
def test_head_dims_outliers(D, n_out):
    """One outlier channel (the side-tile path) and several, up to the
    kernel's eight (the extra-MMA path), at head dims 64 and 256, channels at
    both ends of the row."""
    f = (n_out + 0.5) / D
    check(70 + D, 1, 16, 4, 32 * 9 + 17, 33, 4, 2, f, D=D, outlier_ch=(1, D // 2 + 3, D - 1))


@pytest.mark.parametrize("D", [64, 256])
def test_head_dims_hot_only_ragged(D):
    check(80 + D, 3, 12, 4, 0, 150, 4, 4, 0.0, D=D, hot_len=[150, 1, 77])
    check(81 + D, 3, 12, 4, 32 * 7, 40, 3, 2, 0.0, D=D, hot_len=[40, 0, 13], warm_blocks=[7, 2, 0])


def test_head_dim_64_tinyllama_shape():
    """The paper's ITL model shape (TinyLlama: 32 query / 4 KV heads, head
    dim 64) at a 4K context: 3,584 warm tokens at k4v2 with 1 % outliers,
    512 hot."""
    check(90, 1, 32, 4, 3584, 512, 4, 2, 0.01, D=64, outlier_ch=(9,))


def test_head_dim_256_gqa_groups():
    """Head dim 256 with 16 query heads per KV head (two head groups per CTA row)."""
    check(91, 2, 32, 2, 32 * 12, 64, 3, 3, 0.0, D=256, outlier_ch=(200,))
