"""Generate golden vectors by running the reference ``akv`` package (CPU).

Run in a container where the reference source is available:

    python tests/golden/make_golden.py /path/to/reference

It imports the reference package from that path, feeds it seeded inputs and
stores inputs + outputs as ``.npz`` fixtures next to this script.  The
fixtures pin the numpy oracle (``oracle/akv_oracle.py``) in
``tests/test_oracle_golden.py``; nothing at test or bench time imports the
reference itself.
"""
from __future__ import annotations

import math
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(path: str):
    sys.path.insert(0, path)
    import akv  # noqa: F401  (the reference package)
    from akv import bitpack
    from akv.affine_quantizer import AffineQuantizer, AffineQuantConfig
    from akv import fused_attention, triton_ops, packed_layout
    from akv.drop_in import AKVLayer
    assert os.path.abspath(akv.__file__).startswith(os.path.abspath(path)), akv.__file__
    return dict(bitpack=bitpack, AffineQuantizer=AffineQuantizer, AffineQuantConfig=AffineQuantConfig,
                fused_attention=fused_attention, triton_ops=triton_ops,
                packed_layout=packed_layout, AKVLayer=AKVLayer)


def rope(x, positions, base=10000.0):
    """Half-split rotary embedding (the recipe of the reference's
    ``_diag_quant_rope.py``: base 10000, rotate the two halves of D)."""
    import torch
    D = x.shape[-1]
    half = D // 2
    inv = 1.0 / (base ** (torch.arange(0, half, dtype=torch.float32) / half))
    ang = positions.float()[:, None] * inv[None, :]
    cos, sin = ang.cos(), ang.sin()
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], -1).to(x.dtype)


def make_kv(gen, H, N, D, outlier_ch=(), outlier_scale=12.0, use_rope=False, start=0):
    import torch
    x = torch.randn(H, N, D, generator=gen, dtype=torch.float32)
    for c in outlier_ch:
        x[..., c] *= outlier_scale
    x = x.half()
    if use_rope:
        x = rope(x, torch.arange(start, start + N))
    return x


def main(ref_path: str):
    import torch
    torch.set_num_threads(1)
    R = _import_reference(ref_path)
    bp = R["bitpack"]

    # ---------------- bitpack ----------------
    out = {}
    g = torch.Generator().manual_seed(1)
    for bits in (2, 3, 4):
        for D in (8, 32, 64, 128, 256):
            codes = torch.randint(0, 1 << bits, (2, 5, D), generator=g, dtype=torch.uint8)
            packed = bp.pack(codes, bits)
            out[f"b{bits}_d{D}_codes"] = codes.numpy()
            out[f"b{bits}_d{D}_packed"] = packed.numpy()
            out[f"b{bits}_d{D}_unpacked"] = bp.unpack(packed, bits, D).numpy()
    # odd widths: the reference right-pads with zeros
    for bits, D in ((4, 7), (3, 13), (2, 10)):
        codes = torch.randint(0, 1 << bits, (3, D), generator=g, dtype=torch.uint8)
        out[f"b{bits}_d{D}_codes"] = codes.numpy()
        out[f"b{bits}_d{D}_packed"] = bp.pack(codes, bits).numpy()
    np.savez_compressed(os.path.join(HERE, "bitpack.npz"), **out)

    # ---------------- affine quantiser ----------------
    AQ, AQC = R["AffineQuantizer"], R["AffineQuantConfig"]
    cases = []
    g = torch.Generator().manual_seed(2)
    # full bits x outlier-fraction matrix on small shapes, a few combos on larger ones
    combos = [(b, f) for b in (2, 3, 4) for f in (0.0, 0.01, 0.05)]
    shapes = [((2, 32, 128), combos), ((1, 1, 128), combos), ((2, 7, 64), combos),
              ((4, 32, 32), combos), ((3, 5, 16), combos),
              ((8, 32, 128), [(3, 0.01), (4, 0.0)]), ((2, 64, 128), [(2, 0.05)])]
    for (H, N, D), cmb in shapes:
        for bits, frac in cmb:
            ch = [int(torch.randint(0, D, (1,), generator=g))]
            k = make_kv(g, H, N, D, outlier_ch=ch, use_rope=(D >= 64))
            v = make_kv(g, H, N, D, outlier_ch=[int(torch.randint(0, D, (1,), generator=g))])
            cases.append((f"H{H}_N{N}_D{D}_b{bits}_f{frac}", k, v, bits, bits, frac))
    # asymmetric K/V bits (k4v2, k4v3)
    for kb, vb in ((4, 2), (4, 3)):
        k = make_kv(g, 8, 32, 128, outlier_ch=[5], use_rope=True)
        v = make_kv(g, 8, 32, 128)
        cases.append((f"asym_k{kb}v{vb}", k, v, kb, vb, 0.01))
    # edge cases: constant channel / constant token, zeros, large, subnormal, ties
    k = make_kv(g, 2, 32, 64)
    k[:, :, 3] = 1.5            # constant channel -> scale 0 for K
    k[0, :, 10] = 0.0           # zero channel
    k[1, 4, :] = 65504.0        # fp16 max in one token
    k[1, 5, :] = -65504.0
    v = make_kv(g, 2, 32, 64)
    v[0, 3, :] = 0.25           # constant token -> scale 0 for V
    v[1, 7, :] = 6e-8           # subnormal token
    v[1, 8, :2] = torch.tensor([6e-8, 0.0], dtype=torch.float16)
    for bits in (2, 3, 4):
        cases.append((f"edge_b{bits}", k.clone(), v.clone(), bits, bits, 0.0))
        cases.append((f"edge_out_b{bits}", k.clone(), v.clone(), bits, bits, 0.05))
    # tiny range -> scale underflows to zero while (x - zero) > 0
    k = torch.zeros(1, 4, 16, dtype=torch.float16)
    k[0, 1, :] = 6e-8
    k[0, 2, :] = 1.2e-7
    v = k.transpose(1, 2).contiguous().clone()[:, :4, :4].repeat(1, 1, 4)
    for bits in (2, 3, 4):
        cases.append((f"tiny_b{bits}", k.clone(), v.clone(), bits, bits, 0.0))

    out = {}
    names = []
    for name, k, v, kb, vb, frac in cases:
        qz = AQ(AQC(key_bits=kb, value_bits=vb, outlier_fraction=frac))
        qk = qz.quantize_keys(k.clone())
        qv = qz.quantize_values(v.clone())
        dk = qz.dequantize_keys(qk)
        dv = qz.dequantize_values(qv)
        pl = R["packed_layout"]
        names.append(name)
        out[f"{name}/k"] = k.numpy()
        out[f"{name}/v"] = v.numpy()
        out[f"{name}/meta"] = np.array([kb, vb, frac], np.float64)
        for tag, q, d in (("qk", qk, dk), ("qv", qv, dv)):
            for key in ("codes", "scale", "zero"):
                out[f"{name}/{tag}_{key}"] = q[key].numpy()
            if "outlier_idx" in q:
                out[f"{name}/{tag}_outlier_idx"] = q["outlier_idx"].numpy()
                out[f"{name}/{tag}_outlier_data"] = q["outlier_data"].numpy()
            out[f"{name}/{tag}_deq"] = d.numpy()
            out[f"{name}/{tag}_bytes"] = np.array(
                pl.measure_packed_bytes(q, kb if tag == "qk" else vb), np.int64)
    out["names"] = np.array(names)
    np.savez_compressed(os.path.join(HERE, "affine.npz"), **out)

    # ---------------- config-1 slice: 32-token groups ----------------
    # config 1 shapes (B1, 2 KV heads, D128, 3-bit), first 8 groups.
    g = torch.Generator().manual_seed(0)
    H, N, D = 2, 256, 128
    kout = list(range(0, D, 100))  # one planted outlier channel at D=128
    k = make_kv(g, H, N, D, outlier_ch=kout, use_rope=True)
    v = make_kv(g, H, N, D)
    qz = AQ(AQC(key_bits=3, value_bits=3))
    out = {"k": k.numpy(), "v": v.numpy()}
    for j in range(N // 32):
        qk = qz.quantize_keys(k[:, j * 32:(j + 1) * 32].clone())
        qv = qz.quantize_values(v[:, j * 32:(j + 1) * 32].clone())
        for key in ("codes", "scale", "zero"):
            out[f"g{j}/qk_{key}"] = qk[key].numpy()
            out[f"g{j}/qv_{key}"] = qv[key].numpy()
    np.savez_compressed(os.path.join(HERE, "config1_groups.npz"), **out)

    # ---------------- attention ----------------
    fa = R["fused_attention"]
    out = {}
    g = torch.Generator().manual_seed(3)
    # (a) plain fp32 attention over hot FP16 (MHA, the reference's
    #     mixed_precision_decode_attention with no warm tier)
    for (B, H, N, D) in ((1, 4, 64, 64), (2, 2, 100, 128)):
        q = torch.randn(B, H, 1, D, generator=g).half()
        kk = torch.randn(B, H, N, D, generator=g).half()
        vv = torch.randn(B, H, N, D, generator=g).half()
        o = fa.mixed_precision_decode_attention(q, kk, vv)
        tag = f"hot_B{B}_H{H}_N{N}_D{D}"
        out[f"{tag}/q"], out[f"{tag}/k"], out[f"{tag}/v"] = q.numpy(), kk.numpy(), vv.numpy()
        out[f"{tag}/out"] = o.numpy()
    # (b) mixed hot + INT4 per-token-group warm (reference layout of
    #     fused_attention.py:324-366), group_size 32 and 128
    for gs in (32, 128):
        B, H, Nh, Nw, D = 2, 4, 16, 48, 64
        q = torch.randn(B, H, 1, D, generator=g).half()
        hk = torch.randn(B, H, Nh, D, generator=g).half()
        hv = torch.randn(B, H, Nh, D, generator=g).half()
        G = D // gs if D >= gs else 1
        wkp = torch.randint(0, 256, (H, Nw, D // 2), generator=g, dtype=torch.uint8)
        wvp = torch.randint(0, 256, (H, Nw, D // 2), generator=g, dtype=torch.uint8)
        wks = (torch.rand(H, Nw, G, generator=g) * 0.3 + 0.01).half()
        wkz = (torch.randn(H, Nw, G, generator=g)).half()
        wvs = (torch.rand(H, Nw, G, generator=g) * 0.3 + 0.01).half()
        wvz = (torch.randn(H, Nw, G, generator=g)).half()
        o = fa.mixed_precision_decode_attention(q, hk, hv, wkp, wks, wkz, wvp, wvs, wvz, group_size=gs)
        o2 = fa.fused_int4_decode_attention(q, wkp, wks, wkz, wvp, wvs, wvz, group_size=gs)
        o3 = fa.fused_int4_decode_attention(q, wkp, wks, wkz, wvp, wvs, wvz, group_size=gs,
                                            memory_limit_mb=0.0)  # tiled online-softmax branch
        tag = f"int4_gs{gs}"
        for nm, t in (("q", q), ("hk", hk), ("hv", hv), ("wkp", wkp), ("wvp", wvp), ("wks", wks),
                      ("wkz", wkz), ("wvs", wvs), ("wvz", wvz), ("mixed", o), ("int4", o2), ("int4_tiled", o3)):
            out[f"{tag}/{nm}"] = t.numpy()
        out[f"{tag}/deq_k"] = fa._dequant_int4_tile(wkp, wks, wkz, D, gs).numpy()
    # (c) affine warm (AffineQuantizer) + hot, GQA, evaluated the way the
    #     reference HF path does: dequantise, concatenate, fp32 attention
    B, Hq, Hkv, Nh, Nw, D = 1, 12, 2, 64, 96, 128
    q = torch.randn(B, Hq, 1, D, generator=g).half()
    hk = make_kv(g, Hkv, Nh, D).unsqueeze(0)
    hv = make_kv(g, Hkv, Nh, D).unsqueeze(0)
    wk = make_kv(g, Hkv, Nw, D, outlier_ch=[7], use_rope=True).unsqueeze(0)
    wv = make_kv(g, Hkv, Nw, D).unsqueeze(0)
    qz = AQ(AQC(key_bits=3, value_bits=3))
    dk = torch.cat([qz.dequantize_keys(qz.quantize_keys(wk[0, :, j:j + 32].clone()))
                    for j in range(0, Nw, 32)], 1).unsqueeze(0)
    dv = torch.cat([qz.dequantize_values(qz.quantize_values(wv[0, :, j:j + 32].clone()))
                    for j in range(0, Nw, 32)], 1).unsqueeze(0)
    keys = torch.cat([dk, hk], 2).repeat_interleave(Hq // Hkv, 1)
    vals = torch.cat([dv, hv], 2).repeat_interleave(Hq // Hkv, 1)
    o = fa.mixed_precision_decode_attention(q, keys, vals)
    for nm, t in (("q", q), ("hk", hk), ("hv", hv), ("wk", wk), ("wv", wv), ("out", o)):
        out[f"affine_gqa/{nm}"] = t.numpy()
    np.savez_compressed(os.path.join(HERE, "attention.npz"), **out)

    # ---------------- importance update + demote selection ----------------
    to = R["triton_ops"]
    out = {}
    g = torch.Generator().manual_seed(4)
    for (B, H, M, N, decay) in ((1, 4, 1, 64, 0.95), (2, 8, 3, 257, 0.9), (8, 8, 1, 512, 0.9)):
        attn = torch.rand(B, H, M, N, generator=g)
        attn = attn / attn.sum(-1, keepdim=True)
        scores = torch.rand(N, generator=g)
        s_in = scores.clone()
        s_out = to.fused_importance_update(attn, scores, decay=decay)
        tag = f"imp_B{B}_H{H}_M{M}_N{N}"
        out[f"{tag}/attn"], out[f"{tag}/scores_in"] = attn.numpy(), s_in.numpy()
        out[f"{tag}/scores_out"] = s_out.numpy()
        out[f"{tag}/decay"] = np.array(decay)
    # zero attention: pure decay (tests/test_triton_ops.py:169-174 of the reference)
    s = torch.ones(32)
    out["imp_zero/scores_out"] = to.fused_importance_update(torch.zeros(1, 1, 1, 32), s, decay=0.5).numpy()

    AKVLayer = R["AKVLayer"]
    for (hot_len, budget, n_dem, seed) in ((600, 512, 88, 5), (160, 128, 32, 6), (1024, 256, 768, 7), (64, 16, 40, 8)):
        gg = torch.Generator().manual_seed(seed)
        scores = torch.randperm(hot_len * 4, generator=gg)[:hot_len].float() / (hot_len * 4)  # tie-free
        layer = AKVLayer(hot_budget=budget)
        layer._importance = scores.clone()
        idx = layer._select_demote_indices(n_dem, hot_len)
        tag = f"sel_n{hot_len}_b{budget}_k{n_dem}"
        out[f"{tag}/scores"] = scores.numpy()
        out[f"{tag}/idx"] = idx.numpy()
        out[f"{tag}/meta"] = np.array([hot_len, budget, n_dem])
    np.savez_compressed(os.path.join(HERE, "importance.npz"), **out)
    print("golden fixtures written to", HERE)


def make_drop_in_traces(ref_path: str):
    """AKVCache update traces of the reference (tier positions after every
    update, final chronological K/V view, byte accounting) for seeded inputs.

    Promotion, where enabled, is driven by attention weights on a grid of
    powers of two, so the promotion threshold test is exact on any device."""
    import torch
    torch.set_num_threads(1)
    sys.path.insert(0, ref_path)
    from akv.drop_in import AKVCache
    cases = {
        "a": dict(kw=dict(warm_bits=3, hot_budget=64, enable_promotion=False, enable_promotion_proxy=False),
                  steps=[200] + [1] * 20 + [40] + [1] * 10, attn=False, outlier=()),
        "b": dict(kw=dict(preset="k4v2", outlier_fraction=0.01, enable_promotion=True, enable_promotion_proxy=False,
                          promotion_threshold=0.3),
                  steps=[160] + [1] * 30, attn=True, outlier=(5,), budget=48),
        "c": dict(kw=dict(warm_bits=2, hot_budget=32, adaptive_hot_frac=0.25, enable_promotion=False,
                          enable_promotion_proxy=False),
                  steps=[300] + [1] * 20, attn=False, outlier=()),
    }
    out = {}
    H, D = 2, 64
    for name, c in cases.items():
        g = torch.Generator().manual_seed(ord(name))
        kw = dict(c["kw"])
        cache = AKVCache(num_hidden_layers=1, **kw)
        if "budget" in c:  # presets fix the budget; the trace uses a smaller one
            cache.hot_budget = c["budget"]
        warm_pos, hot_pos, ks, vs, attns = [], [], [], [], []
        total = 0
        for si, n in enumerate(c["steps"]):
            k = make_kv(g, H, n, D, outlier_ch=c["outlier"]).unsqueeze(0)
            v = make_kv(g, H, n, D).unsqueeze(0)
            ck = None
            if c["attn"] and si > 0:
                layer = cache.layers[0]
                warm_len = 0 if layer._warm_keys_fp16 is None else layer._warm_keys_fp16.shape[2]
                a = torch.zeros(1, H, 1, total + n)
                if warm_len:
                    pick = torch.randperm(warm_len, generator=g)[:3]
                    a[0, 0, 0, pick] = 0.5
                    a[0, 1, 0, pick[:2]] = 0.25
                ck = {"attention_weights": a}
                attns.append(a.reshape(-1).numpy())
            full_k, full_v = cache.update(k, v, 0, ck)
            total += n
            layer = cache.layers[0]
            warm_pos.append(np.array([] if layer._warm_positions is None else layer._warm_positions.tolist(),
                                     dtype=np.int64))
            hot_pos.append(layer._hot_positions.numpy().astype(np.int64))
            ks.append(k.numpy())
            vs.append(v.numpy())
        out[f"{name}/steps"] = np.array(c["steps"], dtype=np.int64)
        out[f"{name}/k_in"] = np.concatenate(ks, axis=2)
        out[f"{name}/v_in"] = np.concatenate(vs, axis=2)
        out[f"{name}/warm_pos"] = np.concatenate(warm_pos)
        out[f"{name}/warm_len"] = np.array([len(w) for w in warm_pos], dtype=np.int64)
        out[f"{name}/hot_pos"] = np.concatenate(hot_pos)
        out[f"{name}/hot_len"] = np.array([len(h) for h in hot_pos], dtype=np.int64)
        if attns:
            out[f"{name}/attn"] = np.concatenate(attns)
            out[f"{name}/attn_len"] = np.array([len(a) for a in attns], dtype=np.int64)
        out[f"{name}/full_k"] = full_k.numpy()
        out[f"{name}/full_v"] = full_v.numpy()
        mu = cache.memory_usage()
        for key in ("hot_bytes", "warm_bytes_packed", "warm_bytes_live", "fp16_equivalent_bytes", "total_bytes"):
            out[f"{name}/mem/{key}"] = np.array(mu[key], dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "drop_in.npz"), **out)
    print("drop-in traces written to", HERE)


def make_per_head_trace(ref_path: str):
    """AKVCache update trace of the reference with calibrated per-head bit
    widths on layer 0 (drop_in.py:315-374: each head quantised on its own at
    its width, outlier channels from that head alone): positions after every
    update, the final chronological K/V view, byte accounting."""
    import torch
    torch.set_num_threads(1)
    sys.path.insert(0, ref_path)
    from akv.drop_in import AKVCache
    out = {}
    H, D, name = 2, 64, "d"
    steps = [200] + [1] * 20 + [40] + [1] * 10
    g = torch.Generator().manual_seed(ord(name))
    cache = AKVCache(num_hidden_layers=1, warm_bits=3, hot_budget=64, outlier_fraction=0.05,
                     enable_promotion=False, enable_promotion_proxy=False)
    cache._calibration_per_head_bits = {0: [2, 4]}
    warm_pos, hot_pos, ks, vs = [], [], [], []
    for n in steps:
        k = make_kv(g, H, n, D, outlier_ch=(7,)).unsqueeze(0)
        v = make_kv(g, H, n, D).unsqueeze(0)
        full_k, full_v = cache.update(k, v, 0)
        layer = cache.layers[0]
        assert layer.per_head_bits == [2, 4]
        warm_pos.append(np.array([] if layer._warm_positions is None else layer._warm_positions.tolist(),
                                 dtype=np.int64))
        hot_pos.append(layer._hot_positions.numpy().astype(np.int64))
        ks.append(k.numpy())
        vs.append(v.numpy())
    out[f"{name}/steps"] = np.array(steps, dtype=np.int64)
    out[f"{name}/k_in"] = np.concatenate(ks, axis=2)
    out[f"{name}/v_in"] = np.concatenate(vs, axis=2)
    out[f"{name}/warm_pos"] = np.concatenate(warm_pos)
    out[f"{name}/warm_len"] = np.array([len(w) for w in warm_pos], dtype=np.int64)
    out[f"{name}/hot_pos"] = np.concatenate(hot_pos)
    out[f"{name}/hot_len"] = np.array([len(h) for h in hot_pos], dtype=np.int64)
    out[f"{name}/full_k"] = full_k.numpy()
    out[f"{name}/full_v"] = full_v.numpy()
    mu = cache.memory_usage()
    for key in ("hot_bytes", "warm_bytes_packed", "warm_bytes_live", "fp16_equivalent_bytes", "total_bytes"):
        out[f"{name}/mem/{key}"] = np.array(mu[key], dtype=np.int64)
    np.savez_compressed(os.path.join(HERE, "drop_in_per_head.npz"), **out)
    print("per-head trace written to", HERE)


def make_migrator_trace(ref_path: str):
    """ImportanceBasedMigrator (akv/vmm.py:113-245) of the reference driven by
    seeded attention: importance and eviction candidates after some steps.
    Attention is continuous (no ties among candidates); positions grow."""
    import torch
    torch.set_num_threads(1)
    sys.path.insert(0, ref_path)
    from akv.vmm import ImportanceBasedMigrator, VMMConfig
    cfg = VMMConfig(importance_decay=0.9, protect_initial=4, protect_recent=32)
    mig = ImportanceBasedMigrator(cfg)
    g = torch.Generator().manual_seed(9)
    out = {}
    B, H = 1, 2
    N = 700
    snaps = 0
    for step in range(40):
        N += 3
        logits = torch.randn(B, H, 1, N, generator=g) * 3
        attn = torch.softmax(logits, dim=-1)
        out[f"attn{step}"] = attn.numpy()
        mig.update(0, attn, N)
        if step % 7 == 3:
            idx = torch.randperm(N, generator=g)[:5]
            out[f"promote{step}"] = idx.numpy()
            mig.mark_promoted(0, idx)
        if step % 5 == 4:
            out[f"imp{step}"] = mig.compute_importance(0, N).numpy()
            out[f"evict{step}"] = mig.get_eviction_candidates(0, N, 50).numpy()
            snaps += 1
        mig.advance_step()
    np.savez_compressed(os.path.join(HERE, "migrator.npz"), **out)
    print("migrator trace written to", HERE, snaps, "snapshots")


def make_group_format(ref_path: str):
    """The reference's group-format tier (per token, per D-group, packed
    bytes): KVQuantizer quantise / dequantise (akv/quantizer.py:71-191), the
    dequantiser of the kernel API (triton_ops._dequantize_packed,
    akv/triton_ops.py:657-715), triton_kernels.fused_quantize_evict
    (akv/triton_kernels.py:426-500) in fp16, and fp32 attention over hot +
    dequantised warm with its softmax weights (the recipe of
    triton_kernels._fused_decode_attention_dispatch :350-390 and
    triton_ops._fused_mixed_attention_torch :518-551, in fp32)."""
    import torch
    torch.set_num_threads(1)
    sys.path.insert(0, ref_path)
    from akv.quantizer import KVQuantizer, QuantConfig
    from akv import triton_ops, triton_kernels
    g = torch.Generator().manual_seed(21)
    out = {}
    cases = [(40, 128, 32), (33, 72, 32), (16, 64, 64), (24, 128, 128)]
    for bits in (2, 4, 8):
        for ci, (N, D, gs) in enumerate(cases):
            x = torch.randn(N, D, generator=g)
            x[:, 5] *= 12.0
            x[3] = 0.75  # a constant row: zero range in every group
            x = x.half()
            tag = f"b{bits}_c{ci}"
            out[f"x_{tag}"] = x.numpy()
            for sym in (False, True):
                qz = KVQuantizer(QuantConfig(bits=bits, group_size=gs, symmetric=sym))
                qt = qz.quantize(x)
                st = f"{tag}_{'s' if sym else 'a'}"
                out[f"data_{st}"] = qt.data.numpy()
                out[f"scales_{st}"] = qt.scales.numpy()
                out[f"zeros_{st}"] = qt.zeros.numpy()
                out[f"deq_{st}"] = qz.dequantize(qt).numpy()
                out[f"dp_{st}"] = triton_ops._dequantize_packed(qt.data, qt.scales, qt.zeros, bits, gs, N, D,
                                                                 "cpu", torch.float16).numpy()
            v = torch.randn(N, D, generator=g).half()
            mask = torch.rand(N, generator=g) < 0.5
            mask[3] = True
            out[f"v_{tag}"] = v.numpy()
            out[f"mask_{tag}"] = mask.numpy()
            res = triton_kernels.fused_quantize_evict(x, v, mask, bits=bits, group_size=gs)
            for name, t in zip(("kp", "ks", "kz", "vp", "vs", "vz"), res):
                out[f"qe_{name}_{tag}"] = t.numpy()
    # attention over hot (B, H, N_hot, D) + a 4-bit group-format warm tier (N_warm, D)
    B, H, M, D, n_hot, n_warm, gs = 2, 3, 2, 128, 20, 70, 32
    q = torch.randn(B, H, M, D, generator=g).half()
    hk = torch.randn(B, H, n_hot, D, generator=g).half()
    hv = torch.randn(B, H, n_hot, D, generator=g).half()
    wk = torch.randn(n_warm, D, generator=g).half()
    wv = torch.randn(n_warm, D, generator=g).half()
    qz = KVQuantizer(QuantConfig(bits=4, group_size=gs))
    kq, vq = qz.quantize(wk), qz.quantize(wv)
    dk = triton_ops._dequantize_packed(kq.data, kq.scales, kq.zeros, 4, gs, n_warm, D, "cpu", torch.float16)
    dv = triton_ops._dequantize_packed(vq.data, vq.scales, vq.zeros, 4, gs, n_warm, D, "cpu", torch.float16)
    keys = torch.cat([hk, dk.expand(B, H, -1, -1)], 2).float()
    vals = torch.cat([hv, dv.expand(B, H, -1, -1)], 2).float()
    w = torch.softmax(torch.matmul(q.float(), keys.transpose(-2, -1)) / math.sqrt(D), dim=-1)
    out.update(att_q=q.numpy(), att_hk=hk.numpy(), att_hv=hv.numpy(), att_kd=kq.data.numpy(),
               att_ks=kq.scales.numpy(), att_kz=kq.zeros.numpy(), att_vd=vq.data.numpy(), att_vs=vq.scales.numpy(),
               att_vz=vq.zeros.numpy(), att_gs=np.int64(gs), att_out=torch.matmul(w, vals).numpy(),
               att_w=w.numpy())
    np.savez_compressed(os.path.join(HERE, "group_format.npz"), **out)
    print("group-format fixtures written to", HERE)


def _reference_path() -> str:
    """The reference source tree: the first argument, else $AKV_REFERENCE."""
    path = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("AKV_REFERENCE", "")
    if not path:
        sys.exit("usage: make_golden.py <reference source path> [migrator|drop_in|per_head|group_format] "
                 "(or set AKV_REFERENCE)")
    return path


if __name__ == "__main__":
    if len(sys.argv) > 2 and sys.argv[2] == "migrator":
        make_migrator_trace(sys.argv[1])
        sys.exit(0)
    if len(sys.argv) > 2 and sys.argv[2] == "drop_in":
        make_drop_in_traces(sys.argv[1])
    elif len(sys.argv) > 2 and sys.argv[2] == "per_head":
        make_per_head_trace(sys.argv[1])
    elif len(sys.argv) > 2 and sys.argv[2] == "group_format":
        make_group_format(sys.argv[1])
    else:
        ref = _reference_path()
        main(ref)
        make_drop_in_traces(ref)
        make_migrator_trace(ref)
        make_per_head_trace(ref)
        make_group_format(ref)
