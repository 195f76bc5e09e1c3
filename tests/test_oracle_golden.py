"""Pin the numpy oracle against golden vectors produced by the reference itself.

The fixtures under ``tests/golden`` were written by ``make_golden.py``, which
calls the reference package (``akv.bitpack``, ``AffineQuantizer``,
``fused_attention``, ``triton_ops.fused_importance_update`` and
``AKVLayer._select_demote_indices``) on seeded inputs.
"""
import os

import numpy as np
import pytest

from oracle import akv_oracle as O


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name), allow_pickle=False)


def test_bitpack_golden(golden_dir):
    z = _load(golden_dir, "bitpack.npz")
    for bits in (2, 3, 4):
        for D in (8, 32, 64, 128, 256):
            codes = z[f"b{bits}_d{D}_codes"]
            packed = O.pack(codes, bits)
            assert packed.shape[-1] == O.packed_width(D, bits)
            np.testing.assert_array_equal(packed, z[f"b{bits}_d{D}_packed"])
            np.testing.assert_array_equal(O.unpack(packed, bits, D), z[f"b{bits}_d{D}_unpacked"])
    for bits, D in ((4, 7), (3, 13), (2, 10)):
        np.testing.assert_array_equal(O.pack(z[f"b{bits}_d{D}_codes"], bits), z[f"b{bits}_d{D}_packed"])


def _affine_cases(z):
    return [str(n) for n in z["names"]]


def test_affine_quantizer_golden(golden_dir):
    z = _load(golden_dir, "affine.npz")
    flips = 0
    for name in _affine_cases(z):
        kb, vb, frac = z[f"{name}/meta"]
        kb, vb = int(kb), int(vb)
        for tag, x, bits, fn in (("qk", z[f"{name}/k"], kb, O.quantize_keys),
                                 ("qv", z[f"{name}/v"], vb, O.quantize_values)):
            q = fn(x, bits, float(frac))
            if f"{name}/{tag}_outlier_idx" in z.files:
                ref_idx = z[f"{name}/{tag}_outlier_idx"]
                if not np.array_equal(np.sort(q["outlier_idx"]), np.sort(ref_idx)):
                    flips += 1
                    continue
                np.testing.assert_array_equal(q["outlier_idx"], ref_idx, err_msg=name)
                np.testing.assert_array_equal(q["outlier_data"], z[f"{name}/{tag}_outlier_data"], err_msg=name)
            np.testing.assert_array_equal(q["codes"], z[f"{name}/{tag}_codes"], err_msg=f"{name} {tag} codes")
            np.testing.assert_array_equal(q["scale"].view(np.uint16), z[f"{name}/{tag}_scale"].view(np.uint16),
                                          err_msg=f"{name} {tag} scale")
            np.testing.assert_array_equal(q["zero"].view(np.uint16), z[f"{name}/{tag}_zero"].view(np.uint16),
                                          err_msg=f"{name} {tag} zero")
            deq = O._dequant(q)
            np.testing.assert_array_equal(deq.view(np.uint16), z[f"{name}/{tag}_deq"].view(np.uint16),
                                          err_msg=f"{name} {tag} dequant")
            assert O.measure_packed_bytes(q, bits) == int(z[f"{name}/{tag}_bytes"])
    # outlier top-n may only differ on near-ties of fp32 channel norms
    assert flips == 0, f"{flips} outlier-channel selections differ from the reference"


def test_config1_groups_golden(golden_dir):
    z = _load(golden_dir, "config1_groups.npz")
    k = z["k"][None]
    v = z["v"][None]
    gk = O.quantize_groups(k, 3, 32, True)
    gv = O.quantize_groups(v, 3, 32, False)
    for j in range(k.shape[2] // 32):
        for key in ("codes", "scale", "zero"):
            np.testing.assert_array_equal(np.asarray(gk[0][j][key]).view(np.uint8),
                                          z[f"g{j}/qk_{key}"].view(np.uint8))
            np.testing.assert_array_equal(np.asarray(gv[0][j][key]).view(np.uint8),
                                          z[f"g{j}/qv_{key}"].view(np.uint8))


def test_attention_golden(golden_dir):
    z = _load(golden_dir, "attention.npz")
    for (B, H, N, D) in ((1, 4, 64, 64), (2, 2, 100, 128)):
        t = f"hot_B{B}_H{H}_N{N}_D{D}"
        out = O.decode_attention(z[f"{t}/q"][:, :, 0], z[f"{t}/k"], z[f"{t}/v"])
        np.testing.assert_allclose(out.astype(np.float16).astype(np.float32),
                                   z[f"{t}/out"][:, :, 0].astype(np.float32), atol=2e-3, rtol=0)
    for gs in (32, 128):
        t = f"int4_gs{gs}"
        D = z[f"{t}/q"].shape[-1]
        dk = O.int4_group_dequant(z[f"{t}/wkp"], z[f"{t}/wks"], z[f"{t}/wkz"], D, gs)
        np.testing.assert_array_equal(dk.view(np.uint16), z[f"{t}/deq_k"].view(np.uint16))
        dv = O.int4_group_dequant(z[f"{t}/wvp"], z[f"{t}/wvs"], z[f"{t}/wvz"], D, gs)
        B = z[f"{t}/q"].shape[0]
        wk = np.broadcast_to(dk[None], (B,) + dk.shape)
        wv = np.broadcast_to(dv[None], (B,) + dv.shape)
        keys = np.concatenate([z[f"{t}/hk"], wk], 2)
        vals = np.concatenate([z[f"{t}/hv"], wv], 2)
        out = O.decode_attention(z[f"{t}/q"][:, :, 0], keys, vals)
        np.testing.assert_allclose(out, z[f"{t}/mixed"][:, :, 0].astype(np.float32), atol=2e-3, rtol=0)
        out_w = O.decode_attention(z[f"{t}/q"][:, :, 0], wk, wv)
        for tag in ("int4", "int4_tiled"):
            np.testing.assert_allclose(out_w, z[f"{t}/{tag}"][:, :, 0].astype(np.float32), atol=2e-3, rtol=0)
    t = "affine_gqa"
    wk, wv = z[f"{t}/wk"], z[f"{t}/wv"]
    dk = O.dequantize_groups(O.quantize_groups(wk, 3, 32, True))
    dv = O.dequantize_groups(O.quantize_groups(wv, 3, 32, False))
    keys = np.concatenate([dk, z[f"{t}/hk"]], 2)
    vals = np.concatenate([dv, z[f"{t}/hv"]], 2)
    out = O.decode_attention(z[f"{t}/q"][:, :, 0], keys, vals)
    np.testing.assert_allclose(out, z[f"{t}/out"][:, :, 0].astype(np.float32), atol=2e-3, rtol=0)


def test_importance_golden(golden_dir):
    z = _load(golden_dir, "importance.npz")
    for (B, H, M, N) in ((1, 4, 1, 64), (2, 8, 3, 257), (8, 8, 1, 512)):
        t = f"imp_B{B}_H{H}_M{M}_N{N}"
        s = O.importance_update(z[f"{t}/attn"], z[f"{t}/scores_in"], float(z[f"{t}/decay"]))
        np.testing.assert_array_equal(s, z[f"{t}/scores_out"])
    s = O.importance_update(np.zeros((1, 1, 1, 32), np.float32), np.ones(32, np.float32), 0.5)
    np.testing.assert_array_equal(s, z["imp_zero/scores_out"])
    for key in [k for k in z.files if k.startswith("sel_") and k.endswith("/meta")]:
        t = key[:-5]
        hot_len, budget, n_dem = (int(x) for x in z[key])
        idx = O.select_demote(z[f"{t}/scores"], n_dem, budget)
        np.testing.assert_array_equal(idx, z[f"{t}/idx"], err_msg=t)


# ---------------------------------------------------------------------------- group format
def test_group_format_oracle_matches_reference(golden_dir):
    """The group-format dequantiser (triton_ops._dequantize_packed, also
    KVQuantizer.dequantize) and fused_quantize_evict's fp16 quantiser against
    the reference's own outputs, bit for bit."""
    f = _load(golden_dir, "group_format.npz")
    cases = [(40, 128, 32), (33, 72, 32), (16, 64, 64), (24, 128, 128)]
    for bits in (2, 4, 8):
        for ci, (N, D, gs) in enumerate(cases):
            tag = f"b{bits}_c{ci}"
            for st in ("a", "s"):
                k = f"{tag}_{st}"
                d = O.group_dequantize(f[f"data_{k}"], f[f"scales_{k}"], f[f"zeros_{k}"], bits, gs, N, D)
                np.testing.assert_array_equal(d.view(np.uint16), f[f"dp_{k}"].view(np.uint16))
                np.testing.assert_array_equal(d.view(np.uint16), f[f"deq_{k}"].view(np.uint16))
            x, mask = f[f"x_{tag}"], f[f"mask_{tag}"]
            for src, pre in ((x, "k"), (f[f"v_{tag}"], "v")):
                p, s, z = O.group_quantize_fp16(src[mask], bits, gs)
                np.testing.assert_array_equal(p, f[f"qe_{pre}p_{tag}"])
                np.testing.assert_array_equal(s.view(np.uint16), f[f"qe_{pre}s_{tag}"].view(np.uint16))
                np.testing.assert_array_equal(z.view(np.uint16), f[f"qe_{pre}z_{tag}"].view(np.uint16))


@pytest.mark.parametrize("shape", [(1, 4, 1, 64), (2, 8, 3, 257), (8, 8, 1, 512), (16, 32, 1, 1000), (4, 8, 2, 3000),
                                   (8, 8, 1, 4099), (3, 5, 17, 100), (2, 2, 1, 5), (5, 7, 3, 33), (32, 16, 1, 2000)])
def test_importance_order_is_torch_cpu_order(shape):
    """The oracle's reduction order equals torch's own CPU result on this
    host, bit for bit, across column counts that exercise every path (whole
    blocks, one register, scalar tail) and row counts that exercise every
    cascade level."""
    import torch
    from akv import _C
    torch.set_num_threads(1)
    rng = np.random.default_rng(sum(shape))
    a = rng.random(shape).astype(np.float32)
    a /= a.sum(-1, keepdims=True)
    s = rng.random(shape[-1]).astype(np.float32)
    ref = (torch.from_numpy(s) * 0.9 + torch.from_numpy(a).mean(dim=(0, 1)).sum(dim=0)).numpy()
    out = O.importance_update(a, s, 0.9, vec_width=_C.cpu_reduction_width())
    np.testing.assert_array_equal(out, ref)
