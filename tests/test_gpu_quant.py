"""GPU parity: bit packing, quantise + pack, dequantise vs the oracle and the goldens.

Bar: bit-exact codes, scales, zeros, outlier ids/data and dequantised fp16.
"""
import os

import numpy as np
import pytest
import torch

from oracle import akv_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _akv():
    import akv
    return akv


def _np(t):
    return t.detach().cpu().numpy()


def _bits16(a):
    """fp16 bit patterns, with every NaN mapped to one canonical pattern (NaN payloads
    differ between torch's CPU kernels and the GPU; NaN arises only from inf scales)."""
    h = np.ascontiguousarray(np.asarray(a, dtype=np.float16))
    bits = h.view(np.uint16).copy()
    bits[np.isnan(h)] = 0x7E00
    return bits


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("dim", [7, 8, 13, 32, 64, 128, 256])
def test_pack_unpack_vs_oracle(bits, dim):
    akv = _akv()
    g = torch.Generator().manual_seed(bits * 1000 + dim)
    codes = torch.randint(0, 1 << bits, (3, 17, dim), generator=g, dtype=torch.uint8)
    packed = akv.bitpack.pack(codes.to(DEV), bits)
    np.testing.assert_array_equal(_np(packed), O.pack(_np(codes), bits))
    if bits == 2 and dim % 4:
        return  # the reference cannot unpack widths that are not a multiple of 4
    back = akv.bitpack.unpack(packed, bits, dim)
    np.testing.assert_array_equal(_np(back), _np(codes))


def test_bitpack_golden(golden_dir):
    akv = _akv()
    z = np.load(os.path.join(golden_dir, "bitpack.npz"))
    for bits in (2, 3, 4):
        for D in (8, 32, 64, 128, 256):
            c = torch.from_numpy(z[f"b{bits}_d{D}_codes"]).to(DEV)
            np.testing.assert_array_equal(_np(akv.bitpack.pack(c, bits)), z[f"b{bits}_d{D}_packed"])


def _compare_q(q, ref, tag):
    np.testing.assert_array_equal(_np(q["codes"]), np.asarray(ref["codes"]), err_msg=f"{tag} codes")
    np.testing.assert_array_equal(_bits16(_np(q["scale"])), _bits16(ref["scale"]), err_msg=f"{tag} scale")
    np.testing.assert_array_equal(_bits16(_np(q["zero"])), _bits16(ref["zero"]), err_msg=f"{tag} zero")
    if "outlier_idx" in ref:
        np.testing.assert_array_equal(_np(q["outlier_idx"]), np.asarray(ref["outlier_idx"]), err_msg=f"{tag} oidx")
        np.testing.assert_array_equal(_bits16(_np(q["outlier_data"])), _bits16(ref["outlier_data"]),
                                      err_msg=f"{tag} odata")
    else:
        assert "outlier_idx" not in q


def test_affine_golden(golden_dir):
    """Every golden case with D % 32 == 0: CUDA output == reference output, bit for bit."""
    akv = _akv()
    z = np.load(os.path.join(golden_dir, "affine.npz"))
    ran = 0
    for name in [str(n) for n in z["names"]]:
        k = z[f"{name}/k"]
        if k.shape[-1] % 32:
            continue
        kb, vb, frac = z[f"{name}/meta"]
        qz = akv.AffineQuantizer(akv.AffineQuantConfig(key_bits=int(kb), value_bits=int(vb),
                                                       outlier_fraction=float(frac)))
        for tag, x, fn, dfn in (("qk", k, qz.quantize_keys, qz.dequantize_keys),
                                ("qv", z[f"{name}/v"], qz.quantize_values, qz.dequantize_values)):
            q = fn(torch.from_numpy(x).to(DEV))
            ref = {key: z[f"{name}/{tag}_{key}"] for key in ("codes", "scale", "zero")}
            if f"{name}/{tag}_outlier_idx" in z.files:
                ref["outlier_idx"] = z[f"{name}/{tag}_outlier_idx"]
                ref["outlier_data"] = z[f"{name}/{tag}_outlier_data"]
            _compare_q(q, ref, f"{name}/{tag}")
            np.testing.assert_array_equal(_bits16(_np(dfn(q))), _bits16(z[f"{name}/{tag}_deq"]),
                                          err_msg=f"{name}/{tag} dequant")
            assert akv.measure_packed_bytes(q, int(kb if tag == "qk" else vb)) == int(z[f"{name}/{tag}_bytes"])
        ran += 1
    assert ran >= 30


def _rand_kv(seed, H, N, D, outlier_ch=(), scale=12.0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((H, N, D)).astype(np.float32)
    for c in outlier_ch:
        x[..., c] *= scale
    return x.astype(np.float16)


@pytest.mark.parametrize("bits", [2, 3, 4])
@pytest.mark.parametrize("frac", [0.0, 0.01, 0.1])
@pytest.mark.parametrize("shape", [(1, 1, 128), (2, 32, 128), (8, 32, 128), (4, 77, 64), (2, 3, 256), (3, 300, 32)])
def test_quantize_vs_oracle(bits, frac, shape):
    akv = _akv()
    H, N, D = shape
    seed = hash((bits, frac, shape)) % (2 ** 31)
    k = _rand_kv(seed, H, N, D, outlier_ch=[seed % D])
    v = _rand_kv(seed + 1, H, N, D, outlier_ch=[(seed // 7) % D])
    qz = akv.AffineQuantizer(akv.AffineQuantConfig(key_bits=bits, value_bits=bits, outlier_fraction=frac))
    for x, fn, ofn, dfn in ((k, qz.quantize_keys, O.quantize_keys, qz.dequantize_keys),
                            (v, qz.quantize_values, O.quantize_values, qz.dequantize_values)):
        q = fn(torch.from_numpy(x).to(DEV))
        ref = ofn(x, bits, frac)
        _compare_q(q, ref, f"{shape} b{bits} f{frac}")
        np.testing.assert_array_equal(_bits16(_np(dfn(q))), _bits16(O._dequant(ref)))


def test_quantize_unpacked_codes():
    akv = _akv()
    x = _rand_kv(5, 2, 32, 128)
    qz = akv.AffineQuantizer(akv.AffineQuantConfig(key_bits=3, value_bits=3, packed=False))
    q = qz.quantize_keys(torch.from_numpy(x).to(DEV))
    ref = O.quantize_keys(x, 3, 0.0, packed=False)
    np.testing.assert_array_equal(_np(q["codes"]), ref["codes"])
    np.testing.assert_array_equal(_bits16(_np(qz.dequantize_keys(q))), _bits16(O._dequant(ref)))


def test_quantize_rejects_non_fp16_and_cpu():
    akv = _akv()
    qz = akv.AffineQuantizer(akv.AffineQuantConfig())
    with pytest.raises(TypeError):
        qz.quantize_keys(torch.zeros(2, 4, 128, device=DEV, dtype=torch.float32))
    with pytest.raises(RuntimeError):
        qz.quantize_keys(torch.zeros(2, 4, 128, dtype=torch.float16))


@pytest.mark.parametrize("kb,vb,frac", [(3, 3, 0.0), (4, 2, 0.01), (2, 2, 0.05), (4, 4, 0.0), (4, 3, 0.01)])
def test_warm_arena_groups_vs_oracle(kb, vb, frac):
    """Arena records written per 32-token group == one reference call per group and batch row."""
    akv = _akv()
    B, H, N, D = 3, 4, 32 * 5 + 7, 128
    rng = np.random.default_rng(kb * 10 + vb)
    k = rng.standard_normal((B, H, N, D)).astype(np.float16)
    v = rng.standard_normal((B, H, N, D)).astype(np.float16)
    k[..., 9] *= 12
    arena = akv.WarmArena(B, H, D, kb, vb, outlier_fraction=frac, max_blocks=8, device=DEV)
    arena.append(torch.from_numpy(k).to(DEV), torch.from_numpy(v).to(DEV), group=32)
    assert arena.n_blocks == 6
    dk, dv = arena.dequantize(n_tokens=N)
    gk = O.quantize_groups(k, kb, 32, True, frac)
    gv = O.quantize_groups(v, vb, 32, False, frac)
    np.testing.assert_array_equal(_bits16(_np(dk)), _bits16(O.dequantize_groups(gk)))
    np.testing.assert_array_equal(_bits16(_np(dv)), _bits16(O.dequantize_groups(gv)))
    # raw record fields == oracle dict fields
    from akv.packed_layout import key_scale_channels
    L = arena.layout
    buf = _np(arena.buf)
    dpk, dpv = O.packed_width(D, kb), O.packed_width(D, vb)
    for b in range(B):
        for j, (qk, qv) in enumerate(zip(gk[b], gv[b])):
            nt = qk["codes"].shape[1]
            for h in range(H):
                rec = buf[b, h, j]
                np.testing.assert_array_equal(rec[L.kc:L.kc + nt * dpk].reshape(nt, dpk), qk["codes"][h])
                np.testing.assert_array_equal(rec[L.vc:L.vc + nt * dpv].reshape(nt, dpv), qv["codes"][h])
                # K scale / zero in the decode pair order
                perm = key_scale_channels(kb, D)
                np.testing.assert_array_equal(rec[L.ks:L.ks + 2 * D].view(np.uint16), _bits16(qk["scale"][h, 0])[perm])
                np.testing.assert_array_equal(rec[L.kz:L.kz + 2 * D].view(np.uint16), _bits16(qk["zero"][h, 0])[perm])
                np.testing.assert_array_equal(rec[L.vs:L.vs + 2 * nt].view(np.uint16), _bits16(qv["scale"][h, :, 0]))
                # decode flags: 1 where every scale is +0 or in [2^-14, 65504/1024]
                def dq2_ok(bits16):
                    return bool(np.all((bits16 == 0) | ((bits16 >= 0x0400) & (bits16 <= 0x53FF))))
                assert rec[L.flags] == dq2_ok(_bits16(qk["scale"][h, 0]))
                assert rec[L.flags + 1] == dq2_ok(_bits16(qv["scale"][h, :, 0]))
                mask = int(rec[L.mask:L.mask + 4].view(np.uint32)[0])
                assert mask == (0xFFFFFFFF if nt == 32 else (1 << nt) - 1)
                if frac > 0:
                    n = qk["outlier_idx"].shape[0]
                    np.testing.assert_array_equal(rec[L.ki:L.ki + 2 * n].view(np.int16), qk["outlier_idx"])
                    np.testing.assert_array_equal(rec[L.vi:L.vi + 2 * n].view(np.int16), qv["outlier_idx"])


def test_warm_arena_event_mode_and_gather():
    """One scale group over a whole demote event (the reference's AKVLayer call), rows gathered by index."""
    akv = _akv()
    B, H, Ncap, D = 1, 2, 200, 128
    rng = np.random.default_rng(11)
    hot_k = rng.standard_normal((B, H, Ncap, D)).astype(np.float16)
    hot_v = rng.standard_normal((B, H, Ncap, D)).astype(np.float16)
    idx = np.sort(rng.choice(Ncap, 70, replace=False)).astype(np.int64)
    arena = akv.WarmArena(B, H, D, 3, 3, max_blocks=4, device=DEV)
    arena.append(torch.from_numpy(hot_k).to(DEV), torch.from_numpy(hot_v).to(DEV), group=10 ** 9,
                 tok_idx=torch.from_numpy(idx).to(DEV))
    dk, dv = arena.dequantize(n_tokens=70)
    rk = O._dequant(O.quantize_keys(hot_k[0][:, idx], 3))
    rv = O._dequant(O.quantize_values(hot_v[0][:, idx], 3))
    np.testing.assert_array_equal(_bits16(_np(dk[0])), _bits16(rk))
    np.testing.assert_array_equal(_bits16(_np(dv[0])), _bits16(rv))


@pytest.mark.parametrize("kb,vb,frac,B", [(3, 3, 0.0, 1), (4, 2, 0.01, 2), (2, 4, 0.05, 1), (4, 4, 0.02, 3)])
def test_warm_demote_install_matches_append_then_copy(kb, vb, frac, B):
    """akv_warm_demote_install: the one-token record equals akv_warm_append's
    byte for byte, and the source ring row ends up holding the new token."""
    import ctypes
    akv = _akv()
    from akv import _C
    H, cap, D, r = 4, 96, 128, 37
    g = torch.Generator(device=DEV).manual_seed(kb * 7 + vb + B)
    ring = torch.randn(2, B, H, cap, D, generator=g, device=DEV).half()
    ring[..., 5] *= 12
    new = torch.randn(2, B, H, 1, D, generator=g, device=DEV).half()
    a = akv.WarmArena(B, H, D, kb, vb, outlier_fraction=frac, max_blocks=3, device=DEV)
    b = akv.WarmArena(B, H, D, kb, vb, outlier_fraction=frac, max_blocks=3, device=DEV)
    for ar in (a, b):  # one ordinary block first, so the records land at blk 1
        ar.append(ring[0, :, :, :32].contiguous(), ring[1, :, :, :32].contiguous(), group=32)
    a.append(ring[0, :, :, r:r + 1], ring[1, :, :, r:r + 1], group=1)
    expect = ring.clone()
    expect[:, :, :, r] = new[:, :, :, 0]
    work = ring.clone()
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    kr, vr = work[0, :, :, r], work[1, :, :, r]
    nk, nv = new[0, :, :, 0], new[1, :, :, 0]
    rc = _C.load().akv_warm_demote_install(
        b.buf.data_ptr(), b.buf.stride(0), b.buf.stride(1), ctypes.byref(b.layout), 1,
        kr.data_ptr(), kr.stride(0), kr.stride(1), vr.data_ptr(), vr.stride(0), vr.stride(1),
        nk.data_ptr(), nk.stride(0), nk.stride(1), nv.data_ptr(), nv.stride(0), nv.stride(1), B, H,
        st.data_ptr(), _C.stream_of(work))
    assert rc == 0
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert torch.equal(a.buf[:, :, :2], b.buf[:, :, :2])
    assert torch.equal(work, expect)
