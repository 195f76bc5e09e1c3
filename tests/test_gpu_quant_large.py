"""Scale groups larger than one CTA's shared memory: the chunked quantiser
path (per-chunk column partials -> per-group reduction -> encode), checked
bit-exact against the oracle (one reference quantiser call per group).

Covers AffineQuantizer calls over many tokens (the reference quantises a
whole (H, N, D) tensor in one call, affine_quantizer.py:63-110 / :131-176),
AKVLayer-style demotion events quantised as one group
(drop_in.py:699-701), heads split across CTAs (H * 32 * D too large for one
CTA), and the workspace contract of akv_quantize_ws.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle.akv_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _akv():
    import akv
    return akv


def _np(t):
    return t.detach().cpu().numpy()


def _bits16(a):
    h = np.ascontiguousarray(np.asarray(a, dtype=np.float16))
    bits = h.view(np.uint16).copy()
    bits[np.isnan(h)] = 0x7E00
    return bits


def _rand(seed, shape, outlier_ch=(), scale=12.0):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(shape).astype(np.float32)
    for c in outlier_ch:
        x[..., c] *= scale
    return x.astype(np.float16)


def _compare(q, ref, tag):
    np.testing.assert_array_equal(_np(q["codes"]), np.asarray(ref["codes"]), err_msg=f"{tag} codes")
    np.testing.assert_array_equal(_bits16(_np(q["scale"])), _bits16(ref["scale"]), err_msg=f"{tag} scale")
    np.testing.assert_array_equal(_bits16(_np(q["zero"])), _bits16(ref["zero"]), err_msg=f"{tag} zero")
    if "outlier_idx" in ref:
        np.testing.assert_array_equal(_np(q["outlier_idx"]), np.asarray(ref["outlier_idx"]), err_msg=f"{tag} oidx")
        np.testing.assert_array_equal(_bits16(_np(q["outlier_data"])), _bits16(ref["outlier_data"]),
                                      err_msg=f"{tag} odata")


@pytest.mark.parametrize("bits,frac,shape", [
    (3, 0.0, (2, 3584, 128)),     # config 1's warm tier as one call
    (3, 0.01, (2, 3584, 128)),
    (4, 0.01, (8, 517, 128)),     # ragged last chunk
    (2, 0.05, (4, 300, 64)),
    (4, 0.0, (32, 64, 128)),      # 32 heads: split across CTAs
    (2, 0.03, (32, 96, 128)),
])
def test_affine_quantizer_large_calls_vs_oracle(bits, frac, shape):
    akv = _akv()
    H, N, D = shape
    seed = hash((bits, frac, shape)) % (2 ** 31)
    k = _rand(seed, shape, outlier_ch=[seed % D])
    v = _rand(seed + 1, shape)
    qz = akv.AffineQuantizer(akv.AffineQuantConfig(key_bits=bits, value_bits=bits, outlier_fraction=frac))
    for x, fn, ofn, dfn in ((k, qz.quantize_keys, O.quantize_keys, qz.dequantize_keys),
                            (v, qz.quantize_values, O.quantize_values, qz.dequantize_values)):
        q = fn(torch.from_numpy(x).to(DEV))
        ref = ofn(x, bits, frac)
        _compare(q, ref, f"{shape} b{bits} f{frac}")
        np.testing.assert_array_equal(_bits16(_np(dfn(q))), _bits16(O._dequant(ref)))


def test_large_demotion_event_into_arena_vs_oracle():
    """A 700-token demote event gathered by index, one scale group, k4v2 + outliers."""
    akv = _akv()
    B, H, Ncap, D, n_ev = 2, 8, 1500, 128, 700
    rng = np.random.default_rng(3)
    hot_k = _rand(4, (B, H, Ncap, D), outlier_ch=[17])
    hot_v = _rand(5, (B, H, Ncap, D))
    idx = np.stack([np.sort(rng.choice(Ncap, n_ev, replace=False)) for _ in range(B)]).astype(np.int64)
    arena = akv.WarmArena(B, H, D, 4, 2, outlier_fraction=0.01, max_blocks=(n_ev + 31) // 32, device=DEV)
    arena.append(torch.from_numpy(hot_k).to(DEV), torch.from_numpy(hot_v).to(DEV), group=10 ** 9,
                 tok_idx=torch.from_numpy(idx).to(DEV))
    dk, dv = arena.dequantize(n_tokens=n_ev)
    from akv.packed_layout import key_scale_channels
    L = arena.layout
    buf = _np(arena.buf)
    for b in range(B):
        rk = O.quantize_keys(hot_k[b][:, idx[b]], 4, 0.01)
        rv = O.quantize_values(hot_v[b][:, idx[b]], 2, 0.01)
        np.testing.assert_array_equal(_bits16(_np(dk[b])), _bits16(O._dequant(rk)))
        np.testing.assert_array_equal(_bits16(_np(dv[b])), _bits16(O._dequant(rv)))
        for h in range(H):  # the group's key scale sits in every block record it covers
            for blk in range(arena.n_blocks):
                rec = buf[b, h, blk]
                np.testing.assert_array_equal(rec[L.ks:L.ks + 2 * D].view(np.uint16),
                                              _bits16(rk["scale"][h, 0])[key_scale_channels(4, D)])
                np.testing.assert_array_equal(rec[L.ki:L.ki + 2].view(np.int16), rk["outlier_idx"])


def test_chunked_shape_needs_workspace():
    akv = _akv()
    from akv import _C
    lib = _C.load()
    H, N, D = 8, 1024, 128
    need = lib.akv_quantize_workspace_bytes(1, H, N, D, N, 1, 1)
    assert need > 0
    assert lib.akv_quantize_workspace_bytes(1, H, 32, D, 32, 1, 1) == 0  # one CTA per group
    x = torch.zeros(H, N, D, dtype=torch.float16, device=DEV)
    codes = torch.empty(H, N, D // 2, dtype=torch.uint8, device=DEV)
    scale = torch.empty(H, 1, D, dtype=torch.float16, device=DEV)
    zero = torch.empty(H, 1, D, dtype=torch.float16, device=DEV)
    od = torch.empty(H, N, 1, dtype=torch.float16, device=DEV)
    oi = torch.empty(1, dtype=torch.int16, device=DEV)
    dest = akv.affine_quantizer.dict_dest(codes, scale, zero, od, oi, N, D, 4, 1, True)
    rc = lib.akv_quantize(x.data_ptr(), 0, N * D, D, None, 0, 0, 1, H, N, D, 4, 1, N, 1, ctypes.byref(dest), None,
                          torch.cuda.current_stream().cuda_stream)
    assert rc == -8  # AKV_ERR_WORKSPACE
    ws = torch.empty(need - 256, dtype=torch.uint8, device=DEV)
    rc = lib.akv_quantize_ws(x.data_ptr(), 0, N * D, D, None, 0, 0, 1, H, N, D, 4, 1, N, 1, ctypes.byref(dest),
                             ws.data_ptr(), need - 256, None, torch.cuda.current_stream().cuda_stream)
    assert rc == -8
