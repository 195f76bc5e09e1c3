"""GPU parity: the group-format tier of the reference's older kernel API
(triton_ops / triton_kernels / fused_attention compatibility entries) and the
row scatter.

* ``group_dequantize`` against the reference's ``_dequantize_packed`` and
  ``KVQuantizer.dequantize`` outputs (golden, bit for bit), 2 / 4 / 8 bits,
  asymmetric and symmetric, rows padded to whole groups;
* ``fused_quantize_evict`` (triton_kernels) against the reference's outputs,
  bit for bit, including a constant row (0/0 scale);
* ``fused_mixed_precision_attention`` against fp32 attention over the
  reference-dequantised tiers: output within the decode bar, softmax weights
  within 1e-4;
* ``fused_quantized_attention``, ``triton_kernels.fused_decode_attention`` and
  ``fused_attention.fused_decode_attention`` / ``fused_quantize_evict``
  against the numpy oracle;
* ``scatter_rows`` against torch indexing, with an out-of-range index turned
  into a status code.
"""
import math
import os
import types

import numpy as np
import pytest
import torch

from oracle import akv_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
CASES = [(40, 128, 32), (33, 72, 32), (16, 64, 64), (24, 128, 128)]
ATOL = 2e-3


def _fx(golden_dir):
    return np.load(os.path.join(golden_dir, "group_format.npz"))


def _d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_group_dequantize_golden(golden_dir, bits):
    from akv.group_format import group_dequantize
    f = _fx(golden_dir)
    for ci, (N, D, gs) in enumerate(CASES):
        for st in ("a", "s"):
            k = f"b{bits}_c{ci}_{st}"
            out = group_dequantize(_d(f[f"data_{k}"]), _d(f[f"scales_{k}"]), _d(f[f"zeros_{k}"]), bits, gs, N, D)
            np.testing.assert_array_equal(out.cpu().numpy().view(np.uint16), f[f"dp_{k}"].view(np.uint16))


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_fused_quantize_evict_golden(golden_dir, bits):
    from akv.triton_kernels import fused_quantize_evict
    f = _fx(golden_dir)
    for ci, (N, D, gs) in enumerate(CASES):
        tag = f"b{bits}_c{ci}"
        res = fused_quantize_evict(_d(f[f"x_{tag}"]), _d(f[f"v_{tag}"]), _d(f[f"mask_{tag}"]), bits=bits,
                                   group_size=gs)
        for name, t in zip(("kp", "ks", "kz", "vp", "vs", "vz"), res):
            ref = f[f"qe_{name}_{tag}"]
            got = t.cpu().numpy()
            if got.dtype == np.float16:
                got, ref = got.view(np.uint16), ref.view(np.uint16)
            np.testing.assert_array_equal(got, ref, err_msg=f"{name} {tag}")


def test_fused_quantize_evict_nothing_selected():
    from akv.triton_kernels import fused_quantize_evict
    k = torch.randn(8, 64, device=DEV).half()
    res = fused_quantize_evict(k, k, torch.zeros(8, dtype=torch.bool, device=DEV))
    assert all(t.numel() == 0 for t in res)


def test_fused_mixed_precision_attention_golden(golden_dir):
    from akv.triton_ops import fused_mixed_precision_attention
    f = _fx(golden_dir)
    gs = int(f["att_gs"])
    out, w = fused_mixed_precision_attention(_d(f["att_q"]), _d(f["att_hk"]), _d(f["att_hv"]), _d(f["att_kd"]),
                                             _d(f["att_ks"]), _d(f["att_kz"]), _d(f["att_vd"]), _d(f["att_vs"]),
                                             _d(f["att_vz"]), bits=4, group_size=gs)
    assert out.shape == f["att_q"].shape and out.dtype == torch.float16
    assert np.abs(out.float().cpu().numpy() - f["att_out"]).max() <= ATOL
    np.testing.assert_allclose(w.cpu().numpy(), f["att_w"], atol=1e-4, rtol=0)
    np.testing.assert_allclose(w.sum(-1).cpu().numpy(), 1.0, atol=1e-4)


def _oracle_attention(q, k, v):
    """fp32 softmax attention; q (B, H, M, D), k / v (B, H, N, D)."""
    s = np.einsum("bhmd,bhnd->bhmn", q.astype(np.float32), k.astype(np.float32)) / math.sqrt(q.shape[-1])
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return np.einsum("bhmn,bhnd->bhmd", p, v.astype(np.float32))


@pytest.mark.parametrize("bits,D,gs", [(4, 128, 32), (2, 64, 32), (8, 96, 64)])
def test_fused_quantized_and_decode_attention_vs_oracle(bits, D, gs):
    from akv.group_format import group_quantize
    from akv.triton_kernels import fused_decode_attention
    from akv.triton_ops import fused_quantized_attention
    g = torch.Generator(device=DEV).manual_seed(bits * 7 + D)
    B, H, M, N, n_hot = 2, 4, 3, 150, 37
    q = torch.randn(B, H, M, D, generator=g, device=DEV).half()
    wk = torch.randn(N, D, generator=g, device=DEV).half()
    wv = torch.randn(N, D, generator=g, device=DEV).half()
    kp, ks, kz = group_quantize(wk, bits, gs)
    vp, vs, vz = group_quantize(wv, bits, gs)
    dk = O.group_dequantize(kp.cpu().numpy(), ks.cpu().numpy(), kz.cpu().numpy(), bits, gs, N, D)
    dv = O.group_dequantize(vp.cpu().numpy(), vs.cpu().numpy(), vz.cpu().numpy(), bits, gs, N, D)
    out = fused_quantized_attention(q, kp, ks, kz, vp, vs, vz, bits=bits, group_size=gs)
    ref = _oracle_attention(q.cpu().numpy(), np.broadcast_to(dk, (B, H, N, D)), np.broadcast_to(dv, (B, H, N, D)))
    assert np.abs(out.float().cpu().numpy() - ref).max() <= ATOL
    # decode: one query over [hot; warm]
    hk = torch.randn(B, H, n_hot, D, generator=g, device=DEV).half()
    hv = torch.randn(B, H, n_hot, D, generator=g, device=DEV).half()
    q1 = q[:, :, :1]
    out1 = fused_decode_attention(q1, hk, hv, kp, ks, kz, vp, vs, vz, bits=bits, group_size=gs)
    keys = np.concatenate([hk.cpu().numpy(), np.broadcast_to(dk, (B, H, N, D))], 2)
    vals = np.concatenate([hv.cpu().numpy(), np.broadcast_to(dv, (B, H, N, D))], 2)
    ref1 = _oracle_attention(q1.cpu().numpy(), keys, vals)
    assert np.abs(out1.float().cpu().numpy() - ref1).max() <= ATOL
    # hot only
    out2 = fused_decode_attention(q1, hk, hv)
    ref2 = _oracle_attention(q1.cpu().numpy(), hk.cpu().numpy(), hv.cpu().numpy())
    assert np.abs(out2.float().cpu().numpy() - ref2).max() <= ATOL


def test_fused_attention_compat_wrappers():
    """fused_attention.fused_decode_attention over a QuantizedTensor-shaped
    object (dequantised by the CUDA kernel) and fused_quantize_evict handing
    the masked tokens to the caller's quantiser."""
    from akv import fused_attention as FA
    from akv.group_format import group_quantize
    g = torch.Generator(device=DEV).manual_seed(3)
    B, H, N, D, gs = 2, 3, 90, 128, 32
    k = torch.randn(B, H, N, D, generator=g, device=DEV).half()
    v = torch.randn(B, H, N, D, generator=g, device=DEV).half()
    q = torch.randn(B, H, 1, D, generator=g, device=DEV).half()

    def qt(x):
        p, s, z = group_quantize(x.reshape(-1, D), 4, gs)
        return types.SimpleNamespace(data=p, scales=s, zeros=z, shape=tuple(x.shape), bits=4, group_size=gs)

    class Quantizer:
        def __init__(self):
            self.seen = []

        def quantize(self, x):
            self.seen.append(x)
            return qt(x)

        def dequantize(self, t):  # not reached: the group format dequantises on CUDA
            raise AssertionError

    kq, vq = qt(k), qt(v)
    out = FA.fused_decode_attention(q, kq, vq, Quantizer())
    dk = O.group_dequantize(kq.data.cpu().numpy(), kq.scales.cpu().numpy(), kq.zeros.cpu().numpy(), 4, gs,
                            B * H * N, D).reshape(B, H, N, D)
    dv = O.group_dequantize(vq.data.cpu().numpy(), vq.scales.cpu().numpy(), vq.zeros.cpu().numpy(), 4, gs,
                            B * H * N, D).reshape(B, H, N, D)
    ref = _oracle_attention(q.cpu().numpy(), dk, dv)
    assert np.abs(out.float().cpu().numpy() - ref).max() <= ATOL
    qz = Quantizer()
    mask = torch.rand(N, generator=g, device=DEV) < 0.3
    rk, rv = FA.fused_quantize_evict(k, v, None, mask, qz)
    idx = mask.nonzero(as_tuple=True)[0]
    torch.testing.assert_close(qz.seen[0], k[:, :, idx], rtol=0, atol=0)
    torch.testing.assert_close(qz.seen[1], v[:, :, idx], rtol=0, atol=0)
    assert FA.fused_quantize_evict(k, v, None, torch.zeros_like(mask), qz) == (None, None)


def test_importance_alias():
    import akv.triton_ops as T
    from akv import tiering
    assert T.fused_importance_update is tiering.fused_importance_update and T.HAS_TRITON


def test_scatter_rows():
    from akv import tiering
    g = torch.Generator(device=DEV).manual_seed(5)
    src = torch.randn(2, 3, 40, 128, generator=g, device=DEV).half()
    dst = torch.randn(2, 3, 60, 128, generator=g, device=DEV).half()
    ref = dst.clone()
    di = torch.tensor([5, 59, 0, 17], device=DEV)
    si = torch.tensor([39, 2, 11, 0], device=DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    tiering.scatter_rows(src, dst, di, si, status=st)
    ref[:, :, di] = src[:, :, si]
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    torch.testing.assert_close(dst, ref, rtol=0, atol=0)
    # identity source order, and a move inside one buffer (disjoint rows)
    tiering.scatter_rows(src[:, :, :4], dst, di)
    ref[:, :, di] = src[:, :, :4]
    buf = src.clone()
    tiering.scatter_rows(buf, buf, torch.tensor([1, 2], device=DEV), torch.tensor([30, 31], device=DEV))
    exp = src.clone()
    exp[:, :, [1, 2]] = src[:, :, [30, 31]]
    torch.cuda.synchronize()
    torch.testing.assert_close(dst, ref, rtol=0, atol=0)
    torch.testing.assert_close(buf, exp, rtol=0, atol=0)


@pytest.mark.parametrize("which", ["src", "dst"])
def test_scatter_rows_out_of_range_sets_status(which):
    """An index past either tier's rows is flagged and redirected to row 0 by the kernel's own check."""
    from akv import tiering
    src = torch.randn(1, 2, 10, 64, device=DEV).half()
    dst = torch.zeros(1, 2, 12, 64, device=DEV).half()
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    di = torch.tensor([3, 12 if which == "dst" else 4], device=DEV)
    si = torch.tensor([1, 10 if which == "src" else 2], device=DEV)
    tiering.scatter_rows(src, dst, di, si, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == -1
    torch.testing.assert_close(dst[:, :, 3], src[:, :, 1], rtol=0, atol=0)
