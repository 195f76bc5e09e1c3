"""CPU: the torch restatement of the reference's decode recipe that bench.py
times as the CPU arm agrees with the golden-pinned numpy oracle (dequantised
warm tier bit for bit, attention to fp32 rounding)."""
import numpy as np
import pytest
import torch

from oracle import akv_oracle as O
from oracle import akv_torch_ref as R


@pytest.mark.parametrize("kb,vb,frac", [(4, 2, 0.01), (3, 3, 0.0), (2, 4, 0.05)])
def test_torch_reference_path_matches_oracle(kb, vb, frac):
    n_warm, n_hot, D, g = 32 * 12, 48, 128, 4
    wk, wv, hk, hv, q = R.unit_inputs(3, n_warm, n_hot, D, g, kb, vb, frac)
    rng = np.random.default_rng(3)  # the same draws unit_inputs made
    k = rng.standard_normal((1, 1, n_warm, D)).astype(np.float16)
    v = rng.standard_normal((1, 1, n_warm, D)).astype(np.float16)
    dk = O.dequantize_groups(O.quantize_groups(k, kb, 32, True, frac))
    dv = O.dequantize_groups(O.quantize_groups(v, vb, 32, False, frac))
    np.testing.assert_array_equal(R.dequantize(wk).numpy().view(np.uint16), dk[0, 0].view(np.uint16))
    np.testing.assert_array_equal(R.dequantize(wv).numpy().view(np.uint16), dv[0, 0].view(np.uint16))
    out = R.decode_unit(wk, wv, hk, hv, q).numpy()
    ref = O.decode_attention(q.numpy()[None], np.concatenate([dk, hk.numpy()[None, None]], 2),
                             np.concatenate([dv, hv.numpy()[None, None]], 2))[0]
    np.testing.assert_allclose(out, ref, rtol=0, atol=1e-5)


def test_unpack_layouts():
    rng = np.random.default_rng(0)
    for bits in (2, 3, 4):
        c = rng.integers(0, 1 << bits, (5, 128)).astype(np.uint8)
        p = O.pack(c, bits)
        np.testing.assert_array_equal(R.unpack(torch.from_numpy(p), bits, 128).numpy(), c)
