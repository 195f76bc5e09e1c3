"""The zero-allocation decode entry point, akv_mixed_decode_noalloc, called
through the C ABI.

Callers that cannot allocate device memory on their decode path (an attention
hook inside another serving engine that is handed only tensors and a stream)
use this entry: its split partials live in a fixed 8 MiB device array inside
the library.  The test checks, on two calls in a row with different shapes,
that it returns what the workspace-taking akv_mixed_decode returns, and that a
shape needing more scratch than the array is refused before any launch.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
ATOL = 2e-3


def _case(seed, B, Hq, Hkv, n_warm, n_hot, kb, vb, frac):
    import akv
    g = torch.Generator(device=DEV).manual_seed(seed)
    D = 128
    wk = torch.randn(B, Hkv, n_warm, D, generator=g, device=DEV).half()
    wv = torch.randn(B, Hkv, n_warm, D, generator=g, device=DEV).half()
    hk = torch.randn(B, Hkv, n_hot, D, generator=g, device=DEV).half()
    hv = torch.randn(B, Hkv, n_hot, D, generator=g, device=DEV).half()
    q = torch.randn(B, Hq, D, generator=g, device=DEV).half()
    arena = akv.WarmArena(B, Hkv, D, kb, vb, outlier_fraction=frac, max_blocks=(n_warm + 31) // 32, device=DEV)
    arena.append(wk, wv, group=32)
    return q, hk, hv, arena


def _noalloc(q, hk, hv, arena):
    from akv import _C
    lib = _C.load()
    B, Hq, D = q.shape
    out = torch.full((B, Hq, D), float("nan"), dtype=torch.float16, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = lib.akv_mixed_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1),
        hk.data_ptr(), hv.data_ptr(), hk.stride(0), hk.stride(1), hk.stride(2), hk.shape[2], None,
        arena.buf.data_ptr(), arena.buf.stride(0), arena.buf.stride(1), ctypes.byref(arena.layout),
        arena.n_blocks, None, B, Hq, hk.shape[1], D, 1.0 / np.sqrt(D),
        out.data_ptr(), out.stride(0), out.stride(1), None, None, status.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    _C.check(rc, "akv_mixed_decode_noalloc")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out


def test_noalloc_matches_workspace_entry_two_calls():
    import akv
    cases = [(7, 2, 16, 4, 32 * 5 + 9, 70, 4, 2, 0.01),   # config-3 shape family
             (8, 1, 12, 2, 32 * 112, 512, 3, 3, 0.0)]     # config 1
    for args in cases:
        q, hk, hv, arena = _case(*args)
        ref = akv.mixed_tier_decode_attention(q, hk, hv, arena)
        got = _noalloc(q, hk, hv, arena)
        err = (got.float() - ref.float()).abs().max().item()
        assert err <= ATOL, f"no-alloc entry differs from akv_mixed_decode by {err}"


def test_noalloc_rejects_oversized_request():
    from akv import _C
    lib = _C.load()
    B, Hq, Hkv, n_hot, nwb = 64, 64, 8, 4096, 2048
    assert lib.akv_decode_workspace_bytes(B, Hq, Hkv, 128, n_hot, nwb) > (8 << 20)
    rc = lib.akv_mixed_decode_noalloc(None, 0, 0, None, None, 0, 0, 0, n_hot, None, None, 0, 0, None, nwb, None,
                                      B, Hq, Hkv, 128, 1.0, None, 0, 0, None, None, None, None)
    assert rc == -8  # AKV_ERR_WORKSPACE: more scratch than the fixed array holds; nothing launched
