"""The zero-allocation decode entry point, akv_mixed_decode_noalloc, called
through the C ABI.

Callers that cannot allocate device memory on their decode path (an attention
hook inside another serving engine that is handed only tensors and a stream)
use this entry: its split partials live in a fixed 8 MiB device array inside
the library.  The test checks, on two calls in a row with different shapes,
that it returns bit for bit what the workspace-taking akv_mixed_decode returns
(fp16 output, natural-log LSE and the merged partial record): both run the
same planner and kernels on the same inputs, so any difference would be a
scratch-reuse bug.  It also checks that a shape needing more scratch than the
array holds is refused before any launch.
"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


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


def _decode(q, hk, hv, arena, workspace=None):
    """One decode call through the C ABI: akv_mixed_decode with the given
    workspace, or akv_mixed_decode_noalloc when workspace is None.  Returns
    (out fp16, lse fp32, partial fp32) after checking the status word."""
    from akv import _C
    lib = _C.load()
    B, Hq, D = q.shape
    out = torch.full((B, Hq, D), float("nan"), dtype=torch.float16, device=DEV)
    lse = torch.full((B * Hq,), float("nan"), dtype=torch.float32, device=DEV)
    part = torch.full((B * Hq, D + 2), float("nan"), dtype=torch.float32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    args = (q.data_ptr(), q.stride(0), q.stride(1),
            hk.data_ptr(), hv.data_ptr(), hk.stride(0), hk.stride(1), hk.stride(2), hk.shape[2], None,
            arena.buf.data_ptr(), arena.buf.stride(0), arena.buf.stride(1), ctypes.byref(arena.layout),
            arena.n_blocks, None, B, Hq, hk.shape[1], D, 1.0 / np.sqrt(D),
            out.data_ptr(), out.stride(0), out.stride(1), lse.data_ptr(), part.data_ptr())
    stream = torch.cuda.current_stream().cuda_stream
    if workspace is None:
        rc = lib.akv_mixed_decode_noalloc(*args, status.data_ptr(), stream)
    else:
        rc = lib.akv_mixed_decode(*args, workspace.data_ptr(), workspace.numel(), status.data_ptr(), stream)
    _C.check(rc, "decode")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return out, lse, part


def _bits(t):
    return t.cpu().numpy().view(np.uint16 if t.dtype == torch.float16 else np.uint32)


def test_noalloc_matches_workspace_entry_two_calls():
    from akv import _C
    lib = _C.load()
    cases = [(7, 2, 16, 4, 32 * 5 + 9, 70, 4, 2, 0.01),   # config-3 shape family
             (8, 1, 12, 2, 32 * 112, 512, 3, 3, 0.0)]     # config 1
    for args in cases:
        q, hk, hv, arena = _case(*args)
        B, Hq, D = q.shape
        need = lib.akv_decode_workspace_bytes(B, Hq, hk.shape[1], D, hk.shape[2], arena.n_blocks)
        ws = torch.empty(need, dtype=torch.uint8, device=DEV)
        ref = _decode(q, hk, hv, arena, workspace=ws)
        got = _decode(q, hk, hv, arena)
        for r, x in zip(ref, got):
            np.testing.assert_array_equal(_bits(x), _bits(r))
        assert torch.isfinite(got[0].float()).all()


def test_noalloc_rejects_oversized_request():
    from akv import _C
    lib = _C.load()
    B, Hq, Hkv, n_hot, nwb = 64, 64, 8, 4096, 2048
    assert lib.akv_decode_workspace_bytes(B, Hq, Hkv, 128, n_hot, nwb) > (8 << 20)
    rc = lib.akv_mixed_decode_noalloc(None, 0, 0, None, None, 0, 0, 0, n_hot, None, None, 0, 0, None, nwb, None,
                                      B, Hq, Hkv, 128, 1.0, None, 0, 0, None, None, None, None)
    assert rc == -8  # AKV_ERR_WORKSPACE: more scratch than the fixed array holds; nothing launched
