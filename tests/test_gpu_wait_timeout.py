"""GPU: a bounded device-side wait that runs out reports AKV_ERR_TIMEOUT and
leaves the context usable.

``akv_selftest_wait`` runs the mbarrier wait every kernel of the library uses
(``mbar_wait`` in csrc/common.cuh) with its limit shortened to 50 ms, on a
barrier phase that nothing completes (no fault, no trap: the wait gives up,
records the status and the kernel returns).  The same entry with an arrival
completes normally, and a decode launch afterwards still gives the right
answer.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
AKV_ERR_TIMEOUT = -6


def _run(arrive, limit_ns):
    from akv import _C
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    res = torch.zeros(1, dtype=torch.int32, device=DEV)
    _C.check(_C.load().akv_selftest_wait(arrive, limit_ns, st.data_ptr(), res.data_ptr(), _C.stream_of(st)),
             "akv_selftest_wait")
    torch.cuda.synchronize()
    return int(st.item()), int(res.item())


def test_wait_runs_out_and_reports_timeout():
    import time
    # completed phase: no status, result 1 (this first call also loads the
    # library and its kernels, which the timing below must not include)
    assert _run(1, 50_000_000) == (0, 1)
    t0 = time.perf_counter()
    st, res = _run(0, 50_000_000)
    dt = time.perf_counter() - t0
    assert st == AKV_ERR_TIMEOUT and res == 2
    assert dt < 1.5, dt  # gave up near its 50 ms limit, not at the kernels' 2 s


def test_context_usable_after_timeout():
    import akv
    from oracle import akv_oracle as O
    assert _run(0, 10_000_000)[0] == AKV_ERR_TIMEOUT
    g = torch.Generator(device=DEV).manual_seed(0)
    q = torch.randn(1, 4, 128, generator=g, device=DEV).half()
    k = torch.randn(1, 2, 77, 128, generator=g, device=DEV).half()
    v = torch.randn(1, 2, 77, 128, generator=g, device=DEV).half()
    out = akv.mixed_tier_decode_attention(q, k, v)
    ref = O.decode_attention(q.cpu().numpy(), k.cpu().numpy(), v.cpu().numpy())
    assert np.abs(out.float().cpu().numpy() - ref).max() <= 2e-3


def test_selftest_limit_checked_on_host():
    from akv import _C
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    rc = _C.load().akv_selftest_wait(0, 3_000_000_000, st.data_ptr(), st.data_ptr(), None)
    assert rc == -1  # AKV_ERR_SHAPE: longer than the kernels' own limit, nothing launched


def test_peer_combine_times_out_when_no_rank_published():
    """The sequence split's cross-GPU merge waits on flags that other GPUs'
    publishes raise.  With a fresh exchange buffer on one GPU (every flag 0)
    and epoch 1, nothing ever raises them: each CTA's wait gives up after the
    kernels' 2 s limit, the status word reads AKV_ERR_TIMEOUT, the output is
    zero and the lse -inf, and the context stays usable."""
    import ctypes
    import time
    from akv import _C
    lib = _C.load()
    rows, D, world = 4, 128, 2
    nbytes = 4 * (2 * world * rows * (D + 2)) + 4 * world + 8
    p = ctypes.c_void_p()
    _C.check(lib.akv_peer_alloc(nbytes, ctypes.byref(p)), "akv_peer_alloc")
    try:
        gather = p.value
        flags = gather + 4 * (2 * world * rows * (D + 2))
        out = torch.full((rows, D), 7.0, dtype=torch.float16, device=DEV)
        lse = torch.zeros(rows, dtype=torch.float32, device=DEV)
        st = torch.zeros(1, dtype=torch.int32, device=DEV)
        t0 = time.perf_counter()
        _C.check(lib.akv_peer_combine(gather, flags, rows, D, world, 1, out.data_ptr(), out.stride(0),
                                      lse.data_ptr(), st.data_ptr(), _C.stream_of(out)), "akv_peer_combine")
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        assert int(st.item()) == AKV_ERR_TIMEOUT
        assert torch.all(out == 0) and torch.all(torch.isinf(lse))
        assert 1.5 < dt < 10.0, dt
    finally:
        torch.cuda.synchronize()
        lib.akv_peer_free(p.value)
    x = torch.ones(1024, device=DEV)
    assert float((x * 2).sum().item()) == 2048.0  # the context still runs work
