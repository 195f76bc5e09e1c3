"""Multi-GPU orchestration of akv.parallel driven by two CPU ``gloo`` ranks.

The collectives are real (torch.distributed over gloo on 127.0.0.1); the
compute steps that are CUDA kernels in the product (norm sums, quantiser,
decode partials, LSE combine) are injected from the oracle, so these tests
check the partitioning, the collective pattern and the merge, not the
kernels (tests/test_gpu_parallel.py runs those).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle.akv_oracle as O


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, world=2):
    port = _free_port()
    mp.spawn(_entry, args=(world, port, fn), nprocs=world, join=True)


def _entry(rank, world, port, fn):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fn(rank, world)
    finally:
        dist.destroy_process_group()


def test_plan_modes_and_spans():
    from akv import parallel as P
    assert P.plan(16, 8, 1, 0).mode == "single"
    assert P.plan(16, 8, 8, 3).mode == "batch"
    assert P.plan(1, 8, 8, 3).mode == "head"
    assert P.plan(1, 8, 8, 3, prefer="head").mode == "head"
    assert P.plan(3, 2, 4, 0).mode == "sequence"
    spans = [P.ShardPlan("sequence", 3, r).span(10) for r in range(3)]
    assert spans == [(0, 4), (4, 7), (7, 10)]


class _OracleArena:
    """Stands in for WarmArena: quantises with the oracle, honouring external scores."""

    def __init__(self, bits, frac):
        self.bits, self.frac = bits, frac
        self.n_out = max(1, int(128 * frac)) if frac > 0 else 0
        self.out = None

    def append(self, k, v, group, tok_idx=None, status=None, score_sums=None, score_heads=0):
        res = []
        for i, (x, fn) in enumerate(((k, O.quantize_keys), (v, O.quantize_values))):
            ss = score_sums[i].numpy()[0, 0] if score_sums is not None else None
            res.append(fn(x.numpy()[0], self.bits, self.frac, score_sum=ss, score_heads=score_heads))
        self.out = res
        return 0


def _head_sharded(rank, world):
    from akv import parallel as P
    rng = np.random.default_rng(0)
    H, N, D = 8, 32, 128
    k = rng.standard_normal((1, H, N, D)).astype(np.float16)
    k[..., 77] *= 12
    v = rng.standard_normal((1, H, N, D)).astype(np.float16)
    lo, hi = P.ShardPlan("head", world, rank).span(H)
    arena = _OracleArena(4, 0.01)
    norm_sums = lambda x: torch.from_numpy(O.outlier_norm_sum(x.numpy()[0])).view(1, 1, D)  # noqa: E731
    P.quantize_head_sharded(arena, torch.from_numpy(k[:, lo:hi]), torch.from_numpy(v[:, lo:hi]), total_heads=H,
                            group=N, norm_sums=norm_sums)
    full = (O.quantize_keys(k[0], 4, 0.01), O.quantize_values(v[0], 4, 0.01))
    for got, ref in zip(arena.out, full):
        np.testing.assert_array_equal(got["outlier_idx"], ref["outlier_idx"])
        np.testing.assert_array_equal(got["codes"], ref["codes"][lo:hi])
        np.testing.assert_array_equal(got["scale"].view(np.uint16), ref["scale"][lo:hi].view(np.uint16))


def test_head_sharded_quantise_matches_unsharded_two_ranks():
    _run(_head_sharded)


def _sequence_split(rank, world):
    from akv import parallel as P
    rng = np.random.default_rng(1)
    B, Hq, Hkv, N, Nh, D = 1, 8, 2, 300, 40, 128
    q = rng.standard_normal((B, Hq, D)).astype(np.float16)
    keys = rng.standard_normal((B, Hkv, N, D)).astype(np.float16)
    vals = rng.standard_normal((B, Hkv, N, D)).astype(np.float16)
    hk = rng.standard_normal((B, Hkv, Nh, D)).astype(np.float16)
    hv = rng.standard_normal((B, Hkv, Nh, D)).astype(np.float16)
    lo, hi = P.ShardPlan("sequence", world, rank).span(N)
    mine_k, mine_v = keys[:, :, lo:hi], vals[:, :, lo:hi]
    if rank == 0:  # the hot window lives on rank 0
        mine_k = np.concatenate([mine_k, hk], 2)
        mine_v = np.concatenate([mine_v, hv], 2)

    def partial(query, hot_k, hot_v, warm, sm_scale):
        return torch.from_numpy(O.decode_partial(query.numpy(), hot_k, hot_v))

    def combine(part):
        return torch.from_numpy(O.lse_combine(part.numpy()))

    out = P.sequence_split_decode(torch.from_numpy(q), mine_k, mine_v, None, world, partial=partial, combine=combine)
    ref = O.decode_attention(q, np.concatenate([keys, hk], 2), np.concatenate([vals, hv], 2))
    np.testing.assert_allclose(out.numpy(), ref, atol=1e-5, rtol=0)


def test_sequence_split_decode_two_ranks():
    _run(_sequence_split)


def _sequence_split_empty_rank(rank, world):
    """A rank holding no tokens contributes (0, -inf, 0) and changes nothing."""
    from akv import parallel as P
    rng = np.random.default_rng(2)
    q = rng.standard_normal((2, 4, 128)).astype(np.float16)
    k = rng.standard_normal((2, 4, 50, 128)).astype(np.float16)
    v = rng.standard_normal((2, 4, 50, 128)).astype(np.float16)

    def partial(query, hot_k, hot_v, warm, sm_scale):
        if hot_k is None:
            return P._empty_partial(8, 128, "cpu")
        return torch.from_numpy(O.decode_partial(query.numpy(), hot_k, hot_v))

    def combine(part):
        return torch.from_numpy(O.lse_combine(part.numpy()))

    mine = (k, v) if rank == 1 else (None, None)
    out = P.sequence_split_decode(torch.from_numpy(q), *mine, None, world, partial=partial, combine=combine)
    np.testing.assert_allclose(out.numpy(), O.decode_attention(q, k, v), atol=1e-5, rtol=0)


def test_sequence_split_with_an_empty_rank():
    _run(_sequence_split_empty_rank)
