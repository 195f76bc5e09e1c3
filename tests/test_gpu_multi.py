"""akv.parallel over real NCCL collectives: two processes, one GPU each.
Skipped unless at least two GPUs are visible.

Rank r holds KV heads [4r, 4r+4) of an 8-head layer (head-sharded
quantisation with the outlier-score all-reduce) and the r-th contiguous half
of a sequence's warm blocks (sequence-split decode with the all-gather + LSE
combine).  Each rank checks its results against a single-GPU computation of
the whole problem.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, errfile):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import akv
        from akv import parallel as P
        rng = np.random.default_rng(0)
        B, H, N, D = 2, 8, 64, 128
        k = torch.from_numpy(rng.standard_normal((B, H, N, D)).astype(np.float16)).to(dev)
        k[..., 40] *= 12
        v = torch.from_numpy(rng.standard_normal((B, H, N, D)).astype(np.float16)).to(dev)
        full = akv.WarmArena(B, H, D, 4, 2, 0.01, max_blocks=2, device=dev)
        full.append(k, v, group=32)
        mine = akv.WarmArena(B, 4, D, 4, 2, 0.01, max_blocks=2, device=dev)
        P.quantize_head_sharded(mine, k[:, 4 * rank:4 * rank + 4].contiguous(),
                                v[:, 4 * rank:4 * rank + 4].contiguous(), total_heads=H, group=32)
        assert torch.equal(mine.buf, full.buf[:, 4 * rank:4 * rank + 4]), "head-sharded records differ"

        Hq, Hkv, nblk, nh = 16, 4, 24, 50
        wk = torch.from_numpy(rng.standard_normal((1, Hkv, 32 * nblk, D)).astype(np.float16)).to(dev)
        wv = torch.from_numpy(rng.standard_normal((1, Hkv, 32 * nblk, D)).astype(np.float16)).to(dev)
        hk = torch.from_numpy(rng.standard_normal((1, Hkv, nh, D)).astype(np.float16)).to(dev)
        hv = torch.from_numpy(rng.standard_normal((1, Hkv, nh, D)).astype(np.float16)).to(dev)
        q = torch.from_numpy(rng.standard_normal((1, Hq, D)).astype(np.float16)).to(dev)
        whole = akv.WarmArena(1, Hkv, D, 4, 2, 0.01, max_blocks=nblk, device=dev)
        whole.append(wk, wv, group=32)
        ref = akv.mixed_tier_decode_attention(q, hk, hv, whole)
        lo, hi = P.ShardPlan("sequence", world, rank).span(nblk)
        part = akv.WarmArena(1, Hkv, D, 4, 2, 0.01, max_blocks=hi - lo, device=dev)
        part.append(wk[:, :, 32 * lo:32 * hi], wv[:, :, 32 * lo:32 * hi], group=32)
        out = P.sequence_split_decode(q, hk if rank == 0 else None, hv if rank == 0 else None, part, world)
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= 2e-3, f"sequence split err {err}"
        torch.cuda.synchronize()
        dist.barrier()
        # the same split with the cross-GPU step over NVLink peer memory, five
        # steps (both gather halves, several epochs), new queries each step
        ex = P.PeerExchange(Hq, D, device=dev)
        try:
            st = torch.zeros(1, dtype=torch.int32, device=dev)
            for step in range(5):
                qs = torch.from_numpy(np.random.default_rng(50 + step).standard_normal((1, Hq, D))
                                      .astype(np.float16)).to(dev)
                if step % 2:
                    out_p = P.sequence_split_decode(qs, hk if rank == 0 else None, hv if rank == 0 else None, part,
                                                    world, exchange=ex)
                else:
                    p = P.local_partial(qs, hk if rank == 0 else None, hv if rank == 0 else None, part)
                    out_p = ex.exchange(p, status=st).reshape(qs.shape)
                ref_p = akv.mixed_tier_decode_attention(qs, hk, hv, whole)
                torch.cuda.synchronize()
                e = (out_p.float() - ref_p.float()).abs().max().item()
                assert e <= 2e-3, f"peer sequence split err {e} at step {step}"
            assert int(st.item()) == 0
        finally:
            ex.close()
        dist.barrier()
    except Exception as e:  # report to the parent; every rank still leaves the group
        with open(f"{errfile}.{rank}", "w") as f:
            f.write(repr(e))
    finally:
        dist.destroy_process_group()


def test_two_gpu_head_shard_and_sequence_split(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    errfile = str(tmp_path / "err")
    mp.spawn(_worker, args=(2, _free_port(), errfile), nprocs=2, join=True)
    errs = [open(f"{errfile}.{r}").read() for r in range(2) if os.path.exists(f"{errfile}.{r}")]
    assert not errs, errs
