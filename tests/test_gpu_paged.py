"""GPU: paged warm pool, block-table decode, and the vLLM-style engine.

* akv_mixed_decode_paged over shuffled pages is bit-identical to
  akv_mixed_decode over the same records stored contiguously (same plan,
  same bytes), for ragged rows;
* paged decode over pages written by PagedWarmPool.write matches the oracle
  (reference quantiser per 32-token block, fp32 attention) within 2e-3;
* a block-table entry outside the pool records AKV_ERR_SHAPE (the kernel
  reads page 0 instead; no out-of-bounds access);
* AdaptiveCacheEngine / AdaptiveAttentionBackend (reference
  akv/vllm_integration.py:96-343): batched decode over sequences with
  different lengths, slot reuse after free, token bookkeeping of the tiers.
"""
import numpy as np
import pytest
import torch

from oracle import akv_oracle as O

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _tol(ref):
    ref = np.asarray(ref, np.float32)
    ulp = np.spacing(np.abs(ref).astype(np.float16)).astype(np.float32)
    return np.maximum(2e-3, 0.5 * ulp + 1e-3)


def _kv(g, shape, outlier=(3,)):
    x = torch.randn(shape, generator=g, device=DEV)
    for c in outlier:
        x[..., c] *= 12
    return x.half()


def test_paged_matches_contiguous_bit_exact():
    import akv
    from akv.paged import PagedWarmPool, paged_decode_attention
    g = torch.Generator(device=DEV).manual_seed(0)
    B, Hq, Hkv, D, nblk = 3, 8, 2, 128, 7
    wk, wv = _kv(g, (B, Hkv, 32 * nblk, D)), _kv(g, (B, Hkv, 32 * nblk, D))
    arena = akv.WarmArena(B, Hkv, D, 4, 2, 0.01, max_blocks=nblk, device=DEV)
    arena.append(wk, wv, group=32)
    warm_blocks = [5, 2, 7]
    hot_len = [40, 0, 17]
    hk, hv = _kv(g, (B, Hkv, 40, D)), _kv(g, (B, Hkv, 40, D))
    q = torch.randn(B, Hq, D, generator=g, device=DEV).half()
    pool = PagedWarmPool(64, Hkv, D, 4, 2, 0.01, device=DEV)
    assert pool.rec == arena.rec
    perm = torch.randperm(64, generator=torch.Generator().manual_seed(1)).tolist()
    table = torch.zeros(B, nblk, dtype=torch.int32)
    k = 0
    for b in range(B):
        for j in range(warm_blocks[b]):
            pool.buf[perm[k]] = arena.buf[b, :, j]
            table[b, j] = perm[k]
            k += 1
    wl = torch.tensor(warm_blocks, dtype=torch.int32, device=DEV)
    hl = torch.tensor(hot_len, dtype=torch.int32, device=DEV)
    ref = akv.mixed_tier_decode_attention(q, hk, hv, arena, hot_len=hl, warm_len=wl)
    got = paged_decode_attention(q, hk, hv, hl, pool, table.to(DEV), wl)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int16), ref.view(torch.int16))


@pytest.mark.parametrize("kb,vb,frac", [(4, 2, 0.01), (3, 3, 0.0), (2, 4, 0.0)])
def test_paged_write_and_decode_vs_oracle(kb, vb, frac):
    from akv.paged import PagedWarmPool, paged_decode_attention
    g = torch.Generator(device=DEV).manual_seed(kb * 10 + vb)
    Hq, Hkv, D = 8, 2, 128
    lens = [32 * 4 + 9, 32 * 2, 17]      # warm tokens per sequence
    hot = [24, 5, 0]
    pool = PagedWarmPool(40, Hkv, D, kb, vb, frac, device=DEV)
    junk = pool.alloc(3)                  # interleave: later allocations are not one run
    pages, ks, vs = [], [], []
    for b, n in enumerate(lens):
        nb = (n + 31) // 32
        if b == 0:
            pg = pool.alloc(2) + [junk[1]] + pool.alloc(nb - 3)  # deliberately not ascending
        else:
            pg = pool.alloc(nb)
        k, v = _kv(g, (1, Hkv, n, D)), _kv(g, (1, Hkv, n, D))
        pool.write(k, v, pg)
        pages.append(pg)
        ks.append(k)
        vs.append(v)
    B = len(lens)
    maxb = max(len(p) for p in pages)
    table = torch.zeros(B, maxb, dtype=torch.int32)
    for b, pg in enumerate(pages):
        table[b, :len(pg)] = torch.tensor(pg, dtype=torch.int32)
    hk, hv = _kv(g, (B, Hkv, 24, D)), _kv(g, (B, Hkv, 24, D))
    q = torch.randn(B, Hq, D, generator=g, device=DEV).half()
    out = paged_decode_attention(q, hk, hv, torch.tensor(hot, dtype=torch.int32, device=DEV), pool,
                                 table.to(DEV), torch.tensor([len(p) for p in pages], dtype=torch.int32, device=DEV))
    out = out.float().cpu().numpy()
    for b in range(B):
        k, v = ks[b].cpu().numpy(), vs[b].cpu().numpy()
        dk = O.dequantize_groups(O.quantize_groups(k, kb, 32, True, frac))
        dv = O.dequantize_groups(O.quantize_groups(v, vb, 32, False, frac))
        K = np.concatenate([dk, hk[b:b + 1, :, :hot[b]].cpu().numpy()], 2)
        V = np.concatenate([dv, hv[b:b + 1, :, :hot[b]].cpu().numpy()], 2)
        ref = O.decode_attention(q[b:b + 1].cpu().numpy(), K, V)[0]
        assert (np.abs(out[b] - ref) <= _tol(ref)).all(), np.abs(out[b] - ref).max()
        # the pool's dequantised blocks are the oracle's, bit for bit
        pk, pv = pool.dequantize(pages[b], n_tokens=lens[b])
        np.testing.assert_array_equal(pk.cpu().numpy().view(np.uint16), dk.view(np.uint16))
        np.testing.assert_array_equal(pv.cpu().numpy().view(np.uint16), dv.view(np.uint16))


def test_out_of_range_page_sets_status():
    from akv.paged import PagedWarmPool, paged_decode_attention
    g = torch.Generator(device=DEV).manual_seed(5)
    pool = PagedWarmPool(8, 2, 128, 4, 4, device=DEV)
    pg = pool.alloc(2)
    pool.write(_kv(g, (1, 2, 64, 128)), _kv(g, (1, 2, 64, 128)), pg)
    table = torch.tensor([[pg[0], 8 + 5]], dtype=torch.int32, device=DEV)  # second entry beyond the pool
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    q = torch.randn(1, 4, 128, generator=g, device=DEV).half()
    out = paged_decode_attention(q, None, None, None, pool, table, torch.tensor([2], dtype=torch.int32, device=DEV),
                                 status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == -1  # AKV_ERR_SHAPE
    assert torch.isfinite(out.float()).all()


def _engine(max_seqs=4, layers=2, **kw):
    from akv.vllm_integration import AdaptiveCacheEngine, AdaptiveVLLMConfig
    cfg = AdaptiveVLLMConfig(hot_budget_per_seq=128, warm_budget_per_seq=2048, warm_bits=4, max_seqs=max_seqs,
                             eviction_batch_size=64, recent_tokens_protected=32, **kw)
    return AdaptiveCacheEngine(cfg, num_layers=layers, num_heads=2, head_dim=128, device=DEV)


def _check_batch(eng, backend, seq_ids, layer, g, Hq=8):
    q = torch.randn(len(seq_ids), Hq, 128, generator=g, device=DEV).half()
    out = backend.forward_batch(q, seq_ids, layer).float()
    for i, s in enumerate(seq_ids):
        k, v = eng.get_kv_for_attention(s, layer)
        K = k.float().repeat_interleave(Hq // 2, 1)[0]
        V = v.float().repeat_interleave(Hq // 2, 1)[0]
        p = torch.softmax(torch.einsum("hd,hnd->hn", q[i].float(), K) / 128 ** 0.5, -1)
        ref = torch.einsum("hn,hnd->hd", p, V).cpu().numpy()
        got = out[i].cpu().numpy()
        assert (np.abs(got - ref) <= _tol(ref)).all(), (s, np.abs(got - ref).max())


def test_engine_batched_decode_and_slot_reuse():
    from akv.vllm_integration import AdaptiveAttentionBackend
    eng = _engine()
    backend = AdaptiveAttentionBackend(eng)
    g = torch.Generator(device=DEV).manual_seed(7)
    feeds = {}
    for s, n in ((10, 300), (11, 70), (12, 1000)):
        eng.allocate(s)
        for layer in range(2):
            k, v = _kv(g, (1, 2, n, 128)), _kv(g, (1, 2, n, 128))
            eng.update(s, k, v, layer)
            feeds[(s, layer)] = [k]
    for _ in range(150):  # two or three demotions per sequence with the rows out of token order
        for s in (10, 11, 12):
            for layer in range(2):
                k, v = _kv(g, (1, 2, 1, 128)), _kv(g, (1, 2, 1, 128))
                eng.update(s, k, v, layer)
                feeds[(s, layer)].append(k)
    for layer in range(2):
        _check_batch(eng, backend, [10, 11, 12], layer, g)
    # token bookkeeping: every fed token is present once, in order; hot tokens exact
    for (s, layer), ks in feeds.items():
        fed = torch.cat(ks, 2)
        k, _ = eng.get_kv_for_attention(s, layer)
        assert k.shape == fed.shape
        slot = eng.get_cache(s)
        hl = eng._layers[layer].hot_len[slot]
        assert hl <= 128
        assert torch.equal(k[:, :, -(hl - 4):], fed[:, :, -(hl - 4):])  # the hot window after the protected 4
        assert torch.equal(k[:, :, :4], fed[:, :, :4])
        assert (k.float() - fed.float()).abs().max().item() < 12 * 12 / 15 + 1e-2  # warm: within a 4-bit step
    mu = eng.memory_usage()
    assert mu["active_sequences"] == 3 and mu["total_warm_mb"] > 0 and mu["total_migrations"] > 0
    # free one sequence; a new one reuses its slot and pages
    free_before = eng._layers[0].pool.free_pages
    slot12 = eng.get_cache(12)
    used = len(eng._layers[0].pages[slot12])
    assert used > 0
    eng.free(12)
    assert eng._layers[0].pool.free_pages == free_before + used
    eng.allocate(20)
    assert eng.get_cache(20) == slot12
    for layer in range(2):
        eng.update(20, _kv(g, (1, 2, 500, 128)), _kv(g, (1, 2, 500, 128)), layer)
    for layer in range(2):
        _check_batch(eng, backend, [10, 11, 20], layer, g)
        _check_batch(eng, backend, [20, 10], layer, g)  # rows out of slot order
    # the reference's single-sequence signature, one query and several
    q1 = torch.randn(1, 8, 1, 128, generator=g, device=DEV).half()
    assert backend.forward(q1, 20, 0).shape == (1, 8, 1, 128)
    q4 = torch.randn(1, 8, 4, 128, generator=g, device=DEV).half()
    o4 = backend.forward(q4, 20, 1)
    assert o4.shape == (1, 8, 4, 128)
    k, v = eng.get_kv_for_attention(20, 1)  # M > 1: every query over every key, no mask
    K, V = k.float().repeat_interleave(4, 1), v.float().repeat_interleave(4, 1)
    ref = torch.softmax(q4.float() @ K.transpose(-2, -1) / 128 ** 0.5, -1) @ V
    assert (o4.float() - ref).abs().max().item() <= 2e-3
    with pytest.raises(ValueError):
        backend.forward(q1, 99, 0)
