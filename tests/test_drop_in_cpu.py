"""AKVCache host logic that runs without a GPU.

Ported from the reference's tests/test_bit_exact.py (HF contract when no
token is demoted) and tests/test_cache_ordering.py (position bookkeeping
without demotion), plus the constructor contract of drop_in.py:910-1010.
Anything that demotes needs the CUDA kernels and lives in
tests/test_gpu_drop_in.py.
"""
import pytest
import torch

transformers = pytest.importorskip("transformers")
from transformers import DynamicCache, LlamaConfig, LlamaForCausalLM  # noqa: E402

from akv import AKVCache, recommend_preset  # noqa: E402


@pytest.fixture(scope="module")
def tiny_llama():
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=128, rms_norm_eps=1e-5)
    return cfg, LlamaForCausalLM(cfg).eval()


def _generate(model, cache, ids, n=8):
    return model.generate(ids, max_new_tokens=n, do_sample=False, past_key_values=cache, pad_token_id=0)


def test_bit_exact_with_dynamic_cache_when_no_demotion(tiny_llama):
    cfg, model = tiny_llama
    ids = torch.tensor([[1, 2, 3, 4, 5, 6, 7, 8, 9, 10]])
    with torch.no_grad():
        ref = _generate(model, DynamicCache(), ids)
        cache = AKVCache(warm_bits=4, hot_budget=4096, num_hidden_layers=cfg.num_hidden_layers,
                         enable_promotion=False)
        got = _generate(model, cache, ids)
    assert torch.equal(ref, got), (ref.tolist(), got.tolist())
    assert cache.get_seq_length() == ids.shape[1] + 8 - 1
    assert len(cache) == cfg.num_hidden_layers


def test_protected_layers_never_demote_on_cpu(tiny_llama):
    cfg, model = tiny_llama
    ids = torch.tensor([[1, 2, 3, 4, 5, 6, 7, 8, 9, 10]])
    with torch.no_grad():
        ref = _generate(model, DynamicCache(), ids)
        cache = AKVCache(warm_bits=4, hot_budget=4, num_hidden_layers=2, protect_first=1, protect_last=1)
        got = _generate(model, cache, ids)
    assert torch.equal(ref, got)
    assert all(layer._warm_keys_fp16 is None for layer in cache.layers)


def _prefill(N, hot_budget, num_layers=1, heads=2, head_dim=8):
    cache = AKVCache(warm_bits=3, hot_budget=hot_budget, enable_promotion=False, enable_promotion_proxy=False,
                     num_hidden_layers=num_layers)
    K = torch.arange(N, dtype=torch.float32).view(1, 1, N, 1).expand(1, heads, N, head_dim).contiguous().half()
    for layer_idx in range(num_layers):
        cache.update(K, K.clone(), layer_idx=layer_idx)
    return cache


def test_prefill_no_demote_keeps_positions_in_order():
    layer = _prefill(64, 256).layers[0]
    assert layer._warm_positions is None
    assert layer._hot_positions.tolist() == list(range(64))


def test_decode_step_appends_at_correct_position():
    cache = _prefill(64, 256)
    layer = cache.layers[0]
    cache.update(torch.zeros(1, 2, 1, 8, dtype=torch.float16), torch.zeros(1, 2, 1, 8, dtype=torch.float16), 0)
    assert layer._hot_positions.tolist() == list(range(65))
    cache.update(torch.zeros(1, 2, 16, 8, dtype=torch.float16), torch.zeros(1, 2, 16, 8, dtype=torch.float16), 0)
    assert layer._hot_positions.tolist() == list(range(81))


def test_demotion_needs_cuda():
    with pytest.raises(RuntimeError, match="CUDA"):
        _prefill(64, 16, head_dim=32)


def test_presets_and_argument_contract():
    c = AKVCache(preset="k4v2")
    assert (c.warm_key_bits, c.warm_value_bits, c.hot_budget) == (4, 2, 128)
    c = AKVCache(preset="compact")
    assert (c.warm_bits, c.warm_key_bits, c.warm_value_bits, c.hot_budget) == (2, 2, 2, 64)
    with pytest.raises(ValueError):
        AKVCache(preset="nope")
    with pytest.raises(ValueError):
        AKVCache(preset="quality", warm_bits=3)
    with pytest.raises(ValueError):
        AKVCache(protect_last=2)
    with pytest.raises(ValueError):
        AKVCache(protect_layers=[-1])
    c = AKVCache(num_hidden_layers=10, protect_first=2, protect_last=1, protect_layers=[5, -3])
    assert c._protected_set == {0, 1, 9, 5, 7}
    c = AKVCache(warm_bits=2, warm_value_bits=4)
    assert (c.warm_key_bits, c.warm_value_bits) == (2, 4)


def test_memory_report_and_reset():
    cache = _prefill(40, 256)
    rep = cache.memory_report()
    assert rep["seq_length"] == 40 and rep["num_layers"] == 1
    mu = cache.memory_usage()
    assert mu["hot_bytes"] == 2 * 2 * 40 * 8 * 2
    assert mu["warm_bytes_packed"] == 0 and mu["total_bytes"] == mu["hot_bytes"]
    k, v = cache[0]
    assert k.shape == (1, 2, 40, 8)
    assert len(cache.to_legacy_cache()) == 1
    cache.reset()
    assert len(cache) == 0 and cache.get_seq_length() == 0


def test_for_model_and_recommend_preset(tiny_llama):
    cfg, model = tiny_llama
    c = AKVCache.for_model(model, preset="balanced", protect_last=1)
    assert c.num_hidden_layers == 2 and c._protected_set == {1}
    rec = recommend_preset(model)
    assert rec["preset"] in ("quality", "balanced")


def test_akv_attention_registered_and_sdpa_equivalent_without_warm(tiny_llama):
    """The "akv" attention implementation: without a warm tier (nothing
    demoted) every call is SDPA over the returned K/V, so generation is
    bit-identical to attn_implementation="sdpa"."""
    import akv.hf_attention as hook
    from transformers import AttentionInterface
    assert hook.register() == "akv"
    assert AttentionInterface._global_mapping["akv"] is hook.akv_attention_forward
    cfg, model = tiny_llama
    ids = torch.tensor([[3, 1, 4, 1, 5, 9, 2, 6]])
    impl = model.config._attn_implementation
    try:
        with torch.no_grad():
            model.config._attn_implementation = "sdpa"
            ref = _generate(model, AKVCache(warm_bits=4, hot_budget=4096, enable_promotion=False), ids)
            model.config._attn_implementation = "akv"
            cache = AKVCache(warm_bits=4, hot_budget=4096, enable_promotion=False, fused_decode=True)
            got = _generate(model, cache, ids)
    finally:
        model.config._attn_implementation = impl
    assert torch.equal(ref, got)
    assert getattr(cache.layers[0].keys, "_akv_layer", None) is None  # no warm tier: the view is returned


def test_fused_placeholder_and_warm_append_on_cpu():
    """Fused-decode placeholder (NaN, zero-stride, tagged) and the in-place
    warm-copy append, with the warm tier filled by hand (demotion itself
    needs CUDA).  The tagged decode call raises on CPU: no CPU fallback."""
    import akv.hf_attention as hook
    from akv import AKVLayer
    layer = AKVLayer(warm_bits=3, hot_budget=8, enable_promotion=False, enable_promotion_proxy=False,
                     fused_decode=True)
    g = torch.Generator().manual_seed(0)
    chunks = [torch.randn(1, 2, n, 128, generator=g).half() for n in (5, 40, 3)]
    for c in chunks:
        layer._append_warm_fp16(c, -c)
    want = torch.cat(chunks, 2)
    assert torch.equal(layer._warm_keys_fp16, want) and torch.equal(layer._warm_values_fp16, -want)
    assert layer._warm_keys_fp16.data_ptr() == layer._warm_kbuf.data_ptr()
    layer._warm_keys_fp16 = layer._warm_keys_fp16[:, :, 1:].clone()  # rebuilt elsewhere (promotion)
    layer._warm_values_fp16 = layer._warm_values_fp16[:, :, 1:].clone()
    layer._append_warm_fp16(chunks[0], -chunks[0])
    assert torch.equal(layer._warm_keys_fp16, torch.cat([want[:, :, 1:], chunks[0]], 2))
    layer._hot_keys = torch.randn(1, 2, 8, 128, generator=g).half()
    layer._hot_values = layer._hot_keys.clone()
    layer._warm_len = layer._warm_keys_fp16.shape[2]
    k, v = layer._placeholder()
    assert k.shape == (1, 2, 8 + 52, 128) and k.untyped_storage().nbytes() == 2  # one fp16 element
    assert torch.isnan(k).all() and k._akv_layer is layer
    q = torch.randn(1, 4, 1, 128).half()
    with pytest.raises(RuntimeError):
        hook.akv_attention_forward(None, q, k, v, None, scaling=128 ** -0.5)


def test_vllm_engine_config_and_no_cpu_fallback():
    """AdaptiveVLLMConfig keeps the reference's fields and defaults
    (akv/vllm_integration.py:48-75); the engine refuses a CPU device."""
    from akv.vllm_integration import AdaptiveCacheEngine, AdaptiveVLLMConfig
    c = AdaptiveVLLMConfig()
    assert (c.hot_budget_per_seq, c.warm_budget_per_seq, c.cold_budget_per_seq, c.warm_bits, c.cold_bits,
            c.group_size, c.eviction_trigger_ratio, c.eviction_batch_size, c.initial_tokens_protected,
            c.recent_tokens_protected, c.importance_decay) == (1024, 4096, 8192, 4, 2, 128, 0.9, 64, 4, 32, 0.95)
    with pytest.raises(RuntimeError):
        AdaptiveCacheEngine(c, num_layers=1, num_heads=2, head_dim=128, device="cpu")


def test_from_calibration_applies_per_head_bits(tmp_path):
    """AKVCache.from_calibration (reference drop_in.py:1281-1313) on a report
    JSON: protect window, layer count, warm bits from the average, and the
    per-(layer, head) widths handed to each layer."""
    import json
    rep = {"recommended_protect_first": 1, "recommended_protect_last": 0, "num_layers": 3,
           "recommended_average_bits": 3.2, "recommended_preset": "balanced",
           "per_head_bits": {"1": [2, 4], "2": [4, 4]}}
    path = tmp_path / "calib.json"
    path.write_text(json.dumps(rep))
    cache = AKVCache.from_calibration(str(path), hot_budget=64)
    assert cache.warm_bits == 3 and cache.hot_budget == 64 and cache.num_hidden_layers == 3
    x = torch.zeros(1, 2, 4, 128, dtype=torch.float16)
    for i in range(3):
        cache.update(x, x, i)
    assert cache.layers[0].protect and cache.layers[0].per_head_bits is None
    assert cache.layers[1].per_head_bits == [2, 4] and cache.layers[2].per_head_bits == [4, 4]


def test_paged_pool_allocator_on_cpu():
    """PagedWarmPool page bookkeeping (host logic, no kernels): pages come out
    ascending from a fresh pool, exhaustion raises, released pages are reused."""
    from akv.paged import PagedWarmPool
    pool = PagedWarmPool(8, 2, 128, 4, 2, 0.01, device="cpu")
    assert pool.buf.shape == (8, 2, pool.rec) and pool.free_pages == 8
    a = pool.alloc(3)
    b = pool.alloc(2)
    assert a == [0, 1, 2] and b == [3, 4] and pool.free_pages == 3
    with pytest.raises(RuntimeError):
        pool.alloc(4)
    pool.release(a)
    assert pool.free_pages == 6
    c = pool.alloc(4)
    assert sorted(c) == [0, 1, 2, 5] and c[:3] == [0, 1, 2]  # released pages first, ascending


def test_head_group_arena_grouping_on_cpu():
    """HeadGroupArena (per-head widths, reference drop_in.py:315-374): one
    arena per distinct width over that width's heads, in head order."""
    from akv.packed_layout import HeadGroupArena
    arena = HeadGroupArena(2, [4, 2, 3, 2, 4], 128, 0.0, max_blocks=4, device="cpu")
    groups = [(bits, heads, a.H, a.key_bits, a.value_bits) for bits, heads, a in arena.groups]
    assert groups == [(2, [1, 3], 2, 2, 2), (3, [2], 1, 3, 3), (4, [0, 4], 2, 4, 4)]
    assert arena.H == 5 and arena.B == 2 and arena.n_blocks == 0
    arena.grow(9)
    assert all(a.max_blocks >= 9 for _, _, a in arena.groups) and arena.max_blocks >= 9
    assert arena.resident_bytes() == sum(a.buf.numel() for _, _, a in arena.groups)
