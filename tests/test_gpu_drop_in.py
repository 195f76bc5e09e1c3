"""AKVCache on CUDA against update traces recorded from the reference
AKVCache (tests/golden/make_golden.py: make_drop_in_traces).

After every update the warm and hot position sets must equal the
reference's (tier indices bit-exact: the same CPU topk on the same recency
scores, the same promotion by attention weights), and the final
chronological K/V view must be bit-identical (the warm part is the exact
dequantisation of packed records written by the sm_100a quantiser).  Also
ports the reference's ordering tests (tests/test_cache_ordering.py) to a
head_dim the kernels take, and runs HF generate under demotion.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _traces(golden_dir):
    z = dict(np.load(os.path.join(golden_dir, "drop_in.npz")))
    z.update(np.load(os.path.join(golden_dir, "drop_in_per_head.npz")))  # case "d"
    return z


CASES = {
    "a": dict(warm_bits=3, hot_budget=64, enable_promotion=False, enable_promotion_proxy=False),
    "b": dict(preset="k4v2", outlier_fraction=0.01, enable_promotion=True, enable_promotion_proxy=False,
              promotion_threshold=0.3),
    "c": dict(warm_bits=2, hot_budget=32, adaptive_hot_frac=0.25, enable_promotion=False,
              enable_promotion_proxy=False),
    # calibrated per-head widths (2 and 4 bits) on layer 0, 5 % outlier channels per head
    "d": dict(warm_bits=3, hot_budget=64, outlier_fraction=0.05, enable_promotion=False,
              enable_promotion_proxy=False),
}


@pytest.mark.parametrize("name", ["a", "b", "c", "d"])
def test_update_trace_matches_reference(name, golden_dir):
    from akv import AKVCache
    z = _traces(golden_dir)
    cache = AKVCache(num_hidden_layers=1, **CASES[name])
    if name == "b":
        cache.hot_budget = 48
    if name == "d":
        cache._calibration_per_head_bits = {0: [2, 4]}
    steps = z[f"{name}/steps"]
    k_in = torch.from_numpy(z[f"{name}/k_in"]).to(DEV)
    v_in = torch.from_numpy(z[f"{name}/v_in"]).to(DEV)
    wl, hl = z[f"{name}/warm_len"], z[f"{name}/hot_len"]
    wo = np.concatenate([[0], np.cumsum(wl)])
    ho = np.concatenate([[0], np.cumsum(hl)])
    if f"{name}/attn" in z:
        al = z[f"{name}/attn_len"]
        ao = np.concatenate([[0], np.cumsum(al)])
    t = 0
    for i, n in enumerate(steps):
        ck = None
        if f"{name}/attn" in z and i > 0:
            a = z[f"{name}/attn"][ao[i - 1]:ao[i]]
            ck = {"attention_weights": torch.from_numpy(a).view(1, 2, 1, -1).to(DEV)}
        full_k, full_v = cache.update(k_in[:, :, t:t + n], v_in[:, :, t:t + n], 0, ck)
        t += n
        layer = cache.layers[0]
        warm = [] if layer._warm_positions is None else layer._warm_positions.tolist()
        assert warm == z[f"{name}/warm_pos"][wo[i]:wo[i + 1]].tolist(), f"step {i}: warm positions"
        assert layer._hot_positions.tolist() == z[f"{name}/hot_pos"][ho[i]:ho[i + 1]].tolist(), f"step {i}: hot"
    np.testing.assert_array_equal(full_k.cpu().numpy().view(np.uint16), z[f"{name}/full_k"].view(np.uint16))
    np.testing.assert_array_equal(full_v.cpu().numpy().view(np.uint16), z[f"{name}/full_v"].view(np.uint16))
    mu = cache.memory_usage()
    for key in ("hot_bytes", "warm_bytes_packed", "warm_bytes_live", "fp16_equivalent_bytes", "total_bytes"):
        assert mu[key] == int(z[f"{name}/mem/{key}"]), key
    # the packed records hold exactly the warm tokens (valid-slot masks)
    masks = cache.layers[0]._warm.masks()[0, 0].tolist()
    assert sum(bin(int(m)).count("1") for m in masks) == int(wl[-1])


def _prefill(N, hot_budget, num_layers=1, heads=2, head_dim=32):
    from akv import AKVCache
    cache = AKVCache(warm_bits=3, hot_budget=hot_budget, enable_promotion=False, enable_promotion_proxy=False,
                     num_hidden_layers=num_layers)
    K = torch.arange(N, dtype=torch.float32).view(1, 1, N, 1).expand(1, heads, N, head_dim).contiguous().half()
    K = K.to(DEV)
    for layer_idx in range(num_layers):
        cache.update(K, K.clone(), layer_idx=layer_idx)
    return cache


def test_prefill_with_demote_position_coverage_is_complete():
    layer = _prefill(256, 32).layers[0]
    warm, hot = layer._warm_positions.tolist(), layer._hot_positions.tolist()
    assert len(warm) + len(hot) == 256 and sorted(warm + hot) == list(range(256))


def test_full_view_is_chronologically_sorted():
    layer = _prefill(256, 32).layers[0]
    assert layer.keys.shape[2] == 256
    pos = torch.cat([layer._warm_positions, layer._hot_positions])
    assert pos[pos.argsort()].tolist() == list(range(256))
    # warm rows are quantised, hot rows exact: each slot's value stays near its position
    approx = layer.keys[0, 0, :, 0].float().cpu()
    assert torch.all((approx - torch.arange(256).float()).abs() <= 256 / 7 / 2 + 1)


def test_promote_preserves_position_coverage():
    from akv import AKVCache
    N = 128
    cache = AKVCache(warm_bits=3, hot_budget=16, enable_promotion=True, enable_promotion_proxy=True,
                     promotion_threshold=0.0, num_hidden_layers=1)
    K = torch.arange(N, dtype=torch.float32).view(1, 1, N, 1).expand(1, 2, N, 32).contiguous().half().to(DEV)
    cache.update(K, K.clone(), layer_idx=0)
    g = torch.Generator(device=DEV).manual_seed(0)
    for _ in range(8):
        k1 = torch.randn(1, 2, 1, 32, generator=g, device=DEV).half()
        cache.update(k1, k1.clone(), layer_idx=0)
    layer = cache.layers[0]
    warm = layer._warm_positions.tolist() if layer._warm_positions is not None else []
    hot = layer._hot_positions.tolist()
    assert sorted(warm + hot) == list(range(N + 8))
    # promoted tokens are gone from the packed records too
    live = sum(bin(int(m)).count("1") for m in layer._warm.masks()[0, 0].tolist())
    assert live == len(warm)


def test_multilayer_independence():
    cache = _prefill(128, 32, num_layers=3)
    for layer in cache.layers:
        assert sorted(layer._warm_positions.tolist() + layer._hot_positions.tolist()) == list(range(128))


def test_generate_under_demotion_and_beam_ops():
    pytest.importorskip("transformers")
    from transformers import LlamaConfig, LlamaForCausalLM
    from akv import AKVCache
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=128, hidden_size=128, intermediate_size=256, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256, rms_norm_eps=1e-5)
    model = LlamaForCausalLM(cfg).eval().half().to(DEV)
    ids = torch.arange(1, 81, device=DEV).view(1, -1) % 127 + 1
    with torch.no_grad():
        cache = AKVCache(preset="k4v2", num_hidden_layers=2, outlier_fraction=0.05)
        cache.hot_budget = 24
        out = model.generate(ids, max_new_tokens=12, do_sample=False, past_key_values=cache, pad_token_id=0)
    assert out.shape[1] == ids.shape[1] + 12
    layer = cache.layers[0]
    assert layer._warm_keys_fp16 is not None and layer._hot_keys.shape[2] == 24
    mu = cache.memory_usage()
    assert mu["warm_bytes_packed"] > 0 and mu["savings_ratio"] > 1.0
    # beam-style batch ops keep every tier consistent
    cache.batch_repeat_interleave(2)
    assert layer._hot_keys.shape[0] == 2 and layer._warm.B == 2 and layer._warm_keys_fp16.shape[0] == 2
    cache.batch_select_indices(torch.tensor([1], device=DEV))
    assert layer._hot_keys.shape[0] == 1 and layer._warm.buf.shape[0] == 1


@pytest.mark.parametrize("frac", [0.0, 0.05])
def test_per_head_bits_match_reference_per_head_quantisation(frac):
    """per_head_bits (reference drop_in.py:315-374): head h is quantised on
    its own at per_head_bits[h] (K and V), outlier channels from that head
    alone.  The warm copy must equal the oracle's per-head quantiser calls
    bit for bit; the fused decode over the per-width arenas must match SDPA
    over the chronological view."""
    from akv import AKVLayer
    from oracle import akv_oracle as O
    bits = [2, 4, 3, 4]
    g = torch.Generator(device=DEV).manual_seed(11)
    k = torch.randn(1, 4, 100, 128, generator=g, device=DEV)
    k[..., 9] *= 12
    k, v = k.half(), torch.randn(1, 4, 100, 128, generator=g, device=DEV).half()
    layer = AKVLayer(warm_bits=3, hot_budget=40, enable_promotion=False, enable_promotion_proxy=False,
                     per_head_bits=bits, outlier_fraction=frac)
    layer.update(k, v)
    pos = layer._warm_positions.tolist()
    assert len(pos) == 60
    kn, vn = k.cpu().numpy(), v.cpu().numpy()
    for h, b in enumerate(bits):
        rk = O.dequantize_keys(O.quantize_keys(kn[0, h:h + 1][:, pos], b, frac))
        rv = O.dequantize_values(O.quantize_values(vn[0, h:h + 1][:, pos], b, frac))
        np.testing.assert_array_equal(layer._warm_keys_fp16[0, h:h + 1].cpu().numpy().view(np.uint16), rk.view(np.uint16))
        np.testing.assert_array_equal(layer._warm_values_fp16[0, h:h + 1].cpu().numpy().view(np.uint16), rv.view(np.uint16))
    pw = {2: 32, 3: 48, 4: 64}
    assert layer.memory_usage_bytes()["warm_bytes_packed"] == sum(2 * 60 * pw[b] + 4 * 128 + 4 * 60 for b in bits)
    # one decode step through the per-width arenas
    k1 = torch.randn(1, 4, 1, 128, generator=g, device=DEV).half()
    layer.update(k1, k1.clone())
    q = torch.randn(1, 8, 1, 128, generator=g, device=DEV).half()
    out = layer.decode_attention(q, 128 ** -0.5).float()
    fk, fv = layer.full_view()
    K, V = fk.float().repeat_interleave(2, 1), fv.float().repeat_interleave(2, 1)
    p = torch.softmax(torch.einsum("bhqd,bhnd->bhqn", q.float(), K) / 128 ** 0.5, -1)
    ref = torch.einsum("bhqn,bhnd->bhqd", p, V)
    assert (out - ref).abs().max().item() <= 2e-3


def test_per_head_bits_fallback_and_calibrated_layers():
    """Ported from the reference's tests/test_per_head_bits.py (:28-69): the
    per-head path demotes with one arena per distinct width; a width list that
    does not match the head count falls back to the layer's widths; only
    calibrated layers get per-head widths."""
    from akv import AKVCache, AKVLayer
    from akv.packed_layout import HeadGroupArena, WarmArena
    g = torch.Generator(device=DEV).manual_seed(12)
    x = torch.randn(1, 2, 4, 128, generator=g, device=DEV).half()
    layer = AKVLayer(warm_bits=3, hot_budget=2, per_head_bits=[2, 3, 4, 2])  # 4 widths, 2 heads
    layer.update(x, x.clone())
    assert isinstance(layer._warm, WarmArena) and layer._warm_keys_fp16.shape[2] == 2
    layer = AKVLayer(warm_bits=4, hot_budget=2, per_head_bits=[2, 3])
    layer.update(x, x.clone())
    assert isinstance(layer._warm, HeadGroupArena) and layer._warm_keys_fp16.shape[2] == 2
    assert sorted(b for b, _, _ in layer._warm.groups) == [2, 3]
    cache = AKVCache(warm_bits=3, hot_budget=4)
    cache._calibration_per_head_bits = {0: [2, 4]}
    y = torch.randn(1, 2, 6, 128, generator=g, device=DEV).half()
    cache.update(y, y.clone(), layer_idx=0)
    cache.update(y, y.clone(), layer_idx=1)
    assert cache.layers[0].per_head_bits == [2, 4] and isinstance(cache.layers[0]._warm, HeadGroupArena)
    assert cache.layers[1].per_head_bits is None and isinstance(cache.layers[1]._warm, WarmArena)


def test_byte_accounting_ported_from_reference():
    """Ported from the reference's tests/test_packed_bytes.py (:95-125) and
    tests/test_memory_alignment.py (:140-168): after demotion the measured
    packed bytes are positive, below the FP16 working copy and the FP16
    equivalent, ``warm_bytes`` aliases them, and the cache aggregate exposes
    every key."""
    from akv import AKVCache, AKVLayer
    g = torch.Generator(device=DEV).manual_seed(13)
    layer = AKVLayer(warm_bits=4, hot_budget=4, group_size=32)
    k = torch.randn(1, 2, 8, 128, generator=g, device=DEV).half()
    v = torch.randn(1, 2, 8, 128, generator=g, device=DEV).half()
    layer.update(k, v)
    layer.update(k, v)
    st = layer.memory_usage_bytes()
    for key in ("warm_bytes_live", "warm_bytes_packed", "warm_bytes_formula"):
        assert key in st
    assert 0 < st["warm_bytes_packed"] < st["warm_bytes_live"]
    assert st["warm_bytes_packed"] < st["fp16_equivalent_bytes"]
    assert st["warm_bytes"] == st["warm_bytes_packed"]
    cache = AKVCache(warm_bits=4, hot_budget=4, num_hidden_layers=1)
    cache.update(torch.randn(1, 2, 16, 128, generator=g, device=DEV).half(),
                 torch.randn(1, 2, 16, 128, generator=g, device=DEV).half(), layer_idx=0)
    stats = cache.memory_usage()
    for key in ("hot_bytes", "warm_bytes", "warm_bytes_live", "warm_bytes_packed", "warm_bytes_formula",
                "total_bytes", "fp16_equivalent_bytes", "savings_ratio", "num_layers"):
        assert key in stats
    assert stats["warm_bytes"] == stats["warm_bytes_packed"] <= stats["warm_bytes_live"]
