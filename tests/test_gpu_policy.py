"""GPU: tier-policy behaviour ported from the reference's
tests/test_proxy_promotion.py (attention-free promotion proxy and adaptive
hot budget), run on CUDA tensors at head_dim 128 (the warm tier's kernels
need a GPU; the reference runs these on CPU at head_dim 8-16)."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"


def _step(layer, g, H=4, D=128, direction=None):
    if direction is None:
        k = torch.randn(1, H, 1, D, generator=g, device=DEV)
    else:
        k = direction.expand(1, H, 1, D).clone() + 0.01 * torch.randn(1, H, 1, D, generator=g, device=DEV)
    v = torch.randn(1, H, 1, D, generator=g, device=DEV)
    layer.update(k.half(), v.half(), cache_kwargs=None)


def test_proxy_fires_without_attention_weights():
    """(:32-51) the proxy runs with no attention weights and tracks the warm tier."""
    from akv import AKVLayer
    layer = AKVLayer(warm_bits=3, hot_budget=8, group_size=4, enable_promotion=True, enable_promotion_proxy=True,
                     promotion_threshold=0.0, proxy_decay=0.0)
    g = torch.Generator(device=DEV).manual_seed(0)
    for _ in range(16):
        _step(layer, g)
    assert layer._warm_len > 0
    assert layer._proxy_score is not None and layer._proxy_score.shape[0] == layer._warm_len
    live = sum(bin(int(m) & 0xFFFFFFFF).count("1") for m in layer._warm.masks()[0, 0].tolist())
    assert live == layer._warm_len  # promoted tokens left the packed records too


def test_proxy_disabled_skips_path():
    """(:54-70) no proxy state when the proxy is off and no weights arrive."""
    from akv import AKVLayer
    layer = AKVLayer(warm_bits=3, hot_budget=8, group_size=4, enable_promotion=True, enable_promotion_proxy=False)
    g = torch.Generator(device=DEV).manual_seed(1)
    for _ in range(16):
        _step(layer, g)
    assert layer._proxy_score is None


def test_proxy_ranks_similar_warm_slot_highest():
    """(:73-133) a query along a demoted token's direction ranks that warm slot first."""
    from akv import AKVLayer
    layer = AKVLayer(warm_bits=4, hot_budget=16, group_size=4, enable_promotion=False, enable_promotion_proxy=True,
                     proxy_decay=0.0)
    g = torch.Generator(device=DEV).manual_seed(7)
    for _ in range(4):
        _step(layer, g)
    target = torch.randn(1, 1, 1, 128, generator=g, device=DEV)
    target = target / target.norm()
    _step(layer, g, direction=target)
    for _ in range(40):
        _step(layer, g)
    assert layer._warm_len > 0
    _step(layer, g, direction=target)
    wk = layer._warm_keys_fp16.float().mean(dim=(0, 1))
    wk = wk / (wk.norm(dim=-1, keepdim=True) + 1e-6)
    true_sim = (wk @ target.view(-1)).abs()
    assert int(layer._proxy_score.argmax()) == int(true_sim.argmax())


def test_proxy_score_resizes_on_demote():
    """(:136-153) the proxy vector grows with the warm tier."""
    from akv import AKVLayer
    layer = AKVLayer(warm_bits=3, hot_budget=4, group_size=4, enable_promotion=True, enable_promotion_proxy=True,
                     promotion_threshold=10.0, proxy_decay=0.5)
    g = torch.Generator(device=DEV).manual_seed(2)
    for _ in range(8):
        _step(layer, g, H=2)
    assert layer._warm_len > 0 and layer._proxy_score.shape[0] == layer._warm_len


def test_adaptive_hot_budget_scales_with_context():
    """(:156-188) adaptive_hot_frac grows the hot tier past the fixed budget."""
    from akv import AKVCache
    fixed = AKVCache(warm_bits=3, hot_budget=8, group_size=4, adaptive_hot_frac=0.0)
    adaptive = AKVCache(warm_bits=3, hot_budget=8, group_size=4, adaptive_hot_frac=0.25)
    g = torch.Generator(device=DEV).manual_seed(42)
    for _ in range(40):
        k = torch.randn(1, 4, 1, 128, generator=g, device=DEV).half()
        v = torch.randn(1, 4, 1, 128, generator=g, device=DEV).half()
        fixed.update(k.clone(), v.clone(), layer_idx=0)
        adaptive.update(k.clone(), v.clone(), layer_idx=0)
    fh, ah = fixed.layers[0]._hot_keys.shape[2], adaptive.layers[0]._hot_keys.shape[2]
    assert fh <= 9 and ah > fh
