"""GPU: the "akv" HuggingFace attention hook over AKVCache(fused_decode=True).

A decode step or a causal prefill of a fused cache attends over the packed
warm records and the hot tier in place (akv.hf_attention).  Checked against the reference data
flow (drop_in.py:753-787): SDPA over the chronological [dequantised warm;
hot] FP16 view that a non-fused AKVCache returns.

* per call: on the prefill and every decode step of a Qwen2-shaped model, the
  hook's output equals fp32 SDPA over the same layer's full view within the
  attention bar, or is no further from it than the reference data flow's own
  fp16 SDPA over that view (both round the softmax weights to fp16);
* end to end: teacher-forced decoding through the fused cache gives the same
  logits as the view cache, within a tolerance that allows each layer's
  attention to differ by the attention bar.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda:0"
ATOL = 2e-3


def _excess(out, ref):
    """max over elements of |out - ref| - tol(ref), the attention bar of the
    decode tests: 2e-3, or the fp16 output's half-ulp + 1e-3 where |ref| >= 4."""
    ulp = torch.abs(ref).half().float()
    ulp = torch.nextafter(ulp.half(), torch.tensor(float("inf"), dtype=torch.float16, device=ref.device)).float() - ulp
    tol = torch.clamp(0.5 * ulp + 1e-3, min=ATOL)
    return ((out - ref).abs() - tol).max().item()


def _model(layers=2, vocab=1000, head_dim=128):
    from transformers import Qwen2Config, Qwen2ForCausalLM
    import akv.hf_attention as hook
    hook.register()
    torch.manual_seed(0)
    heads = 512 // head_dim if head_dim <= 128 else 4
    cfg = Qwen2Config(vocab_size=vocab, hidden_size=heads * head_dim, intermediate_size=1024,
                      num_hidden_layers=layers, num_attention_heads=heads, num_key_value_heads=2,
                      max_position_embeddings=4096,
                      rms_norm_eps=1e-6, initializer_range=0.08)
    return Qwen2ForCausalLM(cfg).eval().half().to(DEV)


def _step(model, cache, ids):
    out = model(input_ids=ids, past_key_values=cache, use_cache=True, logits_to_keep=1)
    return out.logits[:, -1].float()


@pytest.mark.parametrize("policy,head_dim", [("recency", 128), ("proxy_promotion", 128), ("k4v2_outliers", 128),
                                             ("recency", 64), ("k4v2_outliers", 64), ("recency", 256),
                                             ("k4v2_outliers", 256)])
def test_hook_matches_sdpa_over_view_each_step(policy, head_dim, monkeypatch):
    """Every fused decode call against SDPA over that layer's full view, on
    models with head dim 128 (Llama / Qwen), 64 (TinyLlama-like: 8 query /
    2 KV heads) and 256 (Gemma-like)."""
    import akv
    import akv.hf_attention as hook
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    kw = {
        "recency": dict(warm_bits=3, hot_budget=48, enable_promotion=False, enable_promotion_proxy=False),
        "proxy_promotion": dict(warm_bits=3, hot_budget=48, enable_promotion=True, enable_promotion_proxy=True,
                                promotion_threshold=0.05),
        "k4v2_outliers": dict(warm_key_bits=4, warm_value_bits=2, warm_bits=4, hot_budget=40,
                              outlier_fraction=0.02, enable_promotion=False, enable_promotion_proxy=False),
    }[policy]
    model = _model(head_dim=head_dim)
    model.config._attn_implementation = "akv"
    errs, calls, prefills = [], [0], [0]
    real = hook.akv_attention_forward

    def checked(module, query, key, value, attention_mask, **k2):
        out, w = real(module, query, key, value, attention_mask, **k2)
        layer = getattr(key, "_akv_layer", None)
        if layer is not None and attention_mask is None:
            causal = query.shape[2] > 1  # a prefill: the tcgen05 kernel, causal by position
            if causal:
                prefills[0] += 1
            else:
                calls[0] += 1
            fk, fv = layer.full_view()
            ref, _ = sdpa_attention_forward(module, query.float(), fk.float(), fv.float(), None,
                                            scaling=k2.get("scaling"), is_causal=causal)
            # the reference data flow itself: fp16 SDPA over the same view
            r16, _ = sdpa_attention_forward(module, query, fk, fv, None, scaling=k2.get("scaling"), is_causal=causal)
            e = (out.float() - ref).abs().max().item()
            e16 = (r16.float() - ref).abs().max().item()
            errs.append((e, _excess(out.float(), ref), e16))
        return out, w

    from transformers import AttentionInterface
    AttentionInterface.register("akv", checked)
    try:
        cache = akv.AKVCache(num_hidden_layers=2, fused_decode=True, **kw)
        g = torch.Generator(device=DEV).manual_seed(1)
        ids = torch.randint(1, 1000, (1, 200), generator=g, device=DEV)
        with torch.no_grad():
            _step(model, cache, ids)
            for _ in range(24):
                ids = torch.randint(1, 1000, (1, 1), generator=g, device=DEV)
                _step(model, cache, ids)
    finally:
        AttentionInterface.register("akv", real)
    assert calls[0] == 2 * 24, calls
    assert prefills[0] == 2, prefills  # the 200-token prompt of both layers went through the prefill kernel
    print(f"[hf hook {policy}] max |fused - sdpa32(view)| = {max(e[0] for e in errs):.2e}, "
          f"fp16 sdpa(view): {max(e[2] for e in errs):.2e}")
    # every call within the attention bar of fp32 attention, or no further from
    # it than the reference's own fp16 SDPA over the same view (plus 25 %)
    assert all(ex <= 0.0 or e <= 1.25 * e16 for e, ex, e16 in errs), [x for x in errs if x[1] > 0]
    layer = cache.layers[0]
    assert layer._warm is not None and layer._hot_keys.shape[2] == cache.hot_budget
    if policy != "proxy_promotion":  # fused and never promoting: no FP16 warm copy is kept
        assert layer._warm_keys_fp16 is None and cache.memory_usage()["warm_bytes_live"] == 0
    if policy == "proxy_promotion":
        live = sum(bin(int(m) & 0xFFFFFFFF).count("1") for m in layer._warm.masks()[0, 0].tolist())
        assert live == layer._warm_keys_fp16.shape[2]


def _fp32_attention(module, query, key, value, attention_mask, dropout=0.0, scaling=None, is_causal=None, **kw):
    """SDPA in fp32 over the (real, non-fused) view: the exact-attention arm."""
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    out, w = sdpa_attention_forward(module, query.float(), key.float(), value.float(), attention_mask,
                                    dropout=dropout, scaling=scaling, is_causal=is_causal, **kw)
    return out.to(query.dtype), w


def test_fused_decoding_logits_match_view_cache():
    """Teacher-forced decoding: the fused cache + "akv" hook (prefill and
    decode kernels) against the reference data flow (view cache + fp16 SDPA),
    both measured against fp32 attention over the same view.  Every attention
    call of either arm differs from fp32 attention by fp16 rounding, and the
    model amplifies that through its layers; the fused arm must stay as close
    to the fp32 arm as the reference flow is."""
    import akv
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask
    AttentionInterface.register("akv_fp32", _fp32_attention)
    AttentionMaskInterface.register("akv_fp32", sdpa_mask)
    model = _model()
    g = torch.Generator(device=DEV).manual_seed(2)
    prompt = torch.randint(1, 1000, (1, 300), generator=g, device=DEV)
    toks = torch.randint(1, 1000, (1, 32), generator=g, device=DEV)
    kw = dict(warm_bits=3, hot_budget=64, enable_promotion=False, enable_promotion_proxy=False, num_hidden_layers=2)
    logits = {}
    for mode, impl in (("view", "sdpa"), ("fused", "akv"), ("fp32", "akv_fp32")):
        model.config._attn_implementation = impl
        cache = akv.AKVCache(fused_decode=(mode == "fused"), **kw)
        rows = []
        with torch.no_grad():
            rows.append(_step(model, cache, prompt))
            for i in range(toks.shape[1]):
                rows.append(_step(model, cache, toks[:, i:i + 1]))
        logits[mode] = torch.cat(rows)
        assert cache.layers[1]._warm is not None
    model.config._attn_implementation = "sdpa"
    ref, view, fused = logits["fp32"], logits["view"], logits["fused"]
    e_view = (view - ref).abs().max().item()
    e_fused = (fused - ref).abs().max().item()
    scale = ref.abs().max().item()
    print(f"[hf hook e2e] max |logits - fp32 arm|: fused {e_fused:.3e}, view+SDPA {e_view:.3e} "
          f"(max |logit| {scale:.2f})")
    assert torch.isfinite(fused).all()
    assert e_fused <= max(1.5 * e_view, 2e-2 * max(scale, 1.0))
    agree = lambda a: (a.argmax(-1) == ref.argmax(-1)).float().mean().item()  # noqa: E731
    assert agree(fused) >= agree(view) - 0.05


def test_generate_with_hook_and_beam_ops():
    """HF generate through the hook; padded batches fall back to SDPA over the view."""
    import akv
    model = _model()
    model.config._attn_implementation = "akv"
    g = torch.Generator(device=DEV).manual_seed(3)
    ids = torch.randint(1, 1000, (2, 120), generator=g, device=DEV)
    mask = torch.ones_like(ids)
    mask[1, :7] = 0  # left padding on row 1: the mask path, not the fused one
    with torch.no_grad():
        cache = akv.AKVCache(warm_bits=3, hot_budget=32, enable_promotion=False, enable_promotion_proxy=False,
                             num_hidden_layers=2, fused_decode=True)
        out = model.generate(ids, attention_mask=mask, max_new_tokens=8, do_sample=False, past_key_values=cache,
                             pad_token_id=0)
        assert out.shape == (2, 128)
        cache2 = akv.AKVCache(warm_bits=3, hot_budget=32, enable_promotion=False, enable_promotion_proxy=False,
                              num_hidden_layers=2, fused_decode=True)
        out2 = model.generate(ids[:1], max_new_tokens=8, do_sample=False, past_key_values=cache2, pad_token_id=0)
        assert out2.shape == (1, 128)
    layer = cache2.layers[0]
    assert getattr(layer.keys, "_akv_layer", None) is layer
    assert layer.get_seq_length() == 127
    cache2.batch_repeat_interleave(2)
    assert layer._hot_keys.shape[0] == 2 and layer.keys.shape[0] == 2
    model.config._attn_implementation = "sdpa"
