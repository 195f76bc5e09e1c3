"""HuggingFace attention hook: decode and prefill attend over the packed warm tier.

The reference's ``AKVLayer.update`` returns the chronologically sorted
[dequantised warm; hot] FP16 view and the model's attention runs over it
(akv/drop_in.py:753-787).  ``register()`` adds an attention implementation
``"akv"`` to ``transformers.AttentionInterface`` (with the SDPA mask
builder under the same name).  With ``AKVCache(fused_decode=True)``:

* a decode step (one query token, no padding mask, no sliding window, head
  dim 64, 128 or 256) calls the sm_100a mixed-tier decode kernel on the
  layer's packed warm block records and FP16 hot tier in place; no FP16
  view is built or read;
* a prefill with no padding mask (HF passes none for a plain causal prompt)
  at head dim 128 calls the tcgen05 prefill kernel on the same tiers,
  causal by token position;
* everything else (masked or padded batches, sliding windows, per-head bit
  widths at prefill, layers without a warm tier, caches that are not fused)
  goes to torch's SDPA over the view, as the reference does.

Softmax attention of a single query does not depend on the order of the
keys, so attending over [warm records; hot] equals attending over the
chronological view.

Usage::

    import akv.hf_attention
    akv.hf_attention.register()
    model = AutoModelForCausalLM.from_config(cfg, attn_implementation="akv")
    cache = akv.AKVCache(warm_bits=3, hot_budget=1024, fused_decode=True)
    model.generate(ids, past_key_values=cache, ...)
"""
from __future__ import annotations

from typing import Optional

import torch

from .fused_attention import KERNEL_HEAD_DIM, KERNEL_HEAD_DIMS

NAME = "akv"


def akv_attention_forward(module: torch.nn.Module, query: torch.Tensor, key: torch.Tensor, value: torch.Tensor,
                          attention_mask: Optional[torch.Tensor], dropout: float = 0.0,
                          scaling: Optional[float] = None, is_causal: Optional[bool] = None, **kwargs):
    """The ``AttentionInterface`` signature: query (B, Hq, q_len, D), key /
    value (B, Hkv, kv_len, D); returns ((B, q_len, Hq, D), None)."""
    layer = getattr(key, "_akv_layer", None)
    if layer is not None:
        plain = attention_mask is None and not dropout and kwargs.get("sliding_window") is None
        if plain and query.shape[2] == 1 and query.shape[-1] in KERNEL_HEAD_DIMS:
            # the output buffer is the layer's own, rewritten at its next decode
            # step; the caller's o_proj has consumed it by then (stream order)
            out = layer.decode_attention(query, scaling, reuse_out=True)  # (B, Hq, 1, D)
            return out.transpose(1, 2), None
        if plain and query.shape[-1] == KERNEL_HEAD_DIM and is_causal is not False and layer.can_prefill_fused():
            out = layer.prefill_attention(query, scaling)  # (B, Hq, q_len, D), causal by position
            return out.transpose(1, 2), None
        key, value = layer.full_view()
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    return sdpa_attention_forward(module, query, key, value, attention_mask, dropout=dropout, scaling=scaling,
                                  is_causal=is_causal, **kwargs)


def register(name: str = NAME) -> str:
    """Register the hook (and the SDPA mask builder) under ``name``."""
    from transformers import AttentionInterface
    from transformers.masking_utils import AttentionMaskInterface, sdpa_mask

    AttentionInterface.register(name, akv_attention_forward)
    AttentionMaskInterface.register(name, sdpa_mask)
    return name
