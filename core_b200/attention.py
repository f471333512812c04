"""Attention hook of the prefill: causal attention on this library's tcgen05
kernel, with the row LSE kept for the press.

Drop-in for ``_core_flash_attention_forward`` (reference
``core/kvpress_pipeline.py:24-91``): the module keeps its post-RoPE queries in
``_core_cached_query_states`` and, when the forward is the plain causal case,
the attention's ``softmax_lse`` in ``_core_cached_softmax_lse``.  The press then
uses that LSE as the QK relation pass's row normaliser and skips its own LSE
pass (``COREScorerPress`` reads it at prefill, as the reference's
``kvpress_adapter.py:400-438`` does).  Forwards outside the plain causal case
(an explicit mask, dropout, a sliding window, softcapping, autograd, dtypes
other than bf16/f16, head_dim other than 128) run transformers' own SDPA
attention and leave the LSE unset, as the reference falls back to the
upstream implementation there.

Use::

    from core_b200 import attention
    attention.register()                        # once per process
    model = AutoModelForCausalLM.from_pretrained(..., attn_implementation="core_b200")
"""

from __future__ import annotations

import torch

from . import ops

IMPLEMENTATION = "core_b200"


def _lse_case(module, query_states, key_states, value_states, attention_mask, kwargs) -> bool:
    dropout = float(kwargs.get("dropout", 0.0) or 0.0)
    scaling = kwargs.get("scaling")
    is_causal = kwargs.get("is_causal")
    if is_causal is None:
        is_causal = bool(getattr(module, "is_causal", True))
    d = query_states.shape[-1]
    scale_ok = scaling is None or abs(float(scaling) - d ** -0.5) <= 1e-12
    return (attention_mask is None and dropout == 0.0 and bool(is_causal) and scale_ok
            and kwargs.get("sliding_window") is None and kwargs.get("softcap") in (None, 0.0)
            and not torch.is_grad_enabled()
            and query_states.is_cuda
            and query_states.dtype in (torch.bfloat16, torch.float16)
            and key_states.dtype == query_states.dtype
            and value_states.dtype == query_states.dtype
            and d == ops.HEAD_DIM
            and query_states.shape[2] <= key_states.shape[2])


def attention_forward(module, query_states, key_states, value_states, attention_mask, **kwargs):
    """An HF attention function: (B, Hq, Lq, d) queries, (B, Hkv, Lk, d) keys and
    values -> ((B, Lq, Hq, d) output, None)."""
    module._core_cached_query_states = query_states
    module._core_cached_softmax_lse = None
    if _lse_case(module, query_states, key_states, value_states, attention_mask, kwargs):
        out, lse = ops.attention_prefill(query_states, key_states, value_states,
                                         softmax_scale=query_states.shape[-1] ** -0.5)
        module._core_cached_softmax_lse = lse
        return out, None
    from transformers.integrations.sdpa_attention import sdpa_attention_forward
    return sdpa_attention_forward(module, query_states, key_states, value_states, attention_mask,
                                  **kwargs)


def register(name: str = IMPLEMENTATION) -> str:
    """Register ``attention_forward`` with transformers under ``name`` (with the
    SDPA mask builder, which hands a plain causal prefill no mask)."""
    from transformers.masking_utils import ALL_MASK_ATTENTION_FUNCTIONS, AttentionMaskInterface
    from transformers.modeling_utils import AttentionInterface

    AttentionInterface.register(name, attention_forward)
    AttentionMaskInterface.register(name, ALL_MASK_ATTENTION_FUNCTIONS["sdpa"])
    return name
