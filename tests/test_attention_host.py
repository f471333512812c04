"""The attention hook's host logic without a GPU: transformers accepts the
registered implementation, and a forward outside the LSE case (here: CPU
tensors) runs transformers' SDPA attention with the LSE left unset."""

import copy

import pytest
import torch


def test_register_and_fallback_forward_on_cpu():
    transformers = pytest.importorskip("transformers")
    from core_b200 import attention

    name = attention.register()
    cfg = transformers.LlamaConfig(vocab_size=64, hidden_size=256, intermediate_size=256,
                                   num_hidden_layers=1, num_attention_heads=2,
                                   num_key_value_heads=1, head_dim=128,
                                   max_position_embeddings=64)
    torch.manual_seed(0)
    m_core = transformers.LlamaForCausalLM._from_config(cfg, attn_implementation=name).eval()
    m_sdpa = transformers.LlamaForCausalLM._from_config(copy.deepcopy(cfg),
                                                      attn_implementation="sdpa").eval()
    m_sdpa.load_state_dict(m_core.state_dict())
    ids = torch.randint(0, 64, (1, 12))
    with torch.no_grad():
        a = m_core(ids).logits
        b = m_sdpa(ids).logits
    assert torch.allclose(a, b, atol=1e-5)
    attn = m_core.model.layers[0].self_attn
    assert getattr(attn, "_core_cached_softmax_lse", "unset") is None
    assert attn._core_cached_query_states.shape == (1, 2, 12, 128)


def test_lse_case_conditions():
    from core_b200 import attention

    mod = torch.nn.Module()
    q = torch.zeros(1, 4, 8, 128, dtype=torch.bfloat16)
    k = torch.zeros(1, 2, 8, 128, dtype=torch.bfloat16)
    with torch.no_grad():
        # CPU tensors never take the kernel path
        assert not attention._lse_case(mod, q, k, k, None, {})
    assert not attention._lse_case(mod, q, k, k, None, {"dropout": 0.1})
