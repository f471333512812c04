"""Causal prefill attention with the row LSE (core_attention_prefill), the
kernel behind the press's attention hook (reference
core/kvpress_pipeline.py:24-91).

Checked against the same attention computed by torch in f64 from the 16-bit
inputs, against flash_attn_func (the library the reference calls) where it
runs on this GPU, and through its use: its LSE as the QK relation pass's row
normaliser against the oracle given the same LSE.

Tolerances.  P is rounded to the input dtype before the P V product (as
FlashAttention does), which moves an output by at most u * max|v| (u = 2^-9
for bf16, 2^-12 for f16: sum p = 1); the output rounding adds u |out|.  The
LSE is an f32 sum of f32 exponentials of scores that the tensor cores
accumulate in f32: within 1e-5 of the largest |LSE| plus 2e-5 (the
specification allows 2e-3 relative)."""

import numpy as np
import pytest
import torch

from helpers import check_qk_features_bounded, flip_bound
from oracle import core_oracle as O

pytestmark = pytest.mark.gpu

LSE_ATOL = 2e-5
LSE_RTOL = 1e-5


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _reference(q, k, v, scale):
    """f64 attention per head: (out (B, Lq, Hq, d), lse (B, Hq, Lq))."""
    B, Hq, Lq, d = q.shape
    Hkv, Lk = k.shape[1], k.shape[2]
    G = Hq // Hkv
    out = torch.empty(B, Lq, Hq, d, dtype=torch.float64, device=q.device)
    lse = torch.empty(B, Hq, Lq, dtype=torch.float64, device=q.device)
    i = torch.arange(Lq, device=q.device)[:, None]
    j = torch.arange(Lk, device=q.device)[None, :]
    masked = j > i + (Lk - Lq)
    for b in range(B):
        for h in range(Hq):
            s = (q[b, h].double() @ k[b, h // G].double().T) * scale
            s = s.masked_fill(masked, float("-inf"))
            l = torch.logsumexp(s, -1)
            lse[b, h] = l
            out[b, :, h] = torch.exp(s - l[:, None]) @ v[b, h // G].double()
    return out, lse


def _inputs(seed, B, Hq, Hkv, Lq, Lk, dtype, dev, outliers=True):
    g = torch.Generator(device="cpu").manual_seed(seed)
    q = torch.randn(B, Hq, Lq, 128, generator=g) / 128 ** 0.5
    k = torch.randn(B, Hkv, Lk, 128, generator=g) / 128 ** 0.5
    if outliers:  # a few large channels, as in real keys, so that rows have peaked softmaxes
        ch = torch.randperm(128, generator=g)[:4]
        q[..., ch] *= 8
        k[..., ch] *= 8 * 4
    v = torch.randn(B, Hkv, Lk, 128, generator=g)
    if Lk > 700:
        # a few late keys with large scores: rows whose running maximum must be
        # raised (and O rescaled) after earlier tiles were accumulated
        k[:, :, 700] *= 60
        k[:, :, Lk - 3] *= 40
    return q.to(dev, dtype), k.to(dev, dtype), v.to(dev, dtype)


def _check(out, lse, ref_out, ref_lse, v, dtype):
    u = 2.0 ** -9 if dtype == torch.bfloat16 else 2.0 ** -12
    err = (out.double() - ref_out).abs()
    bound = 1.05 * u * v.double().abs().max() + 2 * u * ref_out.abs() + 1e-6
    assert bool((err <= bound).all()), float((err - bound).max())
    assert float((lse.double() - ref_lse).abs().max()) <= LSE_ATOL + LSE_RTOL * float(ref_lse.abs().max())


CASES = [
    # (B, Hq, Hkv, Lq, Lk, dtype)
    (1, 8, 2, 1000, 1000, torch.bfloat16),     # ragged tiles, GQA 4
    (2, 32, 8, 384, 384, torch.bfloat16),      # Llama heads, two batch rows
    (1, 4, 4, 200, 777, torch.float16),        # fewer queries than keys: bottom-right causal
    (1, 8, 8, 129, 129, torch.bfloat16),       # one row past a tile
    (1, 2, 1, 1, 300, torch.bfloat16),         # one query (a decode-shaped call)
]


@pytest.mark.parametrize("B,Hq,Hkv,Lq,Lk,dtype", CASES)
def test_attention_matches_f64_reference(B, Hq, Hkv, Lq, Lk, dtype):
    from core_b200 import ops
    dev = _dev()
    q, k, v = _inputs(1, B, Hq, Hkv, Lq, Lk, dtype, dev)
    out, lse = ops.attention_prefill(q, k, v)
    ops.status()
    ref_out, ref_lse = _reference(q, k, v, 128 ** -0.5)
    _check(out, lse, ref_out, ref_lse, v, dtype)


def test_attention_strided_queries_and_repeat_calls():
    """Queries in the (B, L, H, d) memory order an HF module hands over, and
    two calls in a row give identical bits."""
    from core_b200 import ops
    dev = _dev()
    q, k, v = _inputs(2, 1, 32, 8, 2048, 2048, torch.bfloat16, dev)
    qs = q.transpose(1, 2).contiguous().transpose(1, 2)  # strides of (B, L, H, d)
    assert not qs.is_contiguous()
    out, lse = ops.attention_prefill(qs, k, v)
    out2, lse2 = ops.attention_prefill(q, k, v)
    ops.status()
    assert torch.equal(out, out2) and torch.equal(lse, lse2)
    ref_out, ref_lse = _reference(q, k, v, 128 ** -0.5)
    _check(out, lse, ref_out, ref_lse, v, torch.bfloat16)


def test_attention_matches_flash_attn():
    """Against flash_attn_func, the library call of the reference's hook."""
    try:
        from flash_attn import flash_attn_func
    except Exception as e:  # noqa: BLE001
        pytest.skip(f"flash_attn not importable: {e}")
    from core_b200 import ops
    dev = _dev()
    q, k, v = _inputs(3, 1, 32, 8, 1536, 1536, torch.bfloat16, dev)
    try:
        ref_out, ref_lse, _ = flash_attn_func(q.transpose(1, 2), k.transpose(1, 2),
                                              v.transpose(1, 2), dropout_p=0.0,
                                              softmax_scale=128 ** -0.5, causal=True,
                                              return_attn_probs=True)
        torch.cuda.synchronize()
    except RuntimeError as e:
        pytest.skip(f"flash_attn does not run on this GPU: {e}")
    out, lse = ops.attention_prefill(q, k, v)
    ops.status()
    u = 2.0 ** -9
    err = (out.float() - ref_out.float()).abs()
    # both round P and the output to bf16: twice the one-sided bound
    bound = 2.1 * u * v.float().abs().max() + 4 * u * ref_out.float().abs()
    assert bool((err <= bound).all())
    assert float((lse - ref_lse.float()).abs().max()) <= LSE_ATOL + LSE_RTOL * float(ref_lse.abs().max())


def test_attention_lse_drives_qk_features():
    """The exported LSE as the relation pass's row normaliser (the reference's
    row_lse reuse, core/fused_qk.py:444-456): question scope (last 128
    queries) and full scope, against the oracle given the same LSE."""
    from core_b200 import ops, synthetic
    dev = _dev()
    L = 1024
    q, k, v = synthetic.make_layer_inputs(seed=21, batch=1, n_kv_heads=8, n_q_heads=32,
                                          seq_len=L, n_queries=L, device=dev)
    _, lse = ops.attention_prefill(q, k, v)
    ops.status()
    kn = k[0].float().cpu().numpy()
    for nq in (128, L):
        qq = q[:, :, L - nq:].contiguous()
        lq = lse[:, :, L - nq:].contiguous()
        feats, lse_used = ops.qk_features(qq, k, lse=lq)
        ops.status()
        assert torch.equal(lse_used, lq)  # the given LSE is used as is
        qn = qq[0].float().cpu().numpy()
        ref, _, R = O.qk_features(qn, kn, groups=4, round_bf16=True, lse=lq[0].cpu().numpy())
        check_qk_features_bounded(feats[0].cpu().numpy(), ref, R, flip_bound(qn, kn, 0.0),
                                  rtol=2e-3, max_frac=0.01 if nq == 128 else 0.05)


def test_attention_hook_sets_the_press_state():
    """attention.attention_forward as an HF attention function: the module
    keeps its queries and the LSE; a masked forward falls back to SDPA and
    leaves the LSE unset."""
    from core_b200 import attention
    dev = _dev()
    q, k, v = _inputs(4, 1, 8, 2, 300, 300, torch.bfloat16, dev)
    mod = torch.nn.Module()
    mod.is_causal = True
    with torch.no_grad():
        out, _ = attention.attention_forward(mod, q, k, v, None, dropout=0.0, scaling=128 ** -0.5)
    assert mod._core_cached_query_states is q
    assert mod._core_cached_softmax_lse is not None and mod._core_cached_softmax_lse.shape == (1, 8, 300)
    ref_out, ref_lse = _reference(q, k, v, 128 ** -0.5)
    _check(out, mod._core_cached_softmax_lse, ref_out, ref_lse, v, torch.bfloat16)
    mask = torch.ones(1, 1, 300, 300, dtype=torch.bool, device=dev).tril()
    mod.num_key_value_groups = 4
    with torch.no_grad():
        out2, _ = attention.attention_forward(mod, q, k, v, mask, dropout=0.0, scaling=128 ** -0.5)
    assert mod._core_cached_softmax_lse is None
    assert float((out2.double() - ref_out).abs().max()) < 0.05
