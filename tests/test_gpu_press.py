"""The drop-in press on the GPU against fixtures the reference's own presses
wrote: the hook-level case (prefill through the forward hook, decode steps
with the memory readout, decode recompressions scored by queries the press
rebuilds with q_proj and the library's RoPE kernel) and the two-step case.

Tolerances are those of the BASELINE parity rule: keep sets bit-exact except
keys whose score lies within 1e-3 relative of the Top-B boundary; gathered
K/V bit-exact; scores and M/b/Z within 2e-3 relative; bf16 readout outputs
equal up to one bf16 rounding of the residual sum on a few entries.
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from helpers import (HOOK_CASE, TWO_STEP_CASE, hook_decode_steps, hook_events, hook_rotary,
                     load_case)

pytestmark = pytest.mark.gpu

SCORE_TOL = 2e-3
STATE_TOL = 2e-3


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


def _bf16(a, dev):
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev).to(torch.bfloat16)


class _Attention:
    """A Llama attention module as the press's hooks see it."""

    def __init__(self, layer_idx, q_proj, o_proj, rotary, meta):
        self.layer_idx = layer_idx
        self.q_proj = q_proj
        self.o_proj = o_proj
        self.rotary_emb = rotary
        self.head_dim = meta["d"]
        self.config = SimpleNamespace(num_attention_heads=meta["hq"],
                                      num_key_value_heads=meta["hkv"], hidden_size=meta["hidden"])


def _check_keep(got_keep, ref_keep, ref_scores, n_kept, n_sink=4):
    """Bit-exact keep set except keys within 1e-3 relative of the boundary."""
    s = np.asarray(ref_scores, np.float64).copy()
    s[:n_sink] = s.max() + 1
    boundary = np.sort(s)[::-1][n_kept - 1]
    near = np.abs(s - boundary) <= 1e-3 * abs(boundary)
    diff = np.setxor1d(got_keep, ref_keep)
    assert np.all(near[diff]), (diff, s[diff], boundary)
    return diff.size


def _scores_close(got, ref):
    err = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-3)
    assert err.max() < SCORE_TOL, err.max()


def _press(dev, meta):
    from core_b200 import press as P
    return P.load_core_prefill_decoding_press("tests/golden/core_indexer_hook.pt", device=str(dev),
                                              compression_ratio=meta["ratio"],
                                              decoding_compression_interval=meta["interval"])


def test_prefill_decoding_press_reproduces_reference_hooks():
    """Our COREPrefillDecodingPress, built by its factory from the reference's
    checkpoint, driven through the same forward hooks as the reference."""
    dev = _dev()
    d, meta = load_case(HOOK_CASE)
    hq, hkv, dd, L0 = meta["hq"], meta["hkv"], meta["d"], meta["L"]
    press = _press(dev, meta)
    mem_press = press.prefilling_press
    mem_press.base_press.capture_diagnostics = True
    q_proj = torch.nn.Linear(meta["hidden"], hq * dd, bias=False).to(dev, torch.bfloat16)
    o_proj = torch.nn.Linear(hq * dd, meta["hidden"], bias=False).to(dev, torch.bfloat16)
    with torch.no_grad():
        q_proj.weight.copy_(_bf16(d["q_proj"], dev))
        o_proj.weight.copy_(_bf16(d["o_proj"], dev))
    rot = hook_rotary(meta, dev)
    mods = [_Attention(l, q_proj, o_proj, rot, meta) for l in range(2)]
    events = hook_events(d, meta)
    got_events = []
    orig = mem_press.base_press.retain_metadata

    def retain(layer_idx, indices):
        got_events.append((int(layer_idx), indices[0].long().cpu().numpy(),
                           mem_press.base_press.diagnostic_scores[int(layer_idx)][0].numpy()))
        return orig(layer_idx, indices)

    mem_press.base_press.retain_metadata = retain
    press.reset_cache()
    press.begin_sequence(L0)
    press.set_token_ids(torch.from_numpy(d["token_ids0"]).to(dev))
    cache = SimpleNamespace(layers=[SimpleNamespace(keys=_bf16(d[f"k0_l{l}"], dev)[None],
                                                    values=_bf16(d[f"v0_l{l}"], dev)[None])
                                    for l in range(2)])
    hs0 = _bf16(d["hs_prefill"], dev)
    pos0 = torch.arange(L0, device=dev)[None]
    emb0 = rot(hs0, pos0)
    with torch.no_grad():
        for l in range(2):
            if l == 1:
                mods[1]._core_cached_query_states = _bf16(d["q_prefill_l1"], dev)[None]
            kw = dict(hidden_states=hs0, past_key_values=cache,
                      cache_position=torch.arange(L0, device=dev), position_ids=pos0,
                      position_embeddings=emb0)
            press.forward_hook(mods[l], [], kw, (torch.zeros(1, L0, meta["hidden"], device=dev,
                                                             dtype=torch.bfloat16), None))
            if hasattr(mods[l], "_core_cached_query_states"):
                del mods[l]._core_cached_query_states
        pos = L0
        n_diff_entries = 0
        for tok0, n in hook_decode_steps(d):
            pid = torch.arange(pos, pos + n, device=dev)[None]
            press.record_input_tokens(torch.from_numpy(d["decode_ids"][:, tok0:tok0 + n]).to(dev), pid)
            hs = _bf16(d["decode_hs"][:, tok0:tok0 + n], dev)
            emb = rot(hs, pid)
            for l in range(2):
                layer = cache.layers[l]
                layer.keys = torch.cat([layer.keys, _bf16(d["decode_k"][l][:, tok0:tok0 + n], dev)[None]], 2)
                layer.values = torch.cat([layer.values, _bf16(d["decode_v"][l][:, tok0:tok0 + n], dev)[None]], 2)
                phys = layer.keys.shape[2]
                kw = dict(hidden_states=hs, past_key_values=cache,
                          cache_position=torch.arange(phys - n, phys, device=dev), position_ids=pid,
                          position_embeddings=emb)
                attn = _bf16(d["decode_attn"][l, :, tok0:tok0 + n], dev)
                out = press.forward_hook(mods[l], [], kw, (attn, None))
                ref = d["decode_out"][l, 0, tok0:tok0 + n]
                diff = np.abs(out[0][0].float().cpu().numpy() - ref)
                assert diff.max() <= 2 ** -7 * np.abs(ref).max(), (tok0, l, diff.max())
                n_diff_entries += int((diff > 0).sum())
            pos += n
    from core_b200 import ops
    ops.status(dev)
    assert n_diff_entries <= 0.02 * d["decode_out"].size
    # every compression: same layer order, keep sets, scores
    assert len(got_events) == len(events)
    for (gl, gk, gs), (rl, rk, rs) in zip(got_events, events):
        assert gl == rl
        _scores_close(gs, rs)
        assert _check_keep(gk, rk, rs, meta["target"]) == 0, "a boundary key flipped"
    for l in range(2):
        assert torch.equal(cache.layers[l].keys[0].float().cpu(), torch.from_numpy(d[f"final_k_l{l}"]))
        assert torch.equal(cache.layers[l].values[0].float().cpu(), torch.from_numpy(d[f"final_v_l{l}"]))
        for name, got in (("M", mem_press._M[l]), ("b", mem_press._b[l])):
            ref = d[f"{name}_l{l}"]
            assert np.abs(got[0].cpu().numpy() - ref).max() <= STATE_TOL * np.abs(ref).max(), name
        assert abs(float(mem_press._Z[l][0]) - float(d[f"Z_l{l}"][0])) <= 1e-6


def test_memory_press_two_step_fixture():
    """COREMemoryPress.compress at prefill (question scope, r = 0.5), then the
    decoding press's compress back to the prefill budget, then readouts for
    one and three query tokens (the reference-written two-step fixture)."""
    from core_b200 import press as P
    dev = _dev()
    d, m = load_case(TWO_STEP_CASE)
    hq, hkv, L0, nq, hidden = m["hq"], m["hkv"], m["L"], m["nq"], m["hidden"]
    press = P.load_core_memory_press("tests/golden/core_indexer_two_step.pt", device=str(dev),
                                     compression_ratio=m["ratio"])
    press.base_press.prefill_qk_scope = "question"
    press.base_press.capture_diagnostics = True
    o_proj = torch.nn.Linear(hq * 128, hidden, bias=False).to(dev)
    with torch.no_grad():
        o_proj.weight.copy_(torch.from_numpy(d["o_proj"]).to(dev))
    mod = SimpleNamespace(layer_idx=m["layer"], o_proj=o_proj,
                          config=SimpleNamespace(num_attention_heads=hq, num_key_value_heads=hkv,
                                                 hidden_size=hidden))
    full_q = torch.zeros(1, hq, L0, 128, device=dev, dtype=torch.bfloat16)
    full_q[0, :, L0 - nq:] = _bf16(d["q"], dev)
    mod._core_cached_query_states = full_q
    press.set_query_boundary(L0 - nq)
    with torch.no_grad():
        k1, v1 = press.compress(mod, torch.zeros(1, L0, hidden, device=dev), _bf16(d["k"], dev)[None],
                                _bf16(d["v"], dev)[None], None, {})
    keep1 = press.base_press.diagnostic_keep_indices[m["layer"]][0].numpy()
    _scores_close(press.base_press.diagnostic_scores[m["layer"]][0].numpy(), d["scores1"])
    assert _check_keep(keep1, d["keep1"], d["scores1"], len(d["keep1"])) == 0
    for name in ("M1", "b1"):
        got = (press._M if name == "M1" else press._b)[m["layer"]][0].cpu().numpy()
        assert np.abs(got - d[name]).max() <= STATE_TOL * np.abs(d[name]).max()
    # decode: nq new tokens appended, recompressed to the prefill budget
    keys = torch.cat([k1, _bf16(d["k_new"], dev)[None]], dim=2)
    values = torch.cat([v1, _bf16(d["v_new"], dev)[None]], dim=2)
    dec = P.COREDecodingPress(base_press=press, compression_interval=nq, target_size=m["target"])
    mod._core_cached_query_states = _bf16(d["q1"], dev)[None]
    with torch.no_grad():
        k2, v2 = dec.compress(mod, torch.zeros(1, nq, hidden, device=dev), keys, values, None, {})
    keep2 = press.base_press.diagnostic_keep_indices[m["layer"]][0].numpy()
    _scores_close(press.base_press.diagnostic_scores[m["layer"]][0].numpy(), d["scores2"])
    assert _check_keep(keep2, d["keep2"], d["scores2"], m["target"]) == 0
    assert torch.equal(k2[0].float().cpu(), torch.from_numpy(d["out_k2"]))
    assert torch.equal(v2[0].float().cpu(), torch.from_numpy(d["out_v2"]))
    for name, st in (("M2", press._M), ("b2", press._b)):
        got = st[m["layer"]][0].cpu().numpy()
        assert np.abs(got - d[name]).max() <= STATE_TOL * np.abs(d[name]).max()
    assert abs(float(press._Z[m["layer"]][0]) - float(d["Z2"][0])) <= 1e-6
    for ql in (1, 3):
        mod._core_cached_query_states = _bf16(d[f"readout_q{ql}"], dev)[None]
        attn = _bf16(d[f"readout_attn{ql}"], dev)
        out = press.apply_memory_readout(mod, {"hidden_states": torch.zeros(1, ql, hidden, device=dev)},
                                         (attn, None))
        ref = d[f"readout_out{ql}"][0]
        diff = np.abs(out[0][0].float().cpu().numpy() - ref)
        assert (diff > 0).mean() < 0.02 and diff.max() <= 2 ** -7 * np.abs(ref).max()


def test_fp16_cache_keeps_its_own_values():
    """fp16 caches: the retained K/V are the original fp16 rows (no bf16
    round trip), and the memory write sees the fp16 values exactly."""
    from core_b200 import press as P
    dev = _dev()
    d, m = load_case(TWO_STEP_CASE)
    hq, hkv, L0, nq, hidden = m["hq"], m["hkv"], m["L"], m["nq"], m["hidden"]
    press = P.load_core_memory_press("tests/golden/core_indexer_two_step.pt", device=str(dev),
                                     compression_ratio=m["ratio"])
    press.base_press.prefill_qk_scope = "question"
    g = torch.Generator(device=dev).manual_seed(3)
    k = (torch.randn(1, hkv, L0, 128, device=dev, generator=g) / 11.3).half()
    v = torch.randn(1, hkv, L0, 128, device=dev, generator=g).half()
    full_q = torch.zeros(1, hq, L0, 128, device=dev, dtype=torch.float16)
    full_q[0, :, L0 - nq:] = (torch.randn(hq, nq, 128, device=dev, generator=g) / 11.3).half()
    mod = SimpleNamespace(layer_idx=m["layer"], _core_cached_query_states=full_q)
    press.set_query_boundary(L0 - nq)
    with torch.no_grad():
        ok, ov = press.compress(mod, torch.zeros(1, L0, hidden, device=dev), k, v, None, {})
    keep = press.base_press.cache_metadata.positions[m["layer"]][0]
    assert ok.dtype == torch.float16
    idx = keep[None, None, :, None].expand(1, hkv, -1, 128)
    assert torch.equal(ok, k.gather(2, idx)) and torch.equal(ov, v.gather(2, idx))
    # memory write on the fp16 values in f32 against the oracle
    from oracle import core_oracle as O
    from core_b200.checkpoint import load_checkpoint
    parts = load_checkpoint("tests/golden/core_indexer_two_step.pt")
    scores = press.base_press._cached_memory_scores[0].cpu().numpy()
    evict = np.ones(L0, bool)
    evict[keep.cpu().numpy()] = False
    M, b, Z = O.memory_write(k[0].float().cpu().numpy(), v[0].float().cpu().numpy(), scores, evict,
                             parts["memory"].params(m["layer"])[0].numpy(), groups=hq // hkv)
    got_M = press._M[m["layer"]][0].cpu().numpy()
    assert np.abs(got_M - M).max() <= 1e-4 * np.abs(M).max()
    assert abs(float(press._Z[m["layer"]][0]) - float(Z)) <= 1e-6


def test_fp16_readout_rounds_like_the_reference():
    """fp16 attention output: residual and o_proj product rounded to fp16,
    then the fp16 sum (kvpress_adapter.py:1320-1343), against the oracle's
    f64 arithmetic with the same roundings."""
    from core_b200 import engine, ops
    from oracle import core_oracle as O
    dev = _dev()
    d, m = load_case(TWO_STEP_CASE)
    hkv, hq = m["hkv"], m["hq"]
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)  # noqa: E731
    ofold = engine.fold_groups(f(d["o_proj"]), hkv, hq // hkv, 128)
    gate = (f(d["gate_w1"]), f(d["gate_b1"]), f(d["gate_w2"]).reshape(-1), f(d["gate_b2"]).reshape(-1))
    q = f(d["readout_q3"]).half()[None]
    attn = f(d["readout_attn3"]).half()
    out = ops.memory_readout(q, f(d["theta"]), gate, f(d["M2"])[None], f(d["b2"])[None], ofold,
                             attn.clone(), n_kv_heads=hkv)
    ops.status()
    qf = q[0].float().cpu().numpy()
    q_full = qf.transpose(1, 0, 2).reshape(qf.shape[1], -1)
    want = O.memory_readout(q_full, d["theta"], d["gate_w1"], d["gate_b1"], d["gate_w2"],
                            d["gate_b2"], d["M2"], d["b2"], ofold.cpu().numpy(),
                            attn[0].float().cpu().numpy(), out_dtype="f16")
    got = out[0].float().cpu().numpy()
    diff = np.abs(got - want)
    # equal up to one fp16 rounding of the residual sum on a few entries
    assert (diff > 0).mean() < 0.02 and diff.max() <= 2 ** -10 * np.abs(want).max(), diff.max()


def test_negative_gate_override_is_a_constant_gate():
    from core_b200 import engine, ops
    dev = _dev()
    d, m = load_case(TWO_STEP_CASE)
    hkv, hq = m["hkv"], m["hq"]
    f = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)  # noqa: E731
    ofold = engine.fold_groups(f(d["o_proj"]), hkv, hq // hkv, 128)
    gate = (f(d["gate_w1"]), f(d["gate_b1"]), f(d["gate_w2"]).reshape(-1), f(d["gate_b2"]).reshape(-1))
    q = f(d["readout_q1"])[None]
    zero = torch.zeros(1, 1, m["hidden"], device=dev)
    pos = ops.memory_readout(q, f(d["theta"]), gate, f(d["M2"])[None], f(d["b2"])[None], ofold,
                             zero.clone(), n_kv_heads=hkv, gate_override=0.5)
    neg = ops.memory_readout(q, f(d["theta"]), gate, f(d["M2"])[None], f(d["b2"])[None], ofold,
                             zero.clone(), n_kv_heads=hkv, gate_override=-0.5)
    ops.status()
    torch.testing.assert_close(neg, -pos, rtol=0, atol=0)
    with pytest.raises(ValueError):
        ops.memory_readout(q, f(d["theta"]), gate, f(d["M2"])[None], f(d["b2"])[None], ofold,
                           zero.clone(), n_kv_heads=hkv, gate_override=float("inf"))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("given", [False, True])
def test_rope_kernel_equals_transformers(dtype, given):
    """core_rope_queries against transformers' LlamaRotaryEmbedding +
    apply_rotary_pos_emb run on the same GPU, bit for bit."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    from core_b200 import ops
    dev = _dev()
    meta = dict(hidden=4096, hq=32, hkv=8, d=128, rope=dict(
        rope_type="llama3", rope_theta=500000.0, factor=8.0, low_freq_factor=1.0,
        high_freq_factor=4.0, original_max_position_embeddings=8192))
    rot = hook_rotary(meta, dev)
    g = torch.Generator(device=dev).manual_seed(4)
    B, T = 2, 130
    proj = torch.randn(B, T, 32 * 128, device=dev, generator=g).to(dtype)
    pos = (torch.arange(T, device=dev) + 16250)[None].expand(B, T)
    q = proj.view(B, T, 32, 128).transpose(1, 2)
    cos, sin = rot(q, pos)
    want, _ = apply_rotary_pos_emb(q, q, cos, sin)
    if given:
        got = ops.rope_queries(proj, 32, cos=cos, sin=sin)
    else:
        got = ops.rope_queries(proj, 32, positions=pos, inv_freq=rot.inv_freq,
                               attention_scaling=rot.attention_scaling)
    ops.status()
    if given or dtype != torch.float32:
        assert torch.equal(got, want.contiguous())
    else:  # f32 cos/sin from two implementations of cosf/sinf: a few ulps at most
        torch.testing.assert_close(got, want.contiguous(), rtol=2e-6, atol=1e-6)
