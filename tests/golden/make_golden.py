"""Generate the golden fixtures by running the reference CORE press on CPU.

This script is the only place in the repository that executes the reference
implementation.  It imports the reference from the source tree named by the
``CORE_REFERENCE_ROOT`` environment variable (required), builds seeded
synthetic inputs and a random-init indexer / memory stack, calls the
reference's own ``COREMemoryPress.compress`` (``core/kvpress_adapter.py:968-1210``),
``COREDecodingPress.compress`` (``kvpress/kvpress/presses/decoding_press.py:71-115``)
and ``COREMemoryPress.apply_memory_readout`` (``core/kvpress_adapter.py:1212-1352``),
and stores inputs, weights and outputs as ``tests/golden/<case>.npz``.

Only ``fire`` is missing from the image; a one-line stub is written to a
temporary directory and put on ``sys.path`` (the reference tree is untouched).

The hook case (``bf16_hook_decode_L256``) drives the reference's own
``COREPrefillDecodingPress`` forward hooks -- prefill compression, decode
steps with the memory readout, decode recompressions scored with queries the
press rebuilds through q_proj and transformers' RoPE -- over a stand-in
attention module and cache, and also writes the checkpoint it used
(``core_indexer_hook.pt``) with the reference's ``save_indexer_stack``.

Run:  CORE_REFERENCE_ROOT=<reference checkout> python tests/golden/make_golden.py
(about a minute on CPU)
"""

from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path
from types import SimpleNamespace

import numpy as np

HERE = Path(__file__).resolve().parent
def _reference_root() -> Path:
    root = os.environ.get("CORE_REFERENCE_ROOT")
    if not root:
        raise SystemExit("set CORE_REFERENCE_ROOT to the reference checkout")
    return Path(root)


def _import_reference():
    REF = _reference_root()
    stub = Path(tempfile.mkdtemp(prefix="core_ref_stub_"))
    (stub / "fire.py").write_text("def Fire(*args, **kwargs):\n    return None\n")
    for p in (str(REF / "kvpress"), str(REF), str(stub)):
        if p not in sys.path:
            sys.path.insert(0, p)
    import torch  # noqa: F401
    from core import kvpress_adapter as ka
    from core.config import COREConfig
    from core.features import COREFeatureExtractor
    from core.indexer import COREIndexerStack, MemoryModuleStack
    return ka, COREConfig, COREFeatureExtractor, COREIndexerStack, MemoryModuleStack


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round float32 to bfloat16 (nearest-even) and return the uint16 bits."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))
    return (r >> np.uint32(16)).astype(np.uint16)


def bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << np.uint32(16)).view(np.float32)


def gaussian_outliers(rng, heads, n, d, outlier_idx, scale=8.0):
    """N(0,1)/sqrt(d) with four fixed outlier channels per head scaled by 8."""
    x = rng.standard_normal((heads, n, d), dtype=np.float32) / np.float32(np.sqrt(d))
    for h in range(heads):
        x[h, :, outlier_idx[h]] *= np.float32(scale)
    return x


def make_inputs(rng, hkv, hq, d, L, nq, dtype):
    groups = hq // hkv
    out_idx = np.stack([rng.choice(d, 4, replace=False) for _ in range(hkv)])
    k = gaussian_outliers(rng, hkv, L, d, out_idx)
    q = gaussian_outliers(rng, hq, nq, d, np.repeat(out_idx, groups, axis=0))
    v = rng.standard_normal((hkv, L, d), dtype=np.float32)
    if dtype == "bfloat16":
        q, k, v = (bits_to_f32(bf16_bits(a)) for a in (q, k, v))
    return q, k, v, out_idx


class Capture:
    def __init__(self):
        self.indices = None


def build_press(ref, *, seed, n_layers, hkv, hq, d, d_mem, gate_hidden, hidden,
                ratio, dtype, scope):
    ka, COREConfig, COREFeatureExtractor, COREIndexerStack, MemoryModuleStack = ref
    import torch

    torch.manual_seed(seed)
    indexer = COREIndexerStack(n_layers, 14, 128)
    memory = MemoryModuleStack(n_layers, hq * d, d_mem, gate_hidden)
    o_proj = torch.nn.Linear(hq * d, hidden, bias=False)
    q_proj = torch.nn.Linear(hidden, hq * d, bias=False)
    cfg = COREConfig(n_layers=n_layers, n_kv_heads=hkv, n_q_heads=hq, head_dim=d,
                     hidden_size=hidden, dtype=dtype, memory_dim=d_mem,
                     memory_gate_hidden=gate_hidden, geometry_seed=42)
    fe = COREFeatureExtractor(cfg)
    scorer = ka.COREScorerPress(
        indexer=indexer, feature_extractor=fe, compression_ratio=ratio,
        student_temp=1.0, use_indexer_stack=True, scoring_layer_idx=-1,
        n_sink_protect=4, prefill_qk_scope=scope, capture_diagnostics=True,
    )
    press = ka.COREMemoryPress(base_press=scorer, memory_module=memory,
                               memory_decay=0.9, memory_write_eta=1.0)
    cap = Capture()
    orig = scorer.retain_metadata

    def retain(layer_idx, indices):
        cap.indices = indices.clone()
        return orig(layer_idx, indices)

    scorer.retain_metadata = retain
    return press, scorer, indexer, memory, fe, o_proj, q_proj, cap


def weights_dict(indexer, memory, fe, o_proj, layer):
    w = {}
    mlp = indexer[layer].net
    w["mlp_w1"] = mlp[0].weight.detach().numpy()
    w["mlp_b1"] = mlp[0].bias.detach().numpy()
    w["mlp_w2"] = mlp[2].weight.detach().numpy()
    w["mlp_b2"] = mlp[2].bias.detach().numpy()
    w["mlp_w3"] = mlp[4].weight.detach().numpy()
    w["mlp_b3"] = mlp[4].bias.detach().numpy()
    mm = memory[layer]
    w["theta"] = mm.theta_dense_weight().detach().numpy()
    w["gate_w1"] = mm.gate[0].weight.detach().numpy()
    w["gate_b1"] = mm.gate[0].bias.detach().numpy()
    w["gate_w2"] = mm.gate[2].weight.detach().numpy()
    w["gate_b2"] = mm.gate[2].bias.detach().numpy()
    w["geometry"] = fe.key_geometry.weight[layer].detach().numpy()
    w["prototypes"] = fe.prototype_bank.prototypes.detach().numpy()
    w["hadamard"] = fe.hadamard.R.detach().numpy()
    w["o_proj"] = o_proj.weight.detach().numpy()
    return w


def to_torch(a, dtype):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.to(torch.bfloat16) if dtype == "bfloat16" else t


def run_compress_case(ref, name, *, seed, hkv, hq, d, L, nq, ratio, dtype, scope,
                      d_mem=64, gate_hidden=64, hidden=128, layer=1):
    import torch
    rng = np.random.default_rng(seed)
    q, k, v, out_idx = make_inputs(rng, hkv, hq, d, L, nq, dtype)
    press, scorer, indexer, memory, fe, o_proj, q_proj, cap = build_press(
        ref, seed=seed, n_layers=2, hkv=hkv, hq=hq, d=d, d_mem=d_mem,
        gate_hidden=gate_hidden, hidden=hidden, ratio=ratio, dtype=dtype, scope=scope)
    keys = to_torch(k, dtype)[None]
    values = to_torch(v, dtype)[None]
    prefill = scope in ("question", "all") and nq <= L
    if scope == "question":
        full_q = np.zeros((hq, L, d), np.float32)
        full_q[:, L - nq:] = q
        cached_q = to_torch(full_q, dtype)[None]
        scorer.set_query_boundary(L - nq)
        hs = torch.zeros(1, L, hidden)
    elif scope == "all":
        assert nq == L
        cached_q = to_torch(q, dtype)[None]
        hs = torch.zeros(1, L, hidden)
    else:  # decode branch: hidden states hold only the buffered queries
        cached_q = to_torch(q, dtype)[None]
        hs = torch.zeros(1, nq, hidden)
        prefill = False
    module = SimpleNamespace(layer_idx=layer, q_proj=q_proj, o_proj=o_proj,
                             config=SimpleNamespace(num_attention_heads=hq,
                                                    num_key_value_heads=hkv,
                                                    hidden_size=hidden),
                             _core_cached_query_states=cached_q)
    with torch.no_grad():
        out_k, out_v = press.compress(module, hs, keys, values, None, {})
    res = dict(
        q=q, k=k, v=v, outlier_idx=out_idx,
        features=scorer.diagnostic_features[layer].numpy(),
        scores=scorer.diagnostic_scores[layer].numpy()[0],
        keep=cap.indices.numpy()[0],
        out_k=out_k.float().numpy()[0], out_v=out_v.float().numpy()[0],
        M=press._M[layer].numpy()[0], b=press._b[layer].numpy()[0],
        Z=press._Z[layer].numpy(),
    )
    res.update(weights_dict(indexer, memory, fe, o_proj, layer))
    meta = dict(name=name, seed=seed, hkv=hkv, hq=hq, d=d, L=L, nq=nq, ratio=ratio,
                dtype=dtype, scope=scope, prefill=int(prefill), d_mem=d_mem,
                gate_hidden=gate_hidden, hidden=hidden, layer=layer, n_sink=4,
                gamma=0.9, eta=1.0, tau=1.0, rho=0.1)
    return res, meta


def run_two_step_case(ref, name, *, seed, hkv=2, hq=8, d=128, L0=384, nq=64,
                      ratio=0.5, dtype="bfloat16", d_mem=64, gate_hidden=64,
                      hidden=128, layer=1):
    """Prefill compression, one decode recompression, then two readouts."""
    import torch
    ka = ref[0]
    rng = np.random.default_rng(seed)
    q0, k0, v0, out_idx = make_inputs(rng, hkv, hq, d, L0, nq, dtype)
    press, scorer, indexer, memory, fe, o_proj, q_proj, cap = build_press(
        ref, seed=seed, n_layers=2, hkv=hkv, hq=hq, d=d, d_mem=d_mem,
        gate_hidden=gate_hidden, hidden=hidden, ratio=ratio, dtype=dtype,
        scope="question")
    full_q = np.zeros((hq, L0, d), np.float32)
    full_q[:, L0 - nq:] = q0
    scorer.set_query_boundary(L0 - nq)
    module = SimpleNamespace(layer_idx=layer, q_proj=q_proj, o_proj=o_proj,
                             config=SimpleNamespace(num_attention_heads=hq,
                                                    num_key_value_heads=hkv,
                                                    hidden_size=hidden),
                             _core_cached_query_states=to_torch(full_q, dtype)[None])
    with torch.no_grad():
        k1, v1 = press.compress(module, torch.zeros(1, L0, hidden),
                                to_torch(k0, dtype)[None], to_torch(v0, dtype)[None],
                                None, {})
    step1 = dict(features1=scorer.diagnostic_features[layer].numpy(),
                 scores1=scorer.diagnostic_scores[layer].numpy()[0],
                 keep1=cap.indices.numpy()[0],
                 M1=press._M[layer].numpy()[0].copy(), b1=press._b[layer].numpy()[0].copy(),
                 Z1=press._Z[layer].numpy().copy())
    n_kept0 = k1.shape[2]
    # Decode: append nq new tokens and recompress back to the retained budget.
    q1, k_new, v_new, _ = make_inputs(rng, hkv, hq, d, nq, nq, dtype)
    keys = torch.cat([k1, to_torch(k_new, dtype)[None]], dim=2)
    values = torch.cat([v1, to_torch(v_new, dtype)[None]], dim=2)
    dec = ka.COREDecodingPress(base_press=press, compression_interval=nq,
                               target_size=n_kept0)
    module._core_cached_query_states = to_torch(q1, dtype)[None]
    with torch.no_grad():
        k2, v2 = dec.compress(module, torch.zeros(1, nq, hidden), keys, values, None, {})
    step2 = dict(q1=q1, k_new=k_new, v_new=v_new,
                 features2=scorer.diagnostic_features[layer].numpy(),
                 scores2=scorer.diagnostic_scores[layer].numpy()[0],
                 keep2=cap.indices.numpy()[0],
                 M2=press._M[layer].numpy()[0], b2=press._b[layer].numpy()[0],
                 Z2=press._Z[layer].numpy(),
                 out_k2=k2.float().numpy()[0], out_v2=v2.float().numpy()[0])
    # Readouts for a single decoded token and for a three-token forward.
    readouts = {}
    for q_len in (1, 3):
        qr = gaussian_outliers(rng, hq, q_len, d, np.repeat(out_idx, hq // hkv, axis=0))
        attn = rng.standard_normal((1, q_len, hidden), dtype=np.float32)
        if dtype == "bfloat16":
            qr = bits_to_f32(bf16_bits(qr))
            attn = bits_to_f32(bf16_bits(attn))
        module._core_cached_query_states = to_torch(qr, dtype)[None]
        kwargs = {"hidden_states": torch.zeros(1, q_len, hidden)}
        with torch.no_grad():
            out = press.apply_memory_readout(module, kwargs, (to_torch(attn, dtype), None))
        readouts[f"readout_q{q_len}"] = qr
        readouts[f"readout_attn{q_len}"] = attn
        readouts[f"readout_out{q_len}"] = out[0].float().numpy()
    res = dict(q=q0, k=k0, v=v0, outlier_idx=out_idx, **step1, **step2, **readouts)
    res.update(weights_dict(indexer, memory, fe, o_proj, layer))
    meta = dict(name=name, seed=seed, hkv=hkv, hq=hq, d=d, L=L0, nq=nq, ratio=ratio,
                dtype=dtype, scope="question", prefill=1, d_mem=d_mem,
                gate_hidden=gate_hidden, hidden=hidden, layer=layer, n_sink=4,
                gamma=0.9, eta=1.0, tau=1.0, rho=0.1, target=n_kept0)
    return res, meta


def save_reference_checkpoint(ref, *, seed, out, hkv=2, hq=8, d=128, d_mem=64, gate_hidden=64,
                              hidden=128):
    """The two-step case's stacks written by the reference's own save_indexer_stack
    (core/train.py:2982-3047), for the checkpoint-format tests."""
    import shutil
    import torch
    from core.train import save_indexer_stack
    press, scorer, indexer, memory, fe, o_proj, q_proj, cap = build_press(
        ref, seed=seed, n_layers=2, hkv=hkv, hq=hq, d=d, d_mem=d_mem, gate_hidden=gate_hidden,
        hidden=hidden, ratio=0.5, dtype="bfloat16", scope="question")
    cfg = fe.config
    cfg.n_sink_protect = 4
    cfg.compression_ratio = 0.5
    cfg.prefill_qk_scope = "question"
    cfg.span_selection_mode = "tokenwise"
    tmp = Path(tempfile.mkdtemp(prefix="core_ckpt_"))
    cfg.output_dir = str(tmp)
    save_indexer_stack(indexer, cfg, history=[], feature_extractor=fe, memory_module=memory)
    shutil.copy(tmp / "indexer" / "core_indexer.pt", out)


class _HookAttention:
    """Stand-in for a Llama attention module as the press hooks see it."""

    def __init__(self, layer_idx, q_proj, o_proj, rotary, hq, hkv, hidden, d):
        from types import SimpleNamespace
        self.layer_idx = layer_idx
        self.q_proj = q_proj
        self.o_proj = o_proj
        self.rotary_emb = rotary
        self.head_dim = d
        self.config = SimpleNamespace(num_attention_heads=hq, num_key_value_heads=hkv,
                                      hidden_size=hidden)


HOOK_ROPE = {"rope_type": "llama3", "rope_theta": 500000.0, "factor": 8.0, "low_freq_factor": 1.0,
             "high_freq_factor": 4.0, "original_max_position_embeddings": 8192}


def run_hook_case(ref, name, *, seed, hkv=2, hq=8, d=128, L0=256, ratio=0.5, interval=16,
                  n_decode=36, multi_at=20, d_mem=64, gate_hidden=64, hidden=256):
    """Prefill + decode through the reference's COREPrefillDecodingPress hooks.

    Two layers.  Layer 0's prefill queries are rebuilt by the press from the
    hidden states (q_proj + RoPE with the forward's position embeddings);
    layer 1's come from ``_core_cached_query_states``.  Decode forwards carry
    one token, except one 3-token forward at step ``multi_at``; every decode
    forward gets the memory readout, and the press recompresses each layer to
    the prefill budget every ``interval`` forwards with queries it rebuilds
    at their absolute positions."""
    import torch
    from transformers import LlamaConfig
    from transformers.models.llama.modeling_llama import LlamaRotaryEmbedding
    ka = ref[0]
    rng = np.random.default_rng(seed)
    press, scorer, indexer, memory, fe, o_proj, q_proj, cap = build_press(
        ref, seed=seed, n_layers=2, hkv=hkv, hq=hq, d=d, d_mem=d_mem, gate_hidden=gate_hidden,
        hidden=hidden, ratio=ratio, dtype="bfloat16", scope="all")
    q_proj = q_proj.to(torch.bfloat16)
    o_proj = o_proj.to(torch.bfloat16)
    cfg = LlamaConfig(hidden_size=hidden, num_attention_heads=hq, num_key_value_heads=hkv,
                      head_dim=d, max_position_embeddings=131072, rope_parameters=dict(HOOK_ROPE))
    rotary = LlamaRotaryEmbedding(cfg)
    mods = [_HookAttention(l, q_proj, o_proj, rotary, hq, hkv, hidden, d) for l in range(2)]
    decoding = ka.COREDecodingPress(base_press=press, compression_interval=interval, target_size=1)
    combo = ka.COREPrefillDecodingPress(prefilling_press=press, decoding_press=decoding)
    combo.begin_sequence(L0)
    ids = rng.integers(5, 30000, size=(1, L0))
    combo.set_token_ids(torch.from_numpy(ids))

    events = []
    orig = scorer.retain_metadata

    def retain(layer_idx, indices):
        events.append((int(layer_idx), indices.numpy()[0].copy(),
                       scorer.diagnostic_scores[int(layer_idx)].numpy()[0].copy()))
        return orig(layer_idx, indices)

    scorer.retain_metadata = retain

    def bf(a):
        return torch.from_numpy(bits_to_f32(bf16_bits(a))).to(torch.bfloat16)

    out_idx = np.stack([rng.choice(d, 4, replace=False) for _ in range(hkv)])
    caches = []
    res = {"token_ids0": ids}
    for l in range(2):
        k = gaussian_outliers(rng, hkv, L0, d, out_idx)
        v = rng.standard_normal((hkv, L0, d), dtype=np.float32)
        res[f"k0_l{l}"], res[f"v0_l{l}"] = bits_to_f32(bf16_bits(k)), bits_to_f32(bf16_bits(v))
        caches.append((bf(k)[None], bf(v)[None]))
    from types import SimpleNamespace
    cache = SimpleNamespace(layers=[SimpleNamespace(keys=k, values=v) for k, v in caches])
    hs0 = rng.standard_normal((1, L0, hidden), dtype=np.float32)
    res["hs_prefill"] = bits_to_f32(bf16_bits(hs0))
    pos0 = torch.arange(L0)[None]
    hs0_t = bf(hs0)
    q_full = gaussian_outliers(rng, hq, L0, d, np.repeat(out_idx, hq // hkv, axis=0))
    res["q_prefill_l1"] = bits_to_f32(bf16_bits(q_full))
    with torch.no_grad():
        emb = rotary(hs0_t, pos0)
        for l in range(2):
            kwargs = dict(hidden_states=hs0_t, past_key_values=cache, cache_position=torch.arange(L0),
                          position_ids=pos0, position_embeddings=emb)
            if l == 1:
                mods[l]._core_cached_query_states = bf(q_full)[None]
            attn = bf(rng.standard_normal((1, L0, hidden), dtype=np.float32))
            combo.forward_hook(mods[l], [], kwargs, (attn, None))
            if hasattr(mods[l], "_core_cached_query_states"):
                del mods[l]._core_cached_query_states
    res["n_prefill_events"] = np.array(len(events))
    pos = L0
    decode_hs, decode_attn, decode_out, decode_k, decode_v, decode_ids = [], [], [], [], [], []
    with torch.no_grad():
        for step in range(n_decode):
            n_tok = 3 if step == multi_at else 1
            new_ids = rng.integers(5, 30000, size=(1, n_tok))
            pid = torch.arange(pos, pos + n_tok)[None]
            combo.record_input_tokens(torch.from_numpy(new_ids), pid)
            hs = rng.standard_normal((1, n_tok, hidden), dtype=np.float32)
            hs_t = bf(hs)
            emb = rotary(hs_t, pid)
            decode_hs.append(bits_to_f32(bf16_bits(hs)))
            decode_ids.append(new_ids)
            step_k, step_v, step_attn, step_out = [], [], [], []
            for l in range(2):
                kn = gaussian_outliers(rng, hkv, n_tok, d, out_idx)
                vn = rng.standard_normal((hkv, n_tok, d), dtype=np.float32)
                layer = cache.layers[l]
                layer.keys = torch.cat([layer.keys, bf(kn)[None]], dim=2)
                layer.values = torch.cat([layer.values, bf(vn)[None]], dim=2)
                phys = layer.keys.shape[2]
                kwargs = dict(hidden_states=hs_t, past_key_values=cache,
                              cache_position=torch.arange(phys - n_tok, phys), position_ids=pid,
                              position_embeddings=emb)
                attn = rng.standard_normal((1, n_tok, hidden), dtype=np.float32)
                out = combo.forward_hook(mods[l], [], kwargs, (bf(attn), None))
                step_k.append(bits_to_f32(bf16_bits(kn)))
                step_v.append(bits_to_f32(bf16_bits(vn)))
                step_attn.append(bits_to_f32(bf16_bits(attn)))
                step_out.append(out[0].float().numpy())
            decode_k.append(np.stack(step_k))
            decode_v.append(np.stack(step_v))
            decode_attn.append(np.stack(step_attn))
            decode_out.append(np.stack(step_out))
            pos += n_tok
    # ragged decode entries (the 3-token forward) are stored concatenated along tokens
    res["decode_tokens"] = np.array([x.shape[1] for x in decode_hs])
    res["decode_hs"] = np.concatenate(decode_hs, axis=1)
    res["decode_ids"] = np.concatenate(decode_ids, axis=1)
    res["decode_k"] = np.concatenate(decode_k, axis=2)        # (2 layers, hkv, T, d)
    res["decode_v"] = np.concatenate(decode_v, axis=2)
    res["decode_attn"] = np.concatenate(decode_attn, axis=2)  # (2, 1, T, hidden)
    res["decode_out"] = np.concatenate(decode_out, axis=2)
    res["event_layer"] = np.array([e[0] for e in events])
    res["event_len"] = np.array([len(e[2]) for e in events])
    res["event_keep"] = np.concatenate([e[1] for e in events])
    res["event_scores"] = np.concatenate([e[2] for e in events])
    for l in range(2):
        res[f"final_k_l{l}"] = cache.layers[l].keys.float().numpy()[0]
        res[f"final_v_l{l}"] = cache.layers[l].values.float().numpy()[0]
        res[f"M_l{l}"] = press._M[l].numpy()[0]
        res[f"b_l{l}"] = press._b[l].numpy()[0]
        res[f"Z_l{l}"] = press._Z[l].numpy()
    res["q_proj"] = q_proj.weight.detach().float().numpy()
    res["o_proj"] = o_proj.weight.detach().float().numpy()
    meta = dict(name=name, seed=seed, hkv=hkv, hq=hq, d=d, L=L0, ratio=ratio, interval=interval,
                n_decode=n_decode, multi_at=multi_at, d_mem=d_mem, gate_hidden=gate_hidden,
                hidden=hidden, dtype="bfloat16", scope="all", rope=dict(HOOK_ROPE),
                target=int(decoding.target_size), n_sink=4)
    return res, meta, (indexer, memory, fe)


def save_checkpoint_of(ref, stacks, out, *, ratio, scope):
    """``stacks`` = (indexer, memory, feature extractor) written by the
    reference's own save_indexer_stack (core/train.py:2982-3047)."""
    import shutil
    from core.train import save_indexer_stack
    indexer, memory, fe = stacks
    cfg = fe.config
    cfg.n_sink_protect = 4
    cfg.compression_ratio = ratio
    cfg.prefill_qk_scope = scope
    cfg.span_selection_mode = "tokenwise"
    tmp = Path(tempfile.mkdtemp(prefix="core_ckpt_"))
    cfg.output_dir = str(tmp)
    save_indexer_stack(indexer, cfg, history=[], feature_extractor=fe, memory_module=memory)
    shutil.copy(tmp / "indexer" / "core_indexer.pt", out)


CASES = [
    ("fp32_decode_L512_Q64", dict(seed=0, hkv=2, hq=8, d=128, L=512, nq=64,
                                  ratio=0.75, dtype="float32", scope="decode")),
    ("bf16_prefillq_L640_Q128", dict(seed=1, hkv=2, hq=8, d=128, L=640, nq=128,
                                     ratio=0.75, dtype="bfloat16", scope="question")),
    ("bf16_decode_ragged_L333_Q40", dict(seed=2, hkv=2, hq=8, d=128, L=333, nq=40,
                                         ratio=0.6, dtype="bfloat16", scope="decode")),
    ("bf16_prefill_all_L96", dict(seed=3, hkv=1, hq=4, d=128, L=96, nq=96,
                                  ratio=0.5, dtype="bfloat16", scope="all")),
    ("bf16_tiny_L5", dict(seed=4, hkv=1, hq=4, d=128, L=5, nq=5, ratio=0.75,
                          dtype="bfloat16", scope="all")),
    ("bf16_llama_heads_L256_Q32", dict(seed=5, hkv=8, hq=32, d=128, L=256, nq=32,
                                       ratio=0.75, dtype="bfloat16", scope="decode")),
]


BF16_INPUTS = ("q", "k", "v", "q1", "k_new", "v_new", "out_k", "out_v", "out_k2",
               "out_v2", "readout_q1", "readout_q3", "readout_attn1",
               "readout_attn3", "readout_out1", "readout_out3")
HOOK_BF16 = ("hs_prefill", "q_prefill_l1", "k0_l0", "v0_l0", "k0_l1", "v0_l1", "decode_hs",
             "decode_k", "decode_v", "decode_attn", "decode_out", "final_k_l0", "final_v_l0",
             "final_k_l1", "final_v_l1", "q_proj", "o_proj")
READOUT_ONLY = ("gate_w1", "gate_b1", "gate_w2", "gate_b2", "o_proj")


def pack(res, meta, readout):
    """bf16-exact arrays are stored as their uint16 bit patterns."""
    out = {}
    for key, val in res.items():
        if key in READOUT_ONLY and not readout:
            continue
        if meta["dtype"] == "bfloat16" and key in BF16_INPUTS:
            val = bf16_bits(val)
        out[key] = val
    return out


def main(only=None):
    """Write every fixture, or only those whose name contains one of ``only``."""
    ref = _import_reference()
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))

    def wanted(name):
        return not only or any(o in name for o in only)

    for name, kw in CASES:
        if not wanted(name):
            continue
        res, meta = run_compress_case(ref, name, **kw)
        np.savez_compressed(HERE / f"{name}.npz", meta=np.array(repr(meta)),
                            **pack(res, meta, readout=False))
        print("wrote", name, {k: getattr(v, "shape", None) for k, v in res.items()
                              if k in ("features", "keep", "M")})
    if wanted("bf16_two_step_L384_Q64"):
        res, meta = run_two_step_case(ref, "bf16_two_step_L384_Q64", seed=6)
        save_reference_checkpoint(ref, seed=6, out=HERE / "core_indexer_two_step.pt")
        np.savez_compressed(HERE / "bf16_two_step_L384_Q64.npz", meta=np.array(repr(meta)),
                            **pack(res, meta, readout=True))
        print("wrote two-step", res["keep1"].shape, res["keep2"].shape)
    if not wanted("bf16_hook_decode_L256"):
        return
    res, meta, stacks = run_hook_case(ref, "bf16_hook_decode_L256", seed=9)
    save_checkpoint_of(ref, stacks, HERE / "core_indexer_hook.pt", ratio=meta["ratio"],
                       scope=meta["scope"])
    np.savez_compressed(HERE / "bf16_hook_decode_L256.npz", meta=np.array(repr(meta)),
                        **{k: (bf16_bits(v) if k in HOOK_BF16 else v) for k, v in res.items()})
    print("wrote hook case", len(res["event_layer"]), "compressions")


if __name__ == "__main__":
    main(sys.argv[1:])
