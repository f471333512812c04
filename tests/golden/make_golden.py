"""Generate the golden fixtures by running the reference CORE press on CPU.

This script is the only place in the repository that executes the reference
implementation.  It imports the reference from its source tree (default
``/root/reference``; override with ``CORE_REFERENCE_ROOT``), builds seeded
synthetic inputs and a random-init indexer / memory stack, calls the
reference's own ``COREMemoryPress.compress`` (``core/kvpress_adapter.py:968-1210``),
``COREDecodingPress.compress`` (``kvpress/kvpress/presses/decoding_press.py:71-115``)
and ``COREMemoryPress.apply_memory_readout`` (``core/kvpress_adapter.py:1212-1352``),
and stores inputs, weights and outputs as ``tests/golden/<case>.npz``.

Only ``fire`` is missing from the image; a one-line stub is written to a
temporary directory and put on ``sys.path`` (the reference tree is untouched).

Run:  python tests/golden/make_golden.py            (about a minute on CPU)
"""

from __future__ import annotations

import os
import sys
import tempfile
from pathlib import Path
from types import SimpleNamespace

import numpy as np

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("CORE_REFERENCE_ROOT", "/root/reference"))


def _import_reference():
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


def main():
    ref = _import_reference()
    import torch
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, kw in CASES:
        res, meta = run_compress_case(ref, name, **kw)
        np.savez_compressed(HERE / f"{name}.npz", meta=np.array(repr(meta)),
                            **pack(res, meta, readout=False))
        print("wrote", name, {k: getattr(v, "shape", None) for k, v in res.items()
                              if k in ("features", "keep", "M")})
    res, meta = run_two_step_case(ref, "bf16_two_step_L384_Q64", seed=6)
    save_reference_checkpoint(ref, seed=6, out=HERE / "core_indexer_two_step.pt")
    np.savez_compressed(HERE / "bf16_two_step_L384_Q64.npz", meta=np.array(repr(meta)),
                        **pack(res, meta, readout=True))
    print("wrote two-step", res["keep1"].shape, res["keep2"].shape)


if __name__ == "__main__":
    main()
