"""The oracle replays the reference's hook-level fixture (prefill compression,
decode readouts, decode recompressions with rebuilt queries) and agrees with
what the reference's own COREPrefillDecodingPress wrote.  CPU only.

The replay follows the reference's order of work inside a decode forward
(kvpress/kvpress/presses/decoding_press.py:117-188): readout with the memory
written before this forward, then buffering, then (when the interval is
complete) a recompression scored by every buffered query, rebuilt by q_proj
and RoPE at its absolute position (core/kvpress_adapter.py:469-519,
core/collector.py:135-201).
"""

import numpy as np
import torch

from helpers import HOOK_CASE, hook_decode_steps, hook_events, hook_rotary, load_case
from oracle import core_oracle as O

CKPT = "tests/golden/core_indexer_hook.pt"


def _weights(layer):
    from core_b200.checkpoint import load_checkpoint
    parts = load_checkpoint(CKPT)
    fe, mem = parts["geometry"], parts["memory"]
    mlp = tuple(t.numpy() for t in parts["indexer"].params(layer))
    th, gw1, gb1, gw2, gb2 = (t.numpy() for t in mem.params(layer))
    lw = O.LayerWeights(mlp=mlp, geometry=fe.weight[layer].numpy(),
                        prototypes=fe.prototypes_for(layer).numpy(), hadamard=fe.hadamard.numpy(),
                        theta=th)
    return lw, (gw1, gb1, gw2[None], gb2)


def rope_queries_torch(hs, q_proj, rot, meta, positions=None, emb=None):
    """The reference's own query rebuild on the CPU (bf16 q_proj, transformers RoPE)."""
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    x = torch.from_numpy(hs).to(torch.bfloat16)
    w = torch.from_numpy(q_proj).to(torch.bfloat16)
    t = x.shape[1]
    q = torch.nn.functional.linear(x, w).view(1, t, meta["hq"], meta["d"]).transpose(1, 2)
    if emb is None:
        emb = rot(q, torch.from_numpy(np.asarray(positions))[None])
    q, _ = apply_rotary_pos_emb(q, q, *emb)
    return q[0].float().numpy()  # (Hq, T, d)


def replay(d, meta):
    """Yields ("event", i, out) per compression and ("readout", layer, tok0, n, out)."""
    rot = hook_rotary(meta)
    hq, hkv, dd, target = meta["hq"], meta["hkv"], meta["d"], meta["target"]
    weights = [_weights(l) for l in range(2)]
    o_fold = O.fold_groups(d["o_proj"], hkv, hq // hkv, dd)
    caches, positions, nxt, mem = {}, {}, {}, {}
    L0 = meta["L"]
    emb0 = rot(torch.from_numpy(d["hs_prefill"]).to(torch.bfloat16), torch.arange(L0)[None])
    ev = 0
    for layer in range(2):
        if layer == 0:
            q = rope_queries_torch(d["hs_prefill"], d["q_proj"], rot, meta, emb=emb0)
        else:
            q = d["q_prefill_l1"]
        out = O.compress_layer(q, d[f"k0_l{layer}"], d[f"v0_l{layer}"], weights[layer][0],
                               compression_ratio=meta["ratio"], is_prefill=True,
                               positions=np.arange(L0), seq_len=L0, round_bf16=True)
        yield ("event", ev, out)
        ev += 1
        caches[layer] = (out["out_k"], out["out_v"])
        positions[layer] = np.arange(L0)[out["keep"]]
        nxt[layer] = L0
        mem[layer] = (out["M"], out["b"], out["Z"])
    window = {0: [], 1: []}
    steps = {0: 0, 1: 0}
    pos = L0
    for tok0, n in hook_decode_steps(d):
        hs = d["decode_hs"][:, tok0:tok0 + n]
        pid = np.arange(pos, pos + n)
        emb = rot(torch.from_numpy(hs).to(torch.bfloat16), torch.from_numpy(pid)[None])
        for layer in range(2):
            k, v = caches[layer]
            k = np.concatenate([k, d["decode_k"][layer][:, tok0:tok0 + n]], axis=1)
            v = np.concatenate([v, d["decode_v"][layer][:, tok0:tok0 + n]], axis=1)
            positions[layer] = np.concatenate([positions[layer], np.arange(nxt[layer], nxt[layer] + n)])
            nxt[layer] += n
            q = rope_queries_torch(hs, d["q_proj"], rot, meta, emb=emb)
            q_full = q.transpose(1, 0, 2).reshape(n, hq * dd)
            gate = weights[layer][1]
            M, b, _ = mem[layer]
            ro = O.memory_readout(q_full, weights[layer][0].theta, gate[0], gate[1], gate[2],
                                  gate[3], M, b, o_fold, d["decode_attn"][layer, 0, tok0:tok0 + n])
            yield ("readout", layer, tok0, n, ro)
            window[layer].append(hs)
            steps[layer] += 1
            if steps[layer] >= meta["interval"] or n >= target:
                buf = np.concatenate(window[layer], axis=1)
                T = buf.shape[1]
                qpos = np.arange(pid[-1] - T + 1, pid[-1] + 1)
                qb = rope_queries_torch(buf, d["q_proj"], rot, meta, positions=qpos)
                ratio = O.find_target_compression_ratio(k.shape[1], target)
                out = O.compress_layer(qb, k, v, weights[layer][0], compression_ratio=ratio,
                                       is_prefill=False, positions=positions[layer],
                                       seq_len=nxt[layer], round_bf16=True, memory=mem[layer])
                yield ("event", ev, out)
                ev += 1
                k, v = out["out_k"], out["out_v"]
                positions[layer] = positions[layer][out["keep"]]
                mem[layer] = (out["M"], out["b"], out["Z"])
                steps[layer] = 0
                window[layer] = []
            window[layer] = window[layer][-meta["interval"]:]
            caches[layer] = (k, v)
        pos += n
    yield ("final", caches, mem)


def test_oracle_replays_the_reference_hooks():
    d, meta = load_case(HOOK_CASE)
    events = hook_events(d, meta)
    seen = 0
    n_readout_diff = 0
    for item in replay(d, meta):
        if item[0] == "event":
            _, i, out = item
            layer, keep, scores = events[i]
            assert np.array_equal(out["keep"], keep), i
            np.testing.assert_allclose(out["scores"], scores, rtol=1e-6, atol=1e-7)
            seen += 1
        elif item[0] == "readout":
            _, layer, tok0, n, ro = item
            ref = d["decode_out"][layer, 0, tok0:tok0 + n]
            diff = np.abs(ro - ref)
            n_readout_diff += int((diff > 0).sum())
            assert diff.max() <= 2 ** -7 * np.abs(ref).max()
        else:
            _, caches, mem = item
            for layer in range(2):
                assert np.array_equal(caches[layer][0], d[f"final_k_l{layer}"])
                assert np.array_equal(caches[layer][1], d[f"final_v_l{layer}"])
                for name, got in zip("Mb", mem[layer][:2]):
                    ref = d[f"{name}_l{layer}"]
                    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()
                assert abs(float(mem[layer][2]) - float(d[f"Z_l{layer}"][0])) <= 1e-6
    assert seen == len(events) == 6
    # bf16 outputs: the oracle's f64 sums round differently on very few entries
    assert n_readout_diff <= 0.02 * d["decode_out"].size
