"""Time the reference's own torch CPU path for one layer of the benchmark
workload.  TEST INFRASTRUCTURE: the measurement that ``bench.py``'s CPU legs
report beside the numpy restatement, made where the reference imports (it is
not shipped to the GPU host).

One layer of the headline configuration: bf16, batch 1, 8 KV / 32 query
heads, d = 128, L = 16384 cached tokens, the last 128 positions as the
scoring queries (prefill_qk_scope="question"), compression_ratio 0.75,
random-init indexer and memory stack (d_mem 512), through the reference's
``COREMemoryPress.compress`` (core/kvpress_adapter.py:968-1210).

Run:  CORE_REFERENCE_ROOT=<reference checkout> python oracle/time_reference_cpu.py
Writes oracle/reference_cpu_timing.json.
"""

from __future__ import annotations

import json
import os
import statistics
import sys
import time
from pathlib import Path
from types import SimpleNamespace

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent / "tests" / "golden"))


def main(repeats: int = 3) -> dict:
    import make_golden as G
    import torch
    ref = G._import_reference()
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    hkv, hq, d, L, nq, dm = 8, 32, 128, 16384, 128, 512
    times = []
    for rep in range(repeats + 1):
        rng = np.random.default_rng(100 + rep)
        q, k, v, _ = G.make_inputs(rng, hkv, hq, d, L, nq, "bfloat16")
        press, scorer, *_ = G.build_press(ref, seed=100 + rep, n_layers=2, hkv=hkv, hq=hq, d=d,
                                          d_mem=dm, gate_hidden=64, hidden=4096, ratio=0.75,
                                          dtype="bfloat16", scope="question")
        scorer.capture_diagnostics = False
        full_q = np.zeros((hq, L, d), np.float32)
        full_q[:, L - nq:] = q
        scorer.set_query_boundary(L - nq)
        module = SimpleNamespace(layer_idx=1, q_proj=None,
                                 _core_cached_query_states=G.to_torch(full_q, "bfloat16")[None],
                                 config=SimpleNamespace(num_attention_heads=hq, num_key_value_heads=hkv,
                                                        hidden_size=4096))
        keys, values = G.to_torch(k, "bfloat16")[None], G.to_torch(v, "bfloat16")[None]
        hs = torch.zeros(1, L, 8)
        with torch.no_grad():
            t0 = time.perf_counter()
            press.compress(module, hs, keys, values, None, {})
            dt = time.perf_counter() - t0
        if rep:  # the first run warms up
            times.append(dt)
    out = {"s_per_layer": statistics.median(times), "samples": times, "threads": threads,
           "workload": "1 layer: bf16, L=16384, 8/32 heads, 128 question-scope queries, r=0.75, "
                       "d_mem=512, COREMemoryPress.compress on CPU"}
    (HERE / "reference_cpu_timing.json").write_text(json.dumps(out, indent=1) + "\n")
    return out


if __name__ == "__main__":
    print(json.dumps(main()))
