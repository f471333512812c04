"""Benchmark: CORE KV-compression step on B200.

Workload (the headline configuration): a 32-layer Llama-3.1-8B-shaped KV cache
(8 KV heads, 32 query heads, d = 128), bf16, batch 1, 16384 cached tokens per
layer, a 128-query scoring window, compression_ratio 0.75 (4096 kept, 4 sinks),
latent-memory write with d_mem 512.  One step = compressing all 32 layers.
Inputs are seeded synthetic Gaussian-with-outlier caches and random-init
indexer / memory weights (no checkpoints or datasets are available).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Under torchrun every rank compresses its own sequence (batch sharding, no
collective on the data path); ``value`` is the whole-job rate over the slowest
rank.  ``--impl reference`` times the CPU restatement of the reference
algorithm (oracle/core_oracle.py) on the host cores instead.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "KV tokens compressed/sec per B200 (16K ctx, 32 layers); % tensor/HBM roofline"
UNIT = "tokens/s"
# LSE, combine, relation, merge, f6 resolve, 4 coverage, value sums, scores, Top-B,
# 4 memory write, gather
KERNELS_PER_LAYER = 17


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=60)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--seq-len", type=int, default=None,
                   help="cached tokens (default 16384; 131072 for --workload long)")
    p.add_argument("--batch", type=int, default=1, help="sequences per rank (batched serving)")
    p.add_argument("--n-queries", type=int, default=None,
                   help="query buffer (default 128; 512 for --workload long)")
    p.add_argument("--ratio", type=float, default=None,
                   help="compression_ratio (default 0.75; 0.9 for --workload long)")
    p.add_argument("--d-mem", type=int, default=512)
    p.add_argument("--e2e-steps", type=int, default=3)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--workload", default="prefill", choices=["prefill", "decode", "long", "attention"],
                   help="prefill: the headline 32-layer compression step; decode: decode-time "
                        "recompression with the memory readout")
    p.add_argument("--decode-tokens", type=int, default=512)
    p.add_argument("--interval", type=int, default=128)
    p.add_argument("--decode-ratio", type=float, default=0.5)
    p.add_argument("--streams", type=int, default=4, help="layers compressed concurrently")
    p.add_argument("--sharded-streams", type=int, default=3,
                   help="the same for the head-sharded step (its layers' collectives are "
                        "issued in layer order on every rank)")
    p.add_argument("--sharded", action="store_true",
                   help="--workload long: the head-sharded step even on one rank (under torchrun)")
    p.add_argument("--graph", action=argparse.BooleanOptionalAction, default=True,
                   help="replay the whole step (all layers' kernels and, head-sharded, the "
                        "NCCL collectives) as one CUDA graph (--no-graph: issue it eagerly)")
    p.add_argument("--long-steps", type=int, default=5,
                   help="timed steps of the long-context step (131072 tokens, 512 queries, r=0.9; "
                        "head-sharded over the ranks) reported as long_context in the headline "
                        "line; 0 leaves it out")
    p.add_argument("--batched-steps", type=int, default=3,
                   help="timed steps of batched serving (8 sequences x 32768 tokens, r=0.75, "
                        "32 layers, split over the ranks: 8/N sequences per rank) reported as "
                        "batched_serving in the headline line; 0 leaves it out")
    p.add_argument("--sm-reserve", type=int, default=8,
                   help="SMs the persistent grids leave free for the other streams' kernels")
    p.add_argument("--sharded-sm-reserve", type=int, default=34,
                   help="the same for the head-sharded step: NCCL's send/recv kernels (the "
                        "K/V rows gathered into a layer's owner) hold up to 32 SMs while they "
                        "run, and a persistent grid planned over those SMs would wait for them")
    a = p.parse_args()
    long = a.workload == "long"
    if a.seq_len is None:
        a.seq_len = 131072 if long else 16384
    if a.n_queries is None:
        a.n_queries = 512 if long else 128
    if a.ratio is None:
        a.ratio = 0.9 if long else 0.75
    return a


def config_dict(a, n):
    return {"workload": f"core_full compression step, {a.layers} layers x {a.batch} sequence(s) x "
                        f"{a.seq_len} tokens per rank",
            "layers": a.layers, "batch_per_rank": a.batch, "seq_len": a.seq_len,
            "n_kv_heads": 8, "n_q_heads": 32, "head_dim": 128, "query_buffer": a.n_queries,
            "compression_ratio": a.ratio, "n_kept": int(a.seq_len * (1 - a.ratio)),
            "d_mem": a.d_mem, "parallelism": f"batch-sharded x{n}",
            "l2": "inputs larger than L2 (32 layers x 64 MiB of K/V per step)",
            "layers_in_flight": a.streams, "sm_reserve": a.sm_reserve if a.streams > 1 else 0,
            "cuda_graph": bool(a.graph)}


# ---------------------------------------------------------------------------
# multi-rank plumbing (batch sharding: no collective on the data path)
# ---------------------------------------------------------------------------
def max_over_ranks(x: float, dist, device) -> float:
    """The slowest rank's value; every rank calls this at the same point."""
    if dist is None:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def whole_job_rate(n_ranks: int, tokens_per_rank: int, seconds: float) -> float:
    """Tokens compressed per second by all ranks together, timed by the slowest."""
    return n_ranks * tokens_per_rank / seconds


def rank_seed(rank: int) -> int:
    """Each rank compresses its own synthetic sequence."""
    return 1000 + 7919 * rank


# ---------------------------------------------------------------------------
# clocks during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True,
                                     text=True, timeout=5).stdout.strip()
                if out:
                    self.samples.append([x.strip() for x in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._t is not None:
            self._t.join(timeout=10)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU: the oracle port on a bounded sample
# ---------------------------------------------------------------------------
CPU_SAMPLE_MAX_LEN = 16384  # longer caches are sampled at this length (cost per token ~ constant)


def cpu_layer_sample(a, seed=0):
    """Time the oracle's compress_layer on one layer of the workload (at most
    CPU_SAMPLE_MAX_LEN cached tokens)."""
    from core_b200 import checkpoint as C
    from oracle import core_oracle as O
    rng = np.random.default_rng(seed)
    L, nq = min(a.seq_len, CPU_SAMPLE_MAX_LEN), a.n_queries
    out_idx = np.stack([rng.choice(128, 4, replace=False) for _ in range(8)])

    def go(h, n, idx):
        x = rng.standard_normal((h, n, 128), dtype=np.float32) / np.float32(np.sqrt(128))
        for i in range(h):
            x[i, :, idx[i]] *= 8
        return O.bf16_round(x)
    k = go(8, L, out_idx)
    q = go(32, nq, np.repeat(out_idx, 4, axis=0))
    v = O.bf16_round(rng.standard_normal((8, L, 128), dtype=np.float32))
    parts = C.random_checkpoint_parts(seed=seed, n_layers=1, n_kv_heads=8, n_q_heads=32, d_mem=a.d_mem)
    mlp = tuple(t.numpy() for t in parts["indexer"].modules[0])
    geo = parts["geometry"]
    w = O.LayerWeights(mlp=mlp, geometry=geo.weight[0].numpy(), prototypes=geo.prototypes.numpy(),
                       hadamard=geo.hadamard.numpy(), theta=parts["memory"].modules[0][0].numpy())
    t0 = time.perf_counter()
    O.compress_layer(q, k, v, w, compression_ratio=a.ratio, is_prefill=True, round_bf16=True)
    return time.perf_counter() - t0


def _sample_note(a):
    Ls = min(a.seq_len, CPU_SAMPLE_MAX_LEN)
    if Ls == a.seq_len:
        return f"L={Ls}"
    return (f"L={Ls} standing in for L={a.seq_len}: the work per cached token is the same "
            f"(nq fixed), so tokens/s carry over")


def cpu_baseline(a):
    t = cpu_layer_sample(a)
    Ls = min(a.seq_len, CPU_SAMPLE_MAX_LEN)
    return {"value": Ls / (t * a.layers), "unit": UNIT, "cores": os.cpu_count(),
            "kind": "port",
            "sample": f"1 of {a.layers} layers ({_sample_note(a)}, nq={a.n_queries}, "
                      f"r={a.ratio}, bf16-rounded inputs) through oracle.core_oracle.compress_layer "
                      f"in {t:.2f} s, extrapolated x{a.layers} to the {a.layers}-layer step; "
                      f"numpy/BLAS threads = host cores",
            "extrapolated_layers": a.layers,
            "reference_torch_cpu": reference_torch_timing()}


REF_LAYERS_PER_STEP = 4  # layers the CPU arm computes per step (each its own seed)


def reference_torch_timing():
    """The reference's own torch CPU path, one layer of the headline workload,
    measured where the reference imports (oracle/time_reference_cpu.py)."""
    path = os.path.join(ROOT, "oracle", "reference_cpu_timing.json")
    if not os.path.exists(path):
        return None
    rec = json.load(open(path))
    return {"s_per_layer": rec["s_per_layer"], "threads": rec["threads"],
            "where": "build container with the reference importable (not this host); "
                     "oracle/time_reference_cpu.py", "workload": rec["workload"]}


def run_reference(a, rank):
    if rank != 0:
        return
    steps = max(1, min(a.steps, 3))
    warm = min(a.warmup, 1)
    per = min(REF_LAYERS_PER_STEP, a.layers)
    for _ in range(warm):
        cpu_layer_sample(a, seed=1)
    step_s = [sum(cpu_layer_sample(a, seed=2 + per * i + j) for j in range(per))
              for i in range(steps)]
    t = statistics.median(step_s) / per  # seconds per layer
    Ls = min(a.seq_len, CPU_SAMPLE_MAX_LEN)
    value = Ls / (t * a.layers)
    sample = (f"{steps} timed steps (+{warm} warm-up layer), each {per} of the {a.layers} "
              f"layers ({_sample_note(a)}, nq={a.n_queries}, r={a.ratio}, each layer its own "
              f"seed) through oracle.core_oracle.compress_layer (the numpy restatement; the "
              f"reference's torch code is not on this host), median {t:.2f} s per layer; "
              f"value and ms_per_step scale the {per} layers to {a.layers} (x{a.layers / per:g})")
    long = a.workload == "long"
    line = {"metric": LONG_METRIC if long else METRIC, "value": value, "unit": UNIT,
            "impl": "reference", "n_gpus": a.gpus,
            "steps": steps, "warmup": warm, "ms_per_step": t * a.layers * a.seq_len / Ls * 1e3,
            "higher_is_better": True, "scaling": "strong" if long else "weak",
            "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": long_config(a, 1) if long else config_dict(a, 1),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                             "sample": sample, "extrapolated_layers": a.layers / per,
                             "reference_torch_cpu": reference_torch_timing()},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    line["config"]["cpu_sample"] = f"{per} of {a.layers} layers per step, scaled x{a.layers / per:g}"
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def build_layers(a, dev, seed_base=1000):
    from core_b200 import checkpoint as C
    from core_b200 import engine, synthetic
    parts = C.random_checkpoint_parts(seed=seed_base, n_layers=a.layers, n_kv_heads=8, n_q_heads=32,
                                      d_mem=a.d_mem)
    geo = parts["geometry"]
    layers = []
    for l in range(a.layers):
        q, k, v = synthetic.make_layer_inputs(seed=seed_base + 7 * l, batch=a.batch, n_kv_heads=8,
                                              n_q_heads=32, seq_len=a.seq_len,
                                              n_queries=a.n_queries, device=dev)
        lw = engine.LayerWeights.prepare(
            geometry=geo.weight[l], prototypes=geo.prototypes, hadamard=geo.hadamard,
            mlp_params=parts["indexer"].modules[l], theta=parts["memory"].modules[l][0],
            n_kv_heads=8, n_q_heads=32, device=dev)
        mem = engine.MemoryState.zeros(a.batch, a.d_mem, 8 * 128, dev)
        layers.append((q, k, v, lw, mem))
    return parts, layers


def run_prefill_steps(a, dev, dist, rank, local):
    """Build the synthetic 32-layer cache of this rank and time a.steps
    compression steps (one step = all layers, a.batch sequences of a.seq_len
    tokens), CUDA-graph replay unless a.graph is off.  Returns the timings and
    the built inputs (the end-to-end leg reuses them)."""
    from core_b200 import engine, ops
    parts, layers = build_layers(a, dev, seed_base=rank_seed(rank))
    L = a.seq_len
    n_kept = engine.n_kept_for(L, a.ratio, 4)
    pos = torch.arange(L, device=dev)[None].expand(a.batch, L).contiguous()
    n_sms = torch.cuda.get_device_properties(dev).multi_processor_count
    budget = ops.sm_budget(max(1, n_sms - a.sm_reserve) if a.streams > 1 else 0)
    # one workspace per stream, sized under the SM budget the launches will plan with
    from core_b200 import _lib
    dims = _lib.CoreDims(a.batch, 32, 8, 128, a.n_queries, L, _lib.CORE_DTYPE_BF16)
    need = _lib.load().core_compress_layer_workspace_bytes(ctypes.byref(dims), n_kept, a.d_mem)
    ws = [torch.empty(int(need), dtype=torch.uint8, device=dev) for _ in range(a.streams)]
    # one (start, end) pair per layer and timed step, around the QK relation kernel
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(a.layers)] for _ in range(a.steps)]
    for pairs in ev:  # materialise the event handles before the timed region
        for e0, e1 in pairs:
            e0.record()
            e1.record()
    torch.cuda.synchronize()

    def step(pairs, n_streams=a.streams):
        jobs = [dict(q=q, keys=k, values=v, weights=lw, positions=pos, memory=mem,
                     timing_events=None if pairs is None else pairs[l])
                for l, (q, k, v, lw, mem) in enumerate(layers)]
        engine.compress_layers(jobs, n_streams=n_streams, workspaces=ws[:n_streams], n_kept=n_kept,
                               original_length=L, is_prefill=True)

    for _ in range(a.warmup):
        step(None)
    torch.cuda.synchronize()
    ops.status(dev)
    # The relation pass timed in a step issued on one stream: its events then
    # bracket the kernel alone.  With layers in flight on several streams the
    # same events also count the time a launch waits for the SMs that another
    # layer's persistent kernel holds (reported beside it).
    ev_alone = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                for _ in range(a.layers)]
    for e0, e1 in ev_alone:  # materialise the handles (the library records them)
        e0.record()
        e1.record()
    torch.cuda.synchronize()
    step(ev_alone, n_streams=1)
    torch.cuda.synchronize()
    relation_alone_ms = [e0.elapsed_time(e1) for e0, e1 in ev_alone]
    graph = None
    graph_note = None
    if a.graph:
        # one eager step with the relation events for the roofline, then the capture
        step(ev[0])
        torch.cuda.synchronize()
        relation_ms = [e0.elapsed_time(e1) for e0, e1 in ev[0]]
        try:
            graph = torch.cuda.CUDAGraph()
            cap = torch.cuda.Stream(dev)
            cap.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.graph(graph, stream=cap):
                step(None)
            torch.cuda.synchronize()
            graph.replay()
            torch.cuda.synchronize()
        except RuntimeError as exc:  # the step has no collectives: this rank issues eagerly
            graph = None
            graph_note = f"graph capture failed, eager issue: {str(exc).splitlines()[0][:160]}"
            torch.cuda.synchronize()
        ops.status(dev)

    # ---- timed region: device-resident inputs ----
    with ClockSampler(local) as clocks:
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        h0 = time.perf_counter()
        for i in range(a.steps):
            if graph is not None:
                graph.replay()
            else:
                step(ev[i])
            if i == 0:  # the first step's issue time (later ones wait on a full launch queue)
                host_ms = (time.perf_counter() - h0) * 1e3
        t1.record()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
    budget.__exit__(None, None, None)  # the e2e leg below uses the press on one stream
    ms = t0.elapsed_time(t1) / a.steps
    if graph is None:
        relation_ms = [e0.elapsed_time(e1) for pairs in ev for e0, e1 in pairs]
    else:
        del graph
        torch.cuda.synchronize()
    ops.status(dev)
    return dict(ms=ms, relation_ms=relation_ms, relation_alone_ms=relation_alone_ms,
                host_ms=host_ms, clocks=clocks,
                graph_note=graph_note, parts=parts, layers=layers, ws=ws)


def main():
    a = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if a.impl == "reference":
        run_reference(a, rank)
        return
    dist = None
    if world > 1 or (a.workload == "long" and a.sharded):
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    n = world
    from core_b200 import engine, ops

    if a.workload == "long":
        line = run_long(a, dev, dist, rank, world)
        if rank == 0:
            print(json.dumps(line), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return
    if a.workload == "attention":
        line = run_attention(a, dev)
        print(json.dumps(line), flush=True)
        return
    if a.workload == "decode":
        line = run_decode(a, dev, dist, rank)
        if rank == 0:
            print(json.dumps(line), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return
    r = run_prefill_steps(a, dev, dist, rank, local)
    ms, relation_ms, host_ms, clocks, graph_note = (r["ms"], r["relation_ms"], r["host_ms"],
                                                    r["clocks"], r["graph_note"])
    relation_alone_ms = r["relation_alone_ms"]
    parts, layers, ws = r["parts"], r["layers"], r["ws"]
    del r
    L = a.seq_len
    ms = max_over_ranks(ms, dist, dev)
    value = whole_job_rate(n, a.batch * L, ms / 1e3)

    # ---- roofline of the dominant kernel (QK relation pass) ----
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak, peak_src = 1590.0, "fallback"
    if os.path.exists(peaks_path):
        pk = json.load(open(peaks_path))
        peak, peak_src = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))), "measured"
    flops = 2.0 * 32 * a.n_queries * L * 128
    rel_ms = statistics.mean(relation_alone_ms)
    rel_ms_overlapped = statistics.mean(relation_ms)
    achieved = flops / (rel_ms / 1e3) / 1e12
    traffic = None
    tpath = os.path.join(ROOT, "profiles", f"qk_relation_L{L}_traffic.txt")
    if os.path.exists(tpath):
        rec = dict(line.split(None, 1) for line in open(tpath) if line.strip())
        if int(rec.get("seq_len", 0)) == L:
            traffic = int(rec["bytes_per_launch"])
    roofline = {"kernel": "qk_relation_kernel (QK pass 2: relation + per-key statistics)",
                "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": achieved / peak, "peak_source": f"{peak_src} bf16_tflops_sustained",
                "traffic": traffic, "avg_launch_ms": rel_ms,
                "timing": "CUDA events around each layer's relation kernel in an eager step "
                          "issued on one stream (the kernel alone)",
                "avg_launch_ms_layers_in_flight": rel_ms_overlapped,
                "frac_layers_in_flight": flops / (rel_ms_overlapped / 1e3) / 1e12 / peak,
                "algorithmic": f"2*Hq*nq*L*d = {flops / 1e9:.2f} GFLOP per launch"}

    # ---- end to end through the press API with host buffers ----
    e2e = run_e2e(a, dev, parts, layers, dist) if a.e2e_steps > 0 else None

    # ---- the long-context configuration on the same ranks ----
    long_context = None
    if a.long_steps > 0:
        del layers, parts, ws
        torch.cuda.empty_cache()
        la = argparse.Namespace(**vars(a))
        la.workload, la.seq_len, la.n_queries, la.ratio = "long", 131072, 512, 0.9
        la.steps, la.warmup, la.sharded, la.no_cpu_baseline = a.long_steps, max(3, a.warmup), n > 1, True
        ll = run_long(la, dev, dist, rank, n)
        long_context = {k: ll[k] for k in ("metric", "value", "unit", "n_gpus", "steps", "warmup",
                                           "ms_per_step", "scaling", "config", "roofline",
                                           "host_issue_ms_per_step", "gpu_launches", "clocks")}
        long_context["note"] = ("one 131072-token sequence; N=1 runs the fused one-GPU layer step, "
                                "N>1 the head-sharded step (rank r holds KV heads [8r/N, 8(r+1)/N), "
                                "NCCL for the cross-head exchanges, each layer's memory write on "
                                "rank l mod N); its own timed region, max over ranks")

    # ---- batched serving on the same ranks: 8 x 32768 tokens split by sequence ----
    batched = None
    if a.batched_steps > 0 and 8 % n == 0:
        layers = parts = ws = None  # the headline's inputs
        torch.cuda.empty_cache()
        ba = argparse.Namespace(**vars(a))
        ba.batch, ba.seq_len, ba.n_queries, ba.ratio = 8 // n, 32768, 128, 0.75
        ba.steps, ba.warmup = a.batched_steps, max(3, a.warmup)
        br = run_prefill_steps(ba, dev, dist, rank, local)
        bms = max_over_ranks(br["ms"], dist, dev)
        del br["layers"], br["parts"], br["ws"]
        torch.cuda.empty_cache()
        batched = {"metric": "KV tokens compressed/sec, batched serving: 8 sequences x 32768 tokens, "
                             "32 layers, split by sequence over the GPUs",
                   "value": whole_job_rate(n, ba.batch * ba.seq_len, bms / 1e3), "unit": UNIT,
                   "n_gpus": n, "steps": ba.steps, "warmup": ba.warmup, "ms_per_step": bms,
                   "scaling": "strong", "config": config_dict(ba, n),
                   "gpu_launches": KERNELS_PER_LAYER * ba.layers * ba.steps,
                   "clocks": br["clocks"].summary(),
                   "note": "8 sequences in all, 8/N per rank, each rank its own sequences and "
                           "memory state (no collective on the data path); its own timed region, "
                           "max over ranks"}

    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": n, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": config_dict(a, n), "roofline": roofline, "e2e": e2e,
            "gpu_launches": KERNELS_PER_LAYER * a.layers * a.steps,
            "host_issue_ms_per_step": host_ms, "clocks": clocks.summary()}
    if long_context is not None:
        line["long_context"] = long_context
    if batched is not None:
        line["batched_serving"] = batched
    if graph_note is not None:
        line["config"]["cuda_graph"] = False
        line["graph_note"] = graph_note
    if rank == 0 and n == 1 and not a.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(a)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------
# long context: one sequence, KV heads sharded across the ranks
# ---------------------------------------------------------------------------
LONG_METRIC = ("KV tokens compressed/sec, one 131072-token sequence, 32 layers, "
               "KV heads sharded across GPUs")


def measured_peaks() -> dict:
    """The pool's measured peaks (MEASURED_PEAKS.json), empty when absent."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    return json.load(open(path)) if os.path.exists(path) else {}


def run_attention(a, dev):
    """The prefill attention of one layer (32 query / 8 KV heads, d = 128,
    bf16, causal over seq_len tokens) with its row LSE, on this library's
    kernel and on flash_attn_func (the library call of the reference's
    attention hook) when it runs here; CUDA events, max of nothing (one GPU)."""
    from core_b200 import ops
    L, Hq, Hkv = a.seq_len, 32, 8
    g = torch.Generator(device="cpu").manual_seed(5)
    q = (torch.randn(1, Hq, L, 128, generator=g) / 128 ** 0.5).to(dev, torch.bfloat16)
    k = (torch.randn(1, Hkv, L, 128, generator=g) / 128 ** 0.5).to(dev, torch.bfloat16)
    v = torch.randn(1, Hkv, L, 128, generator=g).to(dev, torch.bfloat16)
    flops = 4.0 * 128 * Hq * L * (L + 1) / 2  # QK and PV over the visible (query, key) pairs

    def timed(fn):
        for _ in range(max(a.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(a.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / a.steps

    out = torch.empty(1, L, Hq, 128, dtype=torch.bfloat16, device=dev)
    with ClockSampler(dev.index or 0) as clk:
        ms = timed(lambda: ops.attention_prefill(q, k, v, out=out))
    ops.status(dev)
    peak = measured_peaks().get("bf16_tflops")
    line = {"metric": "prefill attention with row LSE, tokens/s (one layer, 32/8 heads, d 128, causal)",
            "value": L / (ms * 1e-3), "unit": "tokens/s", "ms_per_call": ms, "steps": a.steps,
            "seq_len": L, "dtype": "bf16", "tflops": flops / (ms * 1e-3) / 1e12,
            "roofline": {"bound": "tensor", "peak": peak, "unit": "TFLOP/s",
                         "frac": (flops / (ms * 1e-3) / 1e12 / peak) if peak else None,
                         "peak_source": "measured bf16_tflops (burst)",
                         "algorithmic": "4 d Hq L (L+1) / 2 FLOP per call"},
            "clocks": clk.summary()}
    try:
        from flash_attn import flash_attn_func
        qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        fms = timed(lambda: flash_attn_func(qt, kt, vt, dropout_p=0.0, softmax_scale=128 ** -0.5,
                                            causal=True, return_attn_probs=True))
        line["flash_attn"] = {"ms_per_call": fms, "tflops": flops / (fms * 1e-3) / 1e12,
                              "version": __import__("flash_attn").__version__}
    except Exception as e:  # noqa: BLE001
        line["flash_attn"] = {"unavailable": str(e)[:200]}
    return line


def long_config(a, n):
    return {"workload": f"core_full compression step, {a.layers} layers x 1 sequence x "
                        f"{a.seq_len} tokens, KV heads sharded over {n} GPU(s)",
            "layers": a.layers, "seq_len": a.seq_len, "n_kv_heads": 8, "n_q_heads": 32,
            "head_dim": 128, "query_buffer": a.n_queries, "compression_ratio": a.ratio,
            "n_kept": int(a.seq_len * (1 - a.ratio)), "d_mem": a.d_mem,
            "parallelism": f"head-sharded x{n}" if n > 1 or a.sharded else "1 GPU",
            "cuda_graph": bool(a.graph),
            "sm_reserve": a.sharded_sm_reserve if n > 1 or a.sharded else a.sm_reserve,
            "layers_in_flight": a.sharded_streams if n > 1 or a.sharded else a.streams,
            "l2": f"inputs larger than L2 ({a.layers} x {a.seq_len * 8 * 128 * 4 >> 20} MiB of K/V)"}


def run_long(a, dev, dist, rank, world):
    """One long sequence; one GPU runs the fused layer step (layers on
    concurrent streams), several GPUs the head-sharded step: rank r holds KV
    heads [8r/N, 8(r+1)/N) of every layer and the memory state of the layers
    l = r mod N, with NCCL for the cross-head reductions."""
    from core_b200 import checkpoint as C
    from core_b200 import engine, ops, synthetic
    from core_b200.sharded import DistExchange, HeadShard, ShardWeights, compress_layer_sharded
    L, nq, hkv, hq, d = a.seq_len, a.n_queries, 8, 32, 128
    G = hq // hkv
    seed = 5000  # one sequence: the same inputs on every rank
    parts = C.random_checkpoint_parts(seed=seed, n_layers=a.layers, n_kv_heads=hkv, n_q_heads=hq,
                                      d_mem=a.d_mem)
    geo = parts["geometry"]
    n_kept = engine.n_kept_for(L, a.ratio, 4)
    sh = HeadShard(rank, world, hkv, L)
    sharded = world > 1 or a.sharded
    layers = []
    for l in range(a.layers):
        q, k, v = synthetic.make_layer_inputs(seed=seed + 7 * l, batch=1, n_kv_heads=hkv,
                                              n_q_heads=hq, seq_len=L, n_queries=nq, device=dev)
        theta = parts["memory"].modules[l][0]
        if not sharded:
            lw = engine.LayerWeights.prepare(
                geometry=geo.weight[l], prototypes=geo.prototypes, hadamard=geo.hadamard,
                mlp_params=parts["indexer"].modules[l], theta=theta, n_kv_heads=hkv,
                n_q_heads=hq, device=dev)
            layers.append((q, k, v, lw, engine.MemoryState.zeros(1, a.d_mem, hkv * d, dev)))
        else:
            inp = dict(q=q[:, sh.h0 * G:sh.h1 * G].contiguous(), keys=k[:, sh.h0:sh.h1].contiguous(),
                       values=v[:, sh.h0:sh.h1].contiguous())
            del q, k, v
            own = HeadShard.owner(l, world) == rank
            wt = ShardWeights.prepare(sh, geometry=geo.weight[l], prototypes=geo.prototypes,
                                      hadamard=geo.hadamard, mlp_params=parts["indexer"].modules[l],
                                      theta=theta if own else None, n_q_heads=hq, device=dev)
            mem = engine.MemoryState.zeros(1, a.d_mem, hkv * d, dev) if own else None
            layers.append((inp, wt, mem))
    torch.cuda.empty_cache()
    pos = torch.arange(L, device=dev)
    ev = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(a.layers)] for _ in range(a.steps)]
    for pairs in ev:
        for e0, e1 in pairs:
            e0.record()
            e1.record()
    torch.cuda.synchronize()
    budget = None
    if not sharded:
        n_sms = torch.cuda.get_device_properties(dev).multi_processor_count
        budget = ops.sm_budget(max(1, n_sms - a.sm_reserve) if a.streams > 1 else 0)
        from core_b200 import _lib
        dims = _lib.CoreDims(1, hq, hkv, d, nq, L, _lib.CORE_DTYPE_BF16)
        need = _lib.load().core_compress_layer_workspace_bytes(ctypes.byref(dims), n_kept, a.d_mem)
        ws = [torch.empty(int(need), dtype=torch.uint8, device=dev) for _ in range(a.streams)]
        pos2 = pos[None]

        def step(pairs):
            jobs = [dict(q=q, keys=k, values=v, weights=lw, positions=pos2, memory=mem,
                         timing_events=None if pairs is None else pairs[l])
                    for l, (q, k, v, lw, mem) in enumerate(layers)]
            engine.compress_layers(jobs, n_streams=a.streams, workspaces=ws, n_kept=n_kept,
                                   original_length=L, is_prefill=True)
    else:
        ex = DistExchange()
        # a second communicator for the bulk K/V gathers, so that they overlap
        # the small exchanges of the layer instead of queueing before them
        bulk = DistExchange(dist.new_group(list(range(world))))
        # Layers on side streams, so that one layer's exchanges and its owner's
        # memory write overlap the next layers' QK work.  The host issues every
        # layer's collectives in layer order on every rank.
        n_sms = torch.cuda.get_device_properties(dev).multi_processor_count
        budget = ops.sm_budget(max(1, n_sms - a.sharded_sm_reserve))
        streams = [torch.cuda.Stream(dev) for _ in range(max(1, a.sharded_streams))]

        def step(pairs):
            main = torch.cuda.current_stream(dev)
            fork = torch.cuda.Event()
            fork.record(main)
            for st in streams:
                st.wait_event(fork)
            for l, (inp, wt, mem) in enumerate(layers):
                with torch.cuda.stream(streams[l % len(streams)]):
                    compress_layer_sharded(ex, [sh], [inp], [wt], layer_idx=l, n_kept=n_kept,
                                           positions=pos, original_length=L, is_prefill=True,
                                           memory=mem, bulk=bulk,
                                           qk_events=None if pairs is None else pairs[l])
            for st in streams:
                done = torch.cuda.Event()
                done.record(st)
                main.wait_event(done)

    for _ in range(a.warmup):
        step(None)
    torch.cuda.synchronize()
    ops.status(dev)
    graph = None
    if a.graph:
        # one eager step with the QK events for the roofline, then the capture
        step(ev[0])
        torch.cuda.synchronize()
        qk_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in ev[0])
        graph = torch.cuda.CUDAGraph()
        cap = torch.cuda.Stream(dev)
        cap.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.graph(graph, stream=cap):
            step(None)
        torch.cuda.synchronize()
        graph.replay()  # one replay before the timed region
        torch.cuda.synchronize()
        ops.status(dev)
    with ClockSampler(dev.index) as clocks:
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        h0 = time.perf_counter()
        for i in range(a.steps):
            if graph is not None:
                graph.replay()
            else:
                step(ev[i])
            if i == 0:  # the first step's issue time (later ones wait on a full launch queue)
                host_ms = (time.perf_counter() - h0) * 1e3
        t1.record()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
    if budget is not None:
        budget.__exit__(None, None, None)
    ops.status(dev)
    ms = max_over_ranks(t0.elapsed_time(t1) / a.steps, dist, dev)
    host_ms = max_over_ranks(host_ms, dist, dev)
    if graph is None:
        qk_ms = statistics.mean(e0.elapsed_time(e1) for pairs in ev for e0, e1 in pairs)
    else:
        del graph  # graphs holding NCCL calls go before the process group
        torch.cuda.synchronize()
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak, peak_src = 1590.0, "fallback"
    if os.path.exists(peaks_path):
        pk = json.load(open(peaks_path))
        peak, peak_src = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))), "measured"
    if not sharded:
        flops = 2.0 * hq * nq * L * d
        kernel = "qk_relation_kernel (QK pass 2: relation + per-key statistics)"
        alg = f"2*Hq*nq*L*d = {flops / 1e9:.2f} GFLOP per launch"
    else:
        flops = 2 * 2.0 * (hq // world) * nq * L * d
        kernel = ("QK stage of one rank (qk_lse_kernel + qk_relation_kernel + merge over the "
                  "rank's heads)")
        alg = f"2 passes x 2*Hq_rank*nq*L*d = {flops / 1e9:.2f} GFLOP per layer"
    achieved = flops / (qk_ms / 1e3) / 1e12
    traffic = None
    tpath = os.path.join(ROOT, "profiles", f"qk_relation_L{L}_traffic.txt")
    if not sharded and os.path.exists(tpath):
        rec = dict(line.split(None, 1) for line in open(tpath) if line.strip())
        if int(rec.get("seq_len", 0)) == L:
            traffic = int(rec["bytes_per_launch"])
    roofline = {"kernel": kernel, "bound": "tensor", "achieved": achieved, "peak": peak,
                "unit": "TFLOP/s", "frac": achieved / peak,
                "peak_source": f"{peak_src} bf16_tflops_sustained", "traffic": traffic,
                "avg_launch_ms": qk_ms, "algorithmic": alg}
    if not sharded:
        launches = KERNELS_PER_LAYER * a.layers * a.steps
    else:
        # per layer: 5 QK summary, 1 partial projection, 1 value sums, 1 summary merge,
        # 2 range totals, 2 statistics + assignment, 1 occupancy, 1 scores, 1 Top-B, 1 gather
        # of the kept rows (the owner gathers the evicted rows by index: r >= 0.75); 4
        # memory-write kernels on the layers this rank owns
        owned = sum(1 for l in range(a.layers) if HeadShard.owner(l, world) == rank)
        launches = (16 * a.layers + 4 * owned) * a.steps
    line = {"metric": LONG_METRIC, "value": L / (ms / 1e3), "unit": UNIT, "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": long_config(a, world), "roofline": roofline, "e2e": None,
            "host_issue_ms_per_step": host_ms,
            "gpu_launches": launches, "clocks": clocks.summary()}
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(a)
    return line


# ---------------------------------------------------------------------------
# decode-time recompression (prefill, then decode with readout every step)
# ---------------------------------------------------------------------------
DECODE_METRIC = "KV tokens recompressed/sec during decode (readout every step), 32 layers"


def run_decode(a, dev, dist, rank):
    """Prefill compression of every layer to ratio ``--decode-ratio`` (not
    timed), then ``--decode-tokens`` decode steps: every step appends one K/V
    row per layer and applies the memory readout to that layer's attention
    output; every ``--interval`` steps each layer is recompressed back to the
    post-prefill size with the buffered queries (decode branch).  Decode-step
    K/V rows, post-RoPE queries and attention outputs are synthetic
    (the query projection and RoPE of the reference's decode path are library
    GEMMs and are not part of the timed work)."""
    from core_b200 import checkpoint as C
    from core_b200 import engine, ops, synthetic
    L0, nq, hkv, hq, d = a.seq_len, a.n_queries, 8, 32, 128
    seed = rank_seed(rank)
    parts = C.random_checkpoint_parts(seed=seed, n_layers=a.layers, n_kv_heads=hkv, n_q_heads=hq,
                                      d_mem=a.d_mem)
    geo = parts["geometry"]
    n_keep = engine.n_kept_for(L0, a.decode_ratio, 4)
    cap = n_keep + a.interval
    g = torch.Generator(device=dev).manual_seed(seed)
    layers = []
    for l in range(a.layers):
        q, k, v = synthetic.make_layer_inputs(seed=seed + 7 * l, batch=1, n_kv_heads=hkv,
                                              n_q_heads=hq, seq_len=L0, n_queries=nq, device=dev)
        lw = engine.LayerWeights.prepare(
            geometry=geo.weight[l], prototypes=geo.prototypes, hadamard=geo.hadamard,
            mlp_params=parts["indexer"].modules[l], theta=parts["memory"].modules[l][0],
            n_kv_heads=hkv, n_q_heads=hq, device=dev)
        mem = engine.MemoryState.zeros(1, a.d_mem, hkv * d, dev)
        out = engine.compress_layer(q, k, v, lw, n_kept=n_keep,
                                    positions=torch.arange(L0, device=dev)[None],
                                    original_length=L0, is_prefill=True, memory=mem)
        K = torch.empty(1, hkv, cap, d, dtype=torch.bfloat16, device=dev)
        V = torch.empty_like(K)
        K[:, :, :n_keep] = out["keys"]
        V[:, :, :n_keep] = out["values"]
        pos = torch.empty(1, cap, dtype=torch.int64, device=dev)
        pos[:, :n_keep] = out["keep"].to(torch.int64)
        th, gw1, gb1, gw2, gb2 = (t.to(dev).float() for t in parts["memory"].params(l))
        o_proj = torch.randn(hq * d, hq * d, device=dev, generator=g) / (hq * d) ** 0.5
        layers.append(dict(K=K, V=V, pos=pos, lw=lw, mem=mem, theta=th.contiguous(),
                           gate=(gw1.contiguous(), gb1.contiguous(), gw2.reshape(-1).contiguous(),
                                 gb2.reshape(-1).contiguous()),
                           o_fold=engine.fold_groups(o_proj, hkv, hq // hkv, d)))
    steps = a.decode_tokens
    new_kv = (torch.randn(steps, a.layers, 2, hkv, d, device=dev, generator=g)).to(torch.bfloat16)
    new_q = (torch.randn(steps, a.layers, hq, d, device=dev, generator=g) / d ** 0.5).to(torch.bfloat16)
    attn = torch.randn(1, 1, hq * d, device=dev, generator=g).to(torch.bfloat16)
    qbuf = [torch.empty(1, hq, a.interval, d, dtype=torch.bfloat16, device=dev)
            for _ in range(a.layers)]

    clock = [L0]  # absolute position of the next decoded token (runs on across passes)
    # The memory readout of one decode step for all layers, replayed as a CUDA
    # graph: the per-step inputs are copied into static buffers first.
    from core_b200 import _lib
    rdims = _lib.CoreDims(1, hq, hkv, d, 1, 1, _lib.CORE_DTYPE_BF16)
    ws_ro = torch.empty(int(_lib.load().core_memory_readout_workspace_bytes(
        ctypes.byref(rdims), 1, a.d_mem, layers[0]["gate"][0].shape[0])) + 256,
        dtype=torch.uint8, device=dev)
    q_static = torch.empty(a.layers, 1, hq, 1, d, dtype=torch.bfloat16, device=dev)
    attn_static = torch.empty(a.layers, 1, 1, hq * d, dtype=torch.bfloat16, device=dev)

    def readouts():
        for l, st in enumerate(layers):
            attn_static[l].copy_(attn)
            ops.memory_readout(q_static[l], st["theta"], st["gate"], st["mem"].M, st["mem"].b,
                               st["o_fold"], attn_static[l], n_kv_heads=hkv, workspace=ws_ro)

    q_static.copy_(new_q[0].view(a.layers, 1, hq, 1, d))
    readouts()  # eager once: kernel attributes are set outside the capture
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        readouts()

    def decode_phase(readout_only=False):
        recompressed = 0
        for blk in range(steps // a.interval):
            s0 = blk * a.interval
            if not readout_only:
                # the interval's new K/V rows (written by the attention layers in a model)
                for l, st in enumerate(layers):
                    rows = new_kv[s0:s0 + a.interval, l]  # (interval, 2, hkv, d)
                    st["K"][0, :, n_keep:cap] = rows[:, 0].transpose(0, 1)
                    st["V"][0, :, n_keep:cap] = rows[:, 1].transpose(0, 1)
                    st["pos"][0, n_keep:cap] = torch.arange(clock[0], clock[0] + a.interval,
                                                            device=dev)
                    qbuf[l].copy_(new_q[s0:s0 + a.interval, l].transpose(0, 1)[None])
            for step in range(s0, s0 + a.interval):
                q_static.copy_(new_q[step].view(a.layers, 1, hq, 1, d))
                graph.replay()
            if readout_only:
                continue
            clock[0] += a.interval
            for l, st in enumerate(layers):
                r = engine.compress_layer(
                    qbuf[l], st["K"], st["V"], st["lw"], n_kept=n_keep, positions=st["pos"],
                    original_length=clock[0], is_prefill=False, memory=st["mem"])
                st["K"][:, :, :n_keep] = r["keys"]
                st["V"][:, :, :n_keep] = r["values"]
                st["pos"][0, :n_keep] = st["pos"][0][r["keep"][0].long()]
                recompressed += cap
        return recompressed

    def timed(fn):
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        r = fn()
        e1.record()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        return r, e0.elapsed_time(e1)

    decode_phase()  # warm-up pass (memory states keep evolving, as in a real sequence)
    ops.status(dev)
    tokens, ms = timed(decode_phase)
    _, ms_readout = timed(lambda: decode_phase(readout_only=True))
    ops.status(dev)
    ms = max_over_ranks(ms, dist, dev)
    ms_readout = max_over_ranks(ms_readout, dist, dev)
    n = dist.get_world_size() if dist is not None else 1
    return {"metric": DECODE_METRIC, "value": whole_job_rate(n, tokens, ms / 1e3),
            "unit": UNIT, "n_gpus": n, "steps": 1, "warmup": 1, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": f"decode-time recompression: prefill {L0} tokens to "
                                   f"{n_keep}, {steps} decode steps, recompression every "
                                   f"{a.interval} steps ({steps // a.interval} per layer), "
                                   f"memory readout every step, {a.layers} layers",
                       "layers": a.layers, "prefill_tokens": L0, "decode_tokens": steps,
                       "compression_interval": a.interval, "compression_ratio": a.decode_ratio,
                       "retained": n_keep, "d_mem": a.d_mem},
            "readout_us_per_layer_step": ms_readout * 1e3 / (steps * a.layers),
            "recompressed_tokens": tokens}


class _FakeAttn:
    """Minimal attention module for the press API: layer index, config and the
    post-RoPE queries the CORE attention adapter stashes."""

    def __init__(self, layer_idx):
        self.layer_idx = layer_idx
        self.q_proj = True


def run_e2e(a, dev, parts, layers, dist):
    """Per step: pinned H2D of every layer's K, V and scoring queries, the
    press's compress() for every layer, D2H of retained positions and Z."""
    from core_b200 import press as P
    L, nq = a.seq_len, a.n_queries
    cfg = parts["config"]
    cfg.prefill_qk_scope = "question"
    base = P.COREScorerPress(indexer=parts["indexer"].to(dev), feature_extractor=parts["geometry"].to(dev),
                             compression_ratio=a.ratio, use_indexer_stack=True, scoring_layer_idx=-1,
                             n_sink_protect=4, prefill_qk_scope="question")
    press = P.COREMemoryPress(base_press=base, memory_module=parts["memory"].to(dev))
    host = []
    for (q, k, v, _, _) in layers:
        host.append((q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory()))
    full_q = torch.zeros(a.batch, 32, L, 128, dtype=torch.bfloat16, device=dev)
    hs = torch.zeros(a.batch, L, 1, device=dev)
    mods = [_FakeAttn(l) for l in range(a.layers)]
    h2d = sum(t.numel() * t.element_size() for h in host for t in h)
    d2h_per_step = [0]

    # Double-buffered device slots: the copy stream uploads layer l + 2 while
    # the compute stream compresses layer l + 1 (PCIe and SMs run concurrently).
    nbuf = 2
    copy_stream = torch.cuda.Stream(dev)
    slots = [tuple(torch.empty(t.shape, dtype=t.dtype, device=dev) for t in host[0])
             for _ in range(nbuf)]
    copied = [torch.cuda.Event() for _ in range(nbuf)]
    consumed = [torch.cuda.Event() for _ in range(nbuf)]

    def upload(l):
        j = l % nbuf
        with torch.cuda.stream(copy_stream):
            if l >= nbuf:
                copy_stream.wait_event(consumed[j])
            for dst, src in zip(slots[j], host[l]):
                dst.copy_(src, non_blocking=True)
            copied[j].record(copy_stream)

    def step():
        press.reset_cache()
        base.set_query_boundary(L - nq)
        comp = torch.cuda.current_stream()
        results = []
        for l in range(min(nbuf, len(host))):
            upload(l)
        for l in range(len(host)):
            j = l % nbuf
            comp.wait_event(copied[j])
            q, k, v = slots[j]
            full_q[:, :, L - nq:].copy_(q)
            mods[l]._core_cached_query_states = full_q
            press.compress(mods[l], hs, k, v, None, {})
            consumed[j].record(comp)
            if l + nbuf < len(host):
                upload(l + nbuf)
            results.append(base.cache_metadata.positions[l])
            results.append(press._Z[l])
        out = [r.to("cpu", non_blocking=True) for r in results]
        comp.synchronize()
        d2h_per_step[0] = sum(o.numel() * o.element_size() for o in out)
        return out

    step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(a.e2e_steps):
        step()
    torch.cuda.synchronize()
    dt = (time.perf_counter() - t0) / a.e2e_steps
    dt = max_over_ranks(dt, dist, dev)
    n = dist.get_world_size() if dist is not None else 1
    return {"value": whole_job_rate(n, L, dt), "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h_per_step[0], "ms_per_step": dt * 1e3,
            "steps": a.e2e_steps,
            "path": "core_b200.press.COREMemoryPress.compress per layer, inputs from pinned host "
                    "memory (uploads double-buffered on a copy stream)"}


if __name__ == "__main__":
    main()
