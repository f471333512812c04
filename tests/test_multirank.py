"""The multi-rank host logic of bench.py on world_size-2 gloo groups (CPU):
the slowest-rank reduction, the whole-job rate, per-rank seeds, and the
reference arm running on rank 0 only."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ms = [12.5, 19.0][rank]
        slow = bench.max_over_ranks(ms, dist, torch.device("cpu"))
        rate = bench.whole_job_rate(dist.get_world_size(), 16384, slow / 1e3)
        seeds = [None] * world
        dist.all_gather_object(seeds, bench.rank_seed(rank))
        out[rank] = (slow, rate, seeds)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_two_rank_reduction_and_rate():
    world = 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    for rank in range(world):
        slow, rate, seeds = res[rank]
        assert slow == 19.0                      # max over ranks, on every rank
        assert rate == pytest.approx(2 * 16384 / 0.019)
        assert len(set(seeds)) == world          # distinct sequences per rank


def test_reference_arm_only_on_rank_zero(capsys):
    import json
    import sys
    sys.path.insert(0, ROOT)
    import bench
    sys.argv = ["bench.py", "--impl", "reference", "--gpus", "2", "--steps", "1", "--warmup", "0",
                "--seq-len", "64", "--n-queries", "8", "--layers", "2", "--d-mem", "64"]
    ns = bench.parse()
    bench.run_reference(ns, rank=1)             # a non-zero rank returns without work
    assert capsys.readouterr().out == ""
    bench.run_reference(ns, rank=0)             # rank 0 prints the reference line
    line = json.loads(capsys.readouterr().out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["value"] > 0


def test_bench_defaults_in_the_reported_config():
    """The headline step runs four layers in flight on 140 SMs' persistent
    grids; the head-sharded long-context step keeps three streams and leaves
    34 SMs to NCCL.  The JSON line reports what ran."""
    import sys
    import bench
    argv = sys.argv
    try:
        sys.argv = ["bench.py"]
        a = bench.parse()
    finally:
        sys.argv = argv
    c = bench.config_dict(a, 1)
    assert (c["layers_in_flight"], c["sm_reserve"]) == (4, 8)
    assert c["seq_len"] == 16384 and c["query_buffer"] == 128 and c["compression_ratio"] == 0.75
    a.seq_len, a.n_queries, a.ratio = 131072, 512, 0.9
    lc = bench.long_config(a, 2)
    assert (lc["layers_in_flight"], lc["sm_reserve"]) == (3, 34)
    assert bench.long_config(a, 1)["layers_in_flight"] == 4
