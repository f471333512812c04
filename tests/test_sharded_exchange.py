"""Host logic of the head-sharded layer step on CPU: the rank partition, and
the torch.distributed collectives (world_size-2 gloo groups) against the
single-process emulation that the GPU tests use."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_partition_covers_heads_and_keys():
    from core_b200.sharded import HeadShard
    for world, L in ((1, 5), (2, 333), (4, 131072), (8, 4097), (8, 5)):
        shards = [HeadShard(r, world, 8, L) for r in range(world)]
        heads = [h for s in shards for h in range(s.h0, s.h1)]
        assert heads == list(range(8))
        keys = [k for s in shards for k in range(s.k0, s.k1)]
        assert keys == list(range(L))                       # every key in exactly one range
        assert all(s.padded >= L and s.padded == world * s.chunk for s in shards)
        assert all(0 <= s.n_keys <= s.chunk for s in shards)
    assert [HeadShard.owner(l, 4) for l in range(6)] == [0, 1, 2, 3, 0, 1]
    with pytest.raises(ValueError):
        HeadShard(0, 3, 8, 100)                             # 8 heads do not split over 3 ranks


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(world, rank):
    g = torch.Generator().manual_seed(100 + rank)
    return dict(
        a2a=torch.randn(world * 3, 5, generator=g),
        rs=torch.randn(world * 4, 2, generator=g, dtype=torch.float64),
        ar=torch.randint(0, 50, (64,), generator=g, dtype=torch.int32),
        ag=torch.randn(7, generator=g),
        gt=torch.randn(2, 3, 4, generator=g),
    )


def _worker(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    from core_b200.sharded import DistExchange
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ex = DistExchange()
        x = _inputs(world, rank)
        res = dict(
            a2a=ex.all_to_all([x["a2a"]])[0],
            rs=ex.reduce_scatter_sum([x["rs"]])[0],
            ar=ex.all_reduce_sum([x["ar"]])[0],
            ag=ex.all_gather([x["ag"]])[0],
            gt=ex.gather_to(1, [x["gt"]])[0],
        )
        out[rank] = {k: (None if v is None else v.clone()) for k, v in res.items()}
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_dist_exchange_matches_local_emulation():
    from core_b200.sharded import LocalExchange
    world = 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
        got = dict(out)
    ex = LocalExchange(world)
    xs = [_inputs(world, r) for r in range(world)]
    want = dict(
        a2a=ex.all_to_all([x["a2a"] for x in xs]),
        rs=ex.reduce_scatter_sum([x["rs"] for x in xs]),
        ar=ex.all_reduce_sum([x["ar"] for x in xs]),
        ag=ex.all_gather([x["ag"] for x in xs]),
        gt=ex.gather_to(1, [x["gt"] for x in xs]),
    )
    for r in range(world):
        for k in ("a2a", "ar", "ag"):
            assert torch.equal(got[r][k], want[k][r]), (r, k)
        assert torch.allclose(got[r]["rs"], want["rs"][r], rtol=0, atol=1e-12)
        assert (got[r]["gt"] is None) == (want["gt"][r] is None)
        if r == 1:
            assert torch.equal(got[r]["gt"], want["gt"][r])
    # the all-to-all hands rank r the r-th chunk of every rank, in rank order
    assert torch.equal(want["a2a"][1][0], xs[0]["a2a"][3:6])
    assert torch.equal(want["a2a"][0][1], xs[1]["a2a"][0:3])


def _leaver(rank, world, port, out):
    """Rank 1 leaves between layers; rank 0's next collective must end with
    an error within the group's short timeout instead of waiting for good."""
    import datetime
    import sys
    import time
    sys.path.insert(0, ROOT)
    from core_b200.sharded import DistExchange
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    ex = DistExchange()
    x = torch.ones(world * 4, 3)
    ex.all_to_all([x])                     # layer 0: both ranks
    if rank == 1:
        out[rank] = "left"
        os._exit(0)                        # leaves between layers, nothing in flight
    t0 = time.perf_counter()
    try:
        ex.all_to_all([x])                 # layer 1: the peer is gone
        out[rank] = "no error"
    except Exception as e:  # noqa: BLE001 - any collective error ends the wait
        out[rank] = f"error after {time.perf_counter() - t0:.1f} s: {type(e).__name__}"
    os._exit(0)


def test_peer_leaving_ends_the_next_collective_with_an_error():
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        procs = [ctx.Process(target=_leaver, args=(r, world, port, out)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=60)
        alive = [p.is_alive() for p in procs]
        for p in procs:
            if p.is_alive():
                p.kill()
        res = dict(out)
    assert not any(alive), "a rank was still waiting"
    assert res.get(1) == "left"
    assert str(res.get(0, "")).startswith("error after"), res
