"""One rank of the two-GPU head-sharded check in test_gpu_sharded.py:
compresses the test layer over NCCL and saves this rank's outputs to
<out_dir>/rank<r>.pt.  Launched by torch.distributed.run."""

import os
import sys
from datetime import timedelta

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import test_gpu_sharded as T  # noqa: E402  (the layer definition shared with the test)


def main(out_dir):
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    try:
        from core_b200 import engine, ops
        from core_b200.sharded import DistExchange, HeadShard, ShardWeights, compress_layer_sharded
        q, k, v, w, n_kept = T._layer(dev)
        G = T.HQ // T.HKV
        sh = HeadShard(rank, world, T.HKV, T.L)
        inp = dict(q=q[:, sh.h0 * G:sh.h1 * G].contiguous(), keys=k[:, sh.h0:sh.h1].contiguous(),
                   values=v[:, sh.h0:sh.h1].contiguous())
        wt = ShardWeights.prepare(sh, geometry=w["geometry"], prototypes=w["prototypes"],
                                  hadamard=w["hadamard"], mlp_params=w["mlp"], theta=w["theta"],
                                  n_q_heads=T.HQ, device=dev)
        owner = HeadShard.owner(T.LAYER, world)
        mem = engine.MemoryState.zeros(1, T.D_MEM, T.HKV * 128, dev) if rank == owner else None
        (o,) = compress_layer_sharded(DistExchange(), [sh], [inp], [wt], layer_idx=T.LAYER,
                                      n_kept=n_kept, positions=torch.arange(T.L, device=dev),
                                      original_length=T.L, is_prefill=False, memory=mem,
                                      keep_features=True)
        ops.status(dev)
        res = dict(keep=o["keep"].cpu(), features=o["features"].cpu(), keys=o["keys"].cpu())
        if mem is not None:
            res["M"] = mem.M.cpu()
        torch.save(res, os.path.join(out_dir, f"rank{rank}.pt"))
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
