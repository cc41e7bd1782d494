"""One rank of the world-size-2 CPU test of the multi-GPU path (launched by torch.distributed.run with gloo on
127.0.0.1 from tests/test_multirank.py): the rank takes its share of the batch with bench.rank_chunks, runs
each chunk through the C oracle's Timestral forward (a tiny random-init model), and the shares are gathered on
rank 0, which also checks bench.max_over_ranks. Rank 0 writes everything to the .npz named on the command line."""

import datetime
import os
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

SERIES, CHUNK, LENGTH = 24, 6, 128


def tiny_config():
    from jitcast_b200 import timestral as ts

    return ts.TimestralConfig(patch_size=16, d_model=128, num_heads=2, mlp_hidden_dim=256, block_schedule=["time"],
                              quantile_knots=ts.default_knots(9), block_size=4, context_length=LENGTH).validate()


def chunk_forecast(model, c0: int, n: int) -> np.ndarray:
    from jitcast_b200 import timestral as ts
    from jitcast_b200 import workloads

    x = workloads.sinusoid_noise(n, LENGTH, seed=c0)  # seeded by the chunk's first series, as bench.py does
    q, _ = model.predict_block(ts.BlockInput(x, np.ones_like(x, bool), np.arange(n, dtype=np.int32), 2), nthreads=1)
    return np.asarray(q, np.float32)


def main() -> int:
    import torch.distributed as dist

    import bench
    from jitcast_b200 import timestral as ts
    from oracle import timestral as ots

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    c = tiny_config()
    model = ots.Model(c, ts.random_checkpoint(c, seed=3))
    mine = {c0: chunk_forecast(model, c0, n) for c0, n in bench.rank_chunks(SERIES, CHUNK, world, rank)}
    shares = [None] * world
    dist.all_gather_object(shares, mine)
    slowest = bench.max_over_ranks(float(rank + 1), world, "cpu")
    if rank == 0:
        out = {f"chunk_{c0}": q for share in shares for c0, q in share.items()}
        np.savez(sys.argv[1], slowest=np.float64(slowest), **out)
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
