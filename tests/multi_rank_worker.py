"""One rank of the world-size-2 host test of bench.py's multi-GPU logic (gloo, CPU).

Launched by tests/test_multi_rank.py through torch.distributed.run. Each rank
reports a different step time; the test checks that every rank sees the
slowest one, that the streams' seeds are disjoint across ranks, and that the
whole-job rate counts every rank's streams.
"""
import json
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch.distributed as dist  # noqa: E402

import bench  # noqa: E402

STREAMS, STEPS = 4, 5


def main():
    r = bench.Ranks("gloo", timeout_s=60)
    r.barrier()
    seconds = 1.0 + 0.5 * r.rank
    slowest = r.max(seconds)
    seeds = bench.stream_seeds(r.rank, STREAMS)
    gathered = [None] * r.world
    dist.all_gather_object(gathered, seeds)
    rate = bench.job_rate(r.world, STREAMS, STEPS, slowest)
    r.barrier()
    if r.rank == 0:
        print(json.dumps({"world": r.world, "slowest": slowest, "seeds": gathered, "rate": rate}), flush=True)
    r.close()
    return 0


if __name__ == "__main__":
    sys.exit(main())
