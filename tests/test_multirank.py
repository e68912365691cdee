"""The benchmark's multi-rank host logic, on two gloo ranks (CPU).

Under torchrun every rank decodes its own tree (weak scaling, no data-path
collective); the job's GB/s is the sum of the ranks' bytes over the slowest
rank's device time.  Two spawned ranks run ``bench.combine_ranks`` with
different times and byte counts and must agree on that result, and on each
rank's own time and bytes.  Every rank's tree has the same shape (suffix lengths
from the base seed) and its own K/V values (seed + rank).
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    import torch.distributed as dist
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        ms = [10.0, 12.5][rank]            # device time of the timed loop
        e2e_ms = [20.0, 15.0][rank]
        kv = [1_000_000_000, 3_000_000_000][rank]
        e2e = [500_000_000, 700_000_000][rank]
        out.put((rank, bench.combine_ranks(ms, e2e_ms, kv, e2e, torch.device("cpu"), world)))
    finally:
        dist.barrier()
        dist.destroy_process_group()


@pytest.mark.timeout(120)
def test_two_ranks_sum_bytes_over_slowest_time():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(out.get(timeout=90) for _ in range(2))
    for p in procs:
        p.join(timeout=30)
        assert p.exitcode == 0
    want = (4e9 / (12.5 / 1e3) / 1e9, 1.2e9 / (20.0 / 1e3) / 1e9, 12.5)
    for r in range(2):
        np.testing.assert_allclose(res[r][:3], want, rtol=1e-12)
        assert res[r][3] == [(10.0, 1e9), (12.5, 3e9)]


def test_ranks_decode_trees_of_one_shape():
    import sys
    sys.path.insert(0, ROOT)
    import bench
    # the suffix lengths come from the base seed on every rank (the values from seed + rank)
    a = bench.suffixes(4)
    assert len(a) == bench.NBR and a.min() >= bench.SUF_LO and a.max() <= bench.SUF_HI
    assert not np.array_equal(a, bench.suffixes(5))
    src = open(os.path.join(ROOT, "bench.py")).read()
    assert "build_tree(args.seed, device," in src and "value_seed=args.seed + rank" in src
