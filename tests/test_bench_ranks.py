"""bench.py's multi-GPU host logic on CPU: two gloo ranks (request-parallel replicas, no
data-path collective) combine their per-frame times as the max over ranks, and the job's
frames/s counts every rank's frames."""
import os
import socket

import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", init_method="env://", rank=rank, world_size=world)
    ms, e2e = [2.5, 3.0][rank], [2.9, 2.7][rank]
    res = bench.combine_ranks(ms, e2e, world, dist, "cpu")
    out[rank] = res
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_combination():
    world = 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_rank, args=(world, port, out), nprocs=world, join=True)
        res = dict(out)
    for r in range(world):
        ms, e2e_ms, value, e2e_value = res[r]
        assert ms == 3.0 and e2e_ms == 2.9           # the slowest rank sets the job time
        assert abs(value - 2 * 1000.0 / 3.0) < 1e-9   # frames of both ranks
        assert abs(e2e_value - 2 * 1000.0 / 2.9) < 1e-9


def test_single_rank_is_identity():
    assert bench.combine_ranks(2.0, 4.0, 1, None, "cpu") == (2.0, 4.0, 500.0, 250.0)
