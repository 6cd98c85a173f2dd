"""The multi-GPU plumbing of bench.py on CPU: two `gloo` ranks (127.0.0.1) run the same replica
bookkeeping the GPU run does under torchrun -- process group from the torchrun environment,
max-over-ranks timing, whole-job rate -- with no data-path collective."""
import os
import socket

import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "WORLD_SIZE": str(world),
                       "RANK": str(rank), "LOCAL_RANK": str(rank)})
    import bench

    dist, w, r, local = bench.init_replicas("gloo")
    assert (w, r, local) == (world, rank, rank)
    ms = 100.0 + 25.0 * rank  # the slowest rank sets the job time
    ms_max = bench.max_over_ranks(dist, ms, device="cpu")
    rate = bench.aggregate_rate(64, w, ms_max / 1e3)
    dist.barrier()
    dist.destroy_process_group()
    q.put((rank, ms_max, rate))


@pytest.mark.parametrize("world", [2])
def test_replica_timing_over_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    res = sorted(q.get(timeout=10) for _ in range(world))
    slowest = 100.0 + 25.0 * (world - 1)
    for rank, ms_max, rate in res:
        assert ms_max == slowest
        assert rate == pytest.approx(world * 64 / (slowest / 1e3))


def test_single_process_needs_no_group():
    import bench

    env = {k: os.environ.pop(k) for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK") if k in os.environ}
    try:
        dist, w, r, local = bench.init_replicas("gloo")
        assert dist is None and (w, r) == (1, 0)
        assert bench.max_over_ranks(None, 3.5) == 3.5
    finally:
        os.environ.update(env)
