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


REQUIRED_KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                 "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


def _reference_line(env_extra, gpus):
    import json
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ)
    env.update(env_extra)
    r = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--gpus", str(gpus), "--steps", "1",
                        "--warmup", "0"], cwd=root, env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    return [json.loads(l) for l in lines]


def test_reference_arm_line_matches_the_measured_arm():
    """`bench.py --impl reference` (the reference's CPU path, run on the host) prints one line with
    the measured arm's metric, unit, direction and workload, the launch's GPU count, and its own
    cpu_baseline / e2e blocks; warm-up is raised to the 3-step minimum."""
    import bench

    (line,) = _reference_line({"RANK": "0"}, 2)
    assert REQUIRED_KEYS <= set(line)
    assert line["impl"] == "reference" and line["metric"] == bench.METRIC and line["unit"] == "tokens/s"
    assert line["higher_is_better"] is True and line["n_gpus"] == 2 and line["warmup"] >= 3
    assert line["config"]["workload"] == bench.WORKLOAD
    assert line["value"] > 0 and line["cpu_baseline"]["value"] == line["value"]
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_print_nothing():
    """Under torchrun only rank 0 runs the CPU reference; the other ranks exit 0 without output."""
    assert _reference_line({"RANK": "1"}, 2) == []
