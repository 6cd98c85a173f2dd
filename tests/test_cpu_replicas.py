"""The multi-GPU plumbing on CPU: two `gloo` ranks (127.0.0.1) run the replica bookkeeping of
instantcua_b200.replicas that bench.py and a serving host use under torchrun -- process group from
the torchrun environment, round-robin session routing, max-over-ranks timing, the end-of-run gather
of token counts -- with no collective while decoding (a stand-in engine records what each rank was
asked to decode)."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from instantcua_b200 import replicas as R


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class _FakeEngine:
    """decode_batch / last_timing of Engine, recording the calls (no GPU)."""

    class _T:
        decode_ms = 0.0

    def __init__(self, rank):
        self.rank = rank
        self.calls = []
        self.last_timing = self._T()

    def decode_batch(self, sessions, steps, in_tokens=None):
        self.calls.append((list(sessions), steps, None if in_tokens is None else list(in_tokens)))
        self.last_timing.decode_ms = 100.0 + 25.0 * self.rank  # the slowest rank sets the job time
        out = np.full((len(sessions), steps), 7, np.int32)
        if len(sessions):
            out[0, steps - 1] = -1  # one session stopped early: counts exclude it
        return out


def _rank_main(rank, world, port, q):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port), "WORLD_SIZE": str(world),
                       "RANK": str(rank), "LOCAL_RANK": str(rank)})
    g = R.ReplicaGroup("gloo", timeout_s=60)
    assert (g.world, g.rank, g.local) == (world, rank, rank)
    ms_max = g.max_over_ranks(100.0 + 25.0 * rank)
    rate = R.aggregate_rate(64, g.world, ms_max / 1e3)
    job = list(range(10))
    eng = _FakeEngine(rank)
    toks = {gid: 1000 + gid for gid in job}
    res, total, job_s = R.decode_shard(eng, g, job, 3, in_tokens=toks)
    g.close()
    q.put((rank, ms_max, rate, eng.calls, sorted(res), total, job_s, R.local_sessions(job, g)))


@pytest.mark.parametrize("world", [2])
def test_replica_routing_and_timing_over_gloo(world):
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
    seen = []
    for rank, ms_max, rate, calls, got, total, job_s, mapping in res:
        assert ms_max == slowest
        assert rate == pytest.approx(world * 64 / (slowest / 1e3))
        mine = list(range(10))[rank::world]
        assert got == mine and list(mapping) == mine and list(mapping.values()) == list(range(len(mine)))
        ((sess, steps, toks),) = calls  # one batched call per rank, on engine indices 0..n-1
        assert sess == list(range(len(mine))) and steps == 3 and toks == [1000 + g for g in mine]
        assert total == 10 * 3 - world  # every rank's tokens, minus one stopped session per rank
        assert job_s == pytest.approx(slowest / 1e3)
        seen += got
    assert sorted(seen) == list(range(10))


def test_shard_sessions_round_robin():
    ids = [11, 12, 13, 14, 15, 16, 17]
    shards = [R.shard_sessions(ids, 3, r) for r in range(3)]
    assert shards == [[11, 14, 17], [12, 15], [13, 16]]
    assert sorted(sum(shards, [])) == ids
    assert all(R.owner_of(i, 3) == r for r in range(3) for i in range(r, len(ids), 3))
    with pytest.raises(ValueError):
        R.shard_sessions(ids, 2, 2)


def test_single_process_needs_no_group():
    env = {k: os.environ.pop(k) for k in ("WORLD_SIZE", "RANK", "LOCAL_RANK") if k in os.environ}
    try:
        g = R.ReplicaGroup("gloo")
        assert g.dist is None and (g.world, g.rank) == (1, 0)
        assert g.max_over_ranks(3.5) == 3.5 and g.gather(5, 2.0) == (5, 2.0)
        assert g.shard([4, 5]) == [4, 5]
        g.close()
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
