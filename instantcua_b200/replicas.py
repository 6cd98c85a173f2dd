"""Replica serving on the GPUs of one node: one engine per GPU, sessions sharded round-robin.

The reference engine is single-device (Sources/Engine/Engine.swift:54-65: one MTLDevice, one
queue).  The 2B model fits on every B200 and one session's token loop never needs a second GPU,
so the multi-GPU form of this engine is N independent replicas: each process (one per GPU, the
torchrun environment) owns an engine with its own weights and KV caches and serves its share of
the sessions.  The process group carries only barriers and the end-of-run gather of token counts
and device times; nothing crosses GPUs on the decode path, and no collective runs inside a step.

    group = ReplicaGroup()                       # RANK / WORLD_SIZE / LOCAL_RANK from torchrun
    mine = group.shard(range(n_sessions))        # round-robin: sessions rank, rank + N, ...
    ... decode `mine` on the engine of GPU group.local ...
    total_tokens, job_s = group.gather(tokens_done, seconds)
"""
from __future__ import annotations

import datetime
import os


def shard_sessions(session_ids, world: int, rank: int) -> list:
    """Round-robin share of ``session_ids`` for ``rank`` of ``world`` replicas (order kept)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    return list(session_ids)[rank::world]


def owner_of(session_index: int, world: int) -> int:
    """The replica that serves the session at position ``session_index`` of the id list."""
    return session_index % world


class ReplicaGroup:
    """The replicas of one job.  ``backend``: "gloo" keeps the bookkeeping on the host (the
    serving default); "nccl" puts barriers and timing reductions on the GPUs (the benchmark, whose
    barriers bracket device-timed regions).  A single process (WORLD_SIZE unset or 1) needs no
    process group."""

    def __init__(self, backend: str = "gloo", timeout_s: int = 600):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.backend = backend
        self.dist = None
        if self.world > 1:
            import torch
            import torch.distributed as tdist

            kw = {}
            if backend == "nccl":
                torch.cuda.set_device(self.local)
                kw["device_id"] = torch.device("cuda", self.local)
            tdist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
            self.dist = tdist

    def shard(self, session_ids) -> list:
        return shard_sessions(session_ids, self.world, self.rank)

    def _device(self):
        return f"cuda:{self.local}" if self.backend == "nccl" else "cpu"

    def barrier(self) -> None:
        if self.dist is not None:
            self.dist.barrier()

    def max_over_ranks(self, value: float) -> float:
        """Max of a per-replica value (the slowest replica sets the job time)."""
        if self.dist is None:
            return value
        import torch

        t = torch.tensor([value], dtype=torch.float64, device=self._device())
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather(self, units: int, seconds: float) -> tuple:
        """(units summed over replicas, the slowest replica's seconds)."""
        if self.dist is None:
            return units, seconds
        import torch

        t = torch.tensor([float(units)], dtype=torch.float64, device=self._device())
        self.dist.all_reduce(t, op=self.dist.ReduceOp.SUM)
        return int(t.item()), self.max_over_ranks(seconds)

    def close(self) -> None:
        if self.dist is not None:
            self.dist.barrier()
            self.dist.destroy_process_group()
            self.dist = None


def aggregate_rate(units_per_rank: int, world: int, max_time_s: float) -> float:
    """Whole-job rate when every replica processes the same number of units."""
    return world * units_per_rank / max_time_s


def local_sessions(global_ids, group: ReplicaGroup) -> dict:
    """{global session id: engine session index} for this replica's share (indices 0, 1, ... in the
    order of the share)."""
    return {g: i for i, g in enumerate(group.shard(global_ids))}


def decode_shard(engine, group: ReplicaGroup, global_ids, steps: int, in_tokens=None):
    """Decodes this replica's share of the job's sessions together (one batched call on its own
    engine; the sessions must have been prefilled or injected at the indices of
    :func:`local_sessions`) and gathers the job totals on the host.

    ``in_tokens``: None to continue every session from its last token, or {global id: token}.
    Returns ({global id: generated tokens (list, -1 after an EOS)}, job tokens, job seconds), where
    job tokens counts every replica's generated tokens and job seconds is the slowest replica's
    device time of its call.  No collective runs during decoding."""
    mine = group.shard(global_ids)
    results, n_tok, seconds = {}, 0, 0.0
    if mine:
        idx = list(range(len(mine)))
        toks = None if in_tokens is None else [int(in_tokens[g]) for g in mine]
        import numpy as np

        out = engine.decode_batch(idx, steps, in_tokens=None if toks is None else np.asarray(toks, np.int32))
        seconds = engine.last_timing.decode_ms / 1e3
        for g, row in zip(mine, out):
            results[g] = [int(t) for t in row]
            n_tok += int((row >= 0).sum())
    total, job_s = group.gather(n_tok, seconds)
    return results, total, job_s
