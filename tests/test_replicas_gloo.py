"""Multi-rank host logic on CPU: world_size 2 over gloo (127.0.0.1).

Covers what the N>1 bench and a front-end scheduler do across ranks: LPT
sharding by KV bytes, max-over-ranks timing with summed work, the per-step
token/exit all-gather, and a rank failure surfacing as an error on its peer
(a rank that raises before the collective; the peer's short process-group
timeout ends its wait with an error instead of hanging)."""

from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from vllm_rlt_b200 import replicas, workloads


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, mode, queue):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        if mode == "reduce":
            times, work = replicas.max_over_ranks([10.0 + rank, 3.0 * (rank + 1)], 100 * (rank + 1))
            tokens = torch.tensor([rank * 10 + i for i in range(4)])
            flags = torch.tensor([1, 0, rank, 1], dtype=torch.uint8)
            gathered, exits = replicas.gather_step_outputs(tokens, flags)
            queue.put((rank, times, work, gathered.tolist(), exits.tolist()))
        elif mode == "fail":
            if rank == 1:
                raise RuntimeError("rank 1 fails before the step's collective")
            try:
                replicas.max_over_ranks([1.0], 1.0)
                queue.put((rank, "no error"))
            except Exception as error:  # the peer's timeout ends the wait
                queue.put((rank, type(error).__name__))
    except RuntimeError as error:
        queue.put((rank, str(error)))
    finally:
        if mode != "fail":
            dist.destroy_process_group()


def run_world(mode, world=2):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=60) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return sorted(results, key=lambda r: r[0])


def test_max_over_ranks_and_token_gather_world2():
    results = run_world("reduce")
    for rank, times, work, gathered, exits in results:
        assert times == [11.0, 6.0]  # max over ranks, per timed region
        assert work == 300.0  # summed over ranks
        assert gathered == [[0, 1, 2, 3], [10, 11, 12, 13]]
        assert exits == [[1, 0, 0, 1], [1, 0, 1, 1]]


def test_failed_rank_surfaces_as_error_on_peer():
    results = dict(run_world("fail"))
    assert "rank 1 fails" in results[1]
    assert results[0] != "no error"  # timed out / connection error, not a hang


def test_lpt_sharding_balances_kv_bytes():
    plan = workloads.config5_plan(seed=0, rows=512)
    kv = plan.context_lengths.astype(np.int64) * 16 * 128 * 4
    parts, imbalance = replicas.shard_requests(kv, 8)
    assert sorted(i for p in parts for i in p) == list(range(512))
    assert imbalance < 1.02
    # round-robin on the same skewed contexts is far less balanced
    rr = [list(range(r, 512, 8)) for r in range(8)]
    rr_loads = [kv[p].sum() for p in rr]
    assert max(rr_loads) / np.mean(rr_loads) > imbalance


def test_single_process_fallback():
    assert replicas.max_over_ranks([2.5], 7) == ([2.5], 7.0)
