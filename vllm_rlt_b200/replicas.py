"""Request-sharded replicas: the only multi-GPU structure the path has.

The reference runs independent engine replicas (one per GPU) and routes whole
requests to them (README "4 independent replicas"; PD pools in
vllm_rlt/pd/engine.py:100-133); attention never exchanges data across GPUs.
This module holds the host logic for that layout:

* ``shard_requests`` -- greedy longest-processing-time assignment of requests
  to ranks by KV bytes (what bounds a decode step's time on a rank);
* ``max_over_ranks`` -- the step time of the job is the slowest rank's device
  time, and the work is the sum over ranks;
* ``gather_step_outputs`` -- the optional single front-end: one all-gather per
  decode step of every rank's sampled tokens and exit flags (a few KB, NCCL
  over NVLink on GPUs, gloo on CPU), so one scheduler sees all requests.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from .workloads import lpt_assign


def shard_requests(kv_bytes, world: int):
    """Per rank, the request indices it serves, and max/mean load imbalance."""
    parts = lpt_assign(kv_bytes, world)
    loads = np.array([sum(int(kv_bytes[i]) for i in p) for p in parts], dtype=np.float64)
    imbalance = float(loads.max() / loads.mean()) if loads.mean() > 0 else 1.0
    return parts, imbalance


def max_over_ranks(times_ms, work, device=None, group=None):
    """All-reduce MAX of per-rank times and SUM of per-rank work.

    ``times_ms`` is a sequence of floats (several timed regions at once),
    ``work`` a float; returns (list of max times, total work). With no process
    group initialised, returns the local values."""
    if not dist.is_available() or not dist.is_initialized():
        return [float(t) for t in times_ms], float(work)
    device = device if device is not None else torch.device("cpu")
    t = torch.tensor(list(times_ms), dtype=torch.float64, device=device)
    w = torch.tensor([float(work)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    dist.all_reduce(w, op=dist.ReduceOp.SUM, group=group)
    return t.tolist(), float(w.item())


def gather_step_outputs(tokens: torch.Tensor, exit_flags: torch.Tensor, group=None):
    """All-gather this step's sampled tokens (int64 [batch]) and exit flags
    (uint8 [batch]) of every rank; returns tensors [world, batch]."""
    world = dist.get_world_size(group)
    packed = torch.cat([tokens.to(torch.int64), exit_flags.to(torch.int64)])
    out = [torch.empty_like(packed) for _ in range(world)]
    dist.all_gather(out, packed, group=group)
    stacked = torch.stack(out)
    batch = tokens.shape[0]
    return stacked[:, :batch], stacked[:, batch:].to(torch.uint8)
