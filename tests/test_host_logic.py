"""Host-side behaviour that needs no GPU: argument validation and error
convention (mirroring vllm_rlt/kernels/paged_attention.py:47-50 and
flash_attention.py:55-57), the backend surface, and the workload plans."""

from __future__ import annotations

import math
from types import SimpleNamespace

import numpy as np
import pytest
import torch

import vllm_rlt_b200 as rb
from vllm_rlt_b200 import backend as backend_mod
from vllm_rlt_b200 import workloads


def test_cpu_tensors_are_rejected_explicitly():
    q = torch.zeros(2, 4, 128)
    k = torch.zeros(3, 16, 4, 128)
    t = torch.zeros(2, 1, dtype=torch.int32)
    n = torch.ones(2, dtype=torch.int32)
    with pytest.raises(ValueError, match="requires a CUDA device"):
        rb.b200_paged_attention(q, k, k, t, n)
    # the device check comes first, as in the reference's dispatcher
    with pytest.raises(ValueError, match="requires a CUDA device"):
        rb.b200_paged_attention(torch.zeros(2, 4, 300), k, k, t, n)
    with pytest.raises(ValueError, match="NVIDIA CUDA device"):
        rb.B200PagedAttention(torch.device("cpu"), torch.bfloat16, 128, 16)


def test_backend_rejects_other_architectures(monkeypatch):
    monkeypatch.setattr(torch.version, "hip", None)
    monkeypatch.setattr(torch.cuda, "get_device_capability", lambda device=None: (9, 0))
    with pytest.raises(ValueError, match="sm_100a"):
        rb.B200PagedAttention(torch.device("cuda"), torch.bfloat16, 128, 16)
    with pytest.raises(ValueError, match="float32, float16 or bfloat16"):
        rb.B200PagedAttention(torch.device("cuda"), torch.int8, 128, 16)


def test_backend_surface_and_install(monkeypatch):
    monkeypatch.setattr(torch.version, "hip", None)
    monkeypatch.setattr(torch.cuda, "get_device_capability", lambda device=None: (10, 0))
    attention = rb.B200PagedAttention(torch.device("cuda"), torch.bfloat16, 128, 16)
    assert attention.generation == 4  # receives packed prefill from the unchanged caller
    assert attention.info["backend"] == "b200" and attention.info["arch"] == "sm_100a"
    cache = SimpleNamespace(device=torch.device("cuda"), dtype=torch.bfloat16, head_dim=128,
                            block_size=16, attention=None, attention_info=None,
                            _write_prepared=None)
    proxy = type("Proxy", (), {"_write_prepared": None})
    got = backend_mod.install(cache, graph_proxy_class=proxy)
    assert cache.attention is got and cache.attention_info == got.info
    assert callable(cache._write_prepared) and callable(proxy._write_prepared)


def test_config1_plan_shape():
    plan = workloads.config1_plan(0)
    assert plan.num_rows == 8 and plan.planes == 4 and plan.num_blocks == 1024
    assert all(1 <= c <= 512 for c in plan.context_lengths)
    used = [p for t in plan.plane_tables for plane in t for p in plane]
    assert len(used) == len(set(used))  # every page has one owner


def test_config2_plan_distribution():
    plan = workloads.config2_plan(0)
    lengths = plan.context_lengths
    assert plan.num_rows == 256 and lengths.min() >= 128 and lengths.max() <= 8192
    assert 1500 < np.median(lengths) < 2800
    tables = plan.block_tables()
    assert tables.shape == (256, math.ceil(lengths.max() / 16))
    for r in range(0, 256, 37):
        used = math.ceil(int(lengths[r]) / 16)
        assert (tables[r, :used] >= 0).all() and (tables[r, used:] == -1).all()


def test_decode_bytes_formula():
    # K and V once per token per KV head, q and out once, tables and lengths
    got = rb.decode_bytes([16, 17], 16, 16, 128, 2, page=16)
    assert got == 33 * 16 * 128 * 2 * 2 + 2 * 2 * 16 * 128 * 2 + 3 * 4 + 2 * 4
