"""Host-side behaviour that needs no GPU: argument validation and error
convention (mirroring vllm_rlt/kernels/paged_attention.py:47-50 and
flash_attention.py:55-57), the backend surface, and the workload plans."""

from __future__ import annotations

import math
import sys
from pathlib import Path
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


def test_backend_rejects_head_dims_above_256(monkeypatch):
    """The reference's dispatcher refuses head_dim > 256 before any launch
    (vllm_rlt/kernels/paged_attention.py:47-50); so does the backend, on an
    sm_100a device."""
    monkeypatch.setattr(torch.version, "hip", None)
    monkeypatch.setattr(torch.cuda, "get_device_capability", lambda device=None: (10, 0))
    with pytest.raises(ValueError, match="head_dim"):
        rb.B200PagedAttention(torch.device("cuda"), torch.bfloat16, 320, 16)
    with pytest.raises(ValueError, match="head_dim"):
        rb.B200PagedAttention(torch.device("cuda"), torch.bfloat16, 0, 16)


def test_backend_surface(monkeypatch):
    monkeypatch.setattr(torch.version, "hip", None)
    monkeypatch.setattr(torch.cuda, "get_device_capability", lambda device=None: (10, 0))
    attention = rb.B200PagedAttention(torch.device("cuda"), torch.bfloat16, 128, 16)
    assert attention.generation == 4  # receives packed prefill from the unchanged caller
    assert attention.info["backend"] == "b200" and attention.info["arch"] == "sm_100a"


REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _reference_cache_manager():
    if not (REF / "vllm_rlt" / "__init__.py").exists():
        pytest.skip("the unmodified reference is not installed under baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from vllm_rlt.core.kv_cache_manager import KVCacheManager
    from vllm_rlt.worker import cuda_graph

    return KVCacheManager, cuda_graph


def test_install_runs_the_reference_write_body_with_a_routed_page_write(monkeypatch):
    """install() keeps the reference's own _write_prepared (validation, order of
    checks, written-prefix bookkeeping) and replaces only its K/V index-puts by
    one page-write call with the same addresses; here the call is recorded and
    applied on the CPU so it can be compared with the reference's own write."""
    KVCacheManager, cuda_graph = _reference_cache_manager()
    monkeypatch.setattr(torch.version, "hip", None)
    monkeypatch.setattr(torch.cuda, "get_device_capability", lambda device=None: (10, 0))
    calls = []

    def recording_write(kc, vc, layer, blocks, offsets, k, v):
        calls.append((layer, blocks.tolist(), offsets.tolist()))
        kc[blocks, layer, offsets] = k[: len(blocks)]
        vc[blocks, layer, offsets] = v[: len(blocks)]

    monkeypatch.setattr(backend_mod, "write_kv", recording_write)

    def make():
        torch.manual_seed(3)
        cache = KVCacheManager(num_layers=2, num_kv_heads=1, head_dim=4, num_blocks=32,
                               block_size=2, max_loops=4)
        cache.key_cache.zero_()
        cache.value_cache.zero_()
        cache.allocate("a", 5)
        cache.allocate("b", 3)
        return cache

    plain, routed = make(), make()
    # The attention object needs CUDA, so point install at a CPU pool by
    # swapping the device only for the backend's constructor.
    monkeypatch.setattr(backend_mod, "B200PagedAttention",
                        lambda *a, **k: SimpleNamespace(info={"backend": "b200"}))
    backend_mod.install(routed, graph_proxy_class=None)
    ids, depths, positions = ["a"] * 3 + ["b"] * 2, [0, 0, 0, 2, 2], [0, 1, 2, 0, 1]
    k = torch.randn(5, 1, 4)
    v = torch.randn(5, 1, 4)
    for cache in (plain, routed):
        batch = cache._prepare_batch(ids, depths, positions)
        cache._write_prepared(1, batch, k, v)
        read_only = cache._prepare_batch(ids[:1], depths[:1], positions[:1], for_write=False)
        with pytest.raises(ValueError, match="read-only"):
            cache._write_prepared(1, read_only, k[:1], v[:1])
        with pytest.raises(ValueError, match="layer"):
            cache._write_prepared(2, batch, k, v)
        with pytest.raises(ValueError, match="KV heads"):
            cache._write_prepared(1, batch, torch.randn(5, 2, 4), v)
    assert len(calls) == 1 and calls[0][0] == 1
    assert torch.equal(plain.key_cache, routed.key_cache)
    assert torch.equal(plain.value_cache, routed.value_cache)
    for name in ("a", "b"):
        want = [[w.prefix for w in plane] for plane in plain._allocations[name].written]
        got = [[w.prefix for w in plane] for plane in routed._allocations[name].written]
        assert want == got


def test_install_routes_the_graph_proxy_write_once(monkeypatch):
    KVCacheManager, cuda_graph = _reference_cache_manager()
    calls = []
    monkeypatch.setattr(backend_mod, "write_kv", lambda *args: calls.append(args[2]))
    monkeypatch.setattr(backend_mod, "B200PagedAttention",
                        lambda *a, **k: SimpleNamespace(info={"backend": "b200"}))
    original = cuda_graph._DeviceCache._write_prepared
    cache = KVCacheManager(num_layers=2, num_kv_heads=1, head_dim=4, num_blocks=16,
                           block_size=2, max_loops=4)
    try:
        backend_mod.install(cache, graph_proxy_class=cuda_graph._DeviceCache)
        backend_mod.install(cache, graph_proxy_class=cuda_graph._DeviceCache)
        assert cuda_graph._DeviceCache._rlt_original_write is original
        cache.allocate("a", 2)
        batch = cache._prepare_batch(["a"], [0], [1])
        proxy = cuda_graph._DeviceCache(cache)
        proxy._write_prepared(1, batch, torch.ones(1, 1, 4), torch.ones(1, 1, 4))
        assert calls == [1]
    finally:
        backend_mod.uninstall_graph_proxy(cuda_graph._DeviceCache)
    assert cuda_graph._DeviceCache._write_prepared is original


def test_routing_adapters_keep_the_triton_argument_order(monkeypatch):
    """The launch adapters accept ``kernel[grid](...)`` with the reference's
    argument lists (vllm_rlt/worker/async_state.py:59-75, :99-111,
    vllm_rlt/worker/model_runner.py:543-557, vllm_rlt/worker/prefill_metadata.py:
    53-86) and forward the right values."""
    seen = {}
    monkeypatch.setattr(backend_mod.routing, "metadata",
                        lambda *a: seen.__setitem__("metadata", a[8:]))
    monkeypatch.setattr(backend_mod.routing, "gather",
                        lambda *a: seen.__setitem__("gather", a[3:]))
    monkeypatch.setattr(backend_mod.routing, "scatter",
                        lambda *a: seen.__setitem__("scatter", a[3:]))
    monkeypatch.setattr(backend_mod.cache_ops, "finalize",
                        lambda *a, rows: seen.__setitem__("finalize", rows))
    monkeypatch.setattr(backend_mod.prefill_metadata, "stage_prefill",
                        lambda *a: seen.__setitem__("stage", a[3:]))
    monkeypatch.setattr(backend_mod.prefill_metadata, "expand_prefill",
                        lambda *a: seen.__setitem__("expand", a[5:]))
    launches = {**backend_mod.ROUTING_LAUNCHES, **backend_mod.PREFILL_LAUNCHES}
    t = torch.zeros
    tables = t((3, 4, 8), dtype=torch.int32)
    launches["metadata_kernel"][(6,)](t(6, 3), tables, *[t(6)] * 5, t(6, 8), 5, 6, 8, 16, 4, 3,
                                      256)
    assert seen["metadata"] == (5, 6, 16, 4, 3)
    pool, out = t(3, 10), t(6, 10)
    launches["gather_kernel"][(6, 1)](pool, t(6), out, 4, 10, 10, 10, 256)
    assert seen["gather"] == (4, 6)
    launches["scatter_kernel"][(4, 1)](out, t(6), pool, 10, 10, 10, 256)
    assert seen["scatter"] == (4,)
    kc = t(5, 2, 16, 2, 8)
    launches["finalize_kernel"][(3, 4, 1)](t(3, 3), tables, kc, kc, 8, 4, 16, 2, 16,
                                           *kc.stride()[:3], 256)
    assert seen["finalize"] == 3
    launches["stage_prefill"][(1,)](t(9), t(9), t(9), 9, 256)
    assert seen["stage"] == (9,)
    launches["expand_prefill"][(1,)](t(4), t(4), t(2, 8), t(4), t(4), 4, 8, 16, 256)
    assert seen["expand"] == (4, 8, 16)
    with pytest.raises(ValueError, match="WIDTH"):
        launches["metadata_kernel"][(6,)](t(6, 3), tables, *[t(6)] * 5, t(6, 8), 5, 6, 7, 16,
                                          4, 3, 256)


def test_install_routing_restores_module_attributes():
    module = SimpleNamespace(**{name: object() for name in backend_mod.ROUTING_LAUNCHES})
    originals = dict(vars(module))
    restore = backend_mod.install_routing(module)
    assert all(isinstance(getattr(module, n), backend_mod._GridLaunch) for n in originals)
    restore()
    assert dict(vars(module)) == originals


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
