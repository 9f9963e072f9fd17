"""The reference's own callers running on the B200 backend.

The unmodified reference (installed under baseline/_ref) builds its engine,
KV cache manager, model runner and CUDA-graph capture as usual; ``install``
then puts the sm_100a backend into the cache manager and routes the page
writes, and ``install_routing`` replaces the runner's Triton launches. The
scenarios are the reference's own integration tests, rerun on this backend:

* tests/test_cuda_graph.py:24-71 -- graph replay equals eager, requests reused
  (here with bit-identical KV pools between the two runs as well);
* tests/test_flash_attention.py:92-132 -- sync/async/multi-stream engines
  with trace exits agree with one another and with the reference's torch
  backend (vllm_rlt/kernels/paged_attention.py:12-36);
* tests/test_prepared_kv.py:30-82 -- fragmented mixed-depth rows equal dense
  attention, protected pages untouched;
* tests/test_prepared_kv.py:85-172 -- the cache manager's validation (stale
  batches, read-only batches, uninitialised prefixes) still guards the
  routed page write;
* tests/test_flash_attention.py:146-208 -- packed prefill with ragged
  prefixes at unequal depths, ragged strided decode, batch invariance.
"""

from __future__ import annotations

import sys
from dataclasses import replace
from pathlib import Path

import pytest
import torch

import vllm_rlt_b200 as rb
from gpu_helpers import to_numpy
from helpers import assert_close
from vllm_rlt_b200 import backend as backend_mod

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"
DTYPE_NAMES = {torch.float32: "f32", torch.float16: "f16", torch.bfloat16: "bf16"}


def _reference():
    if not (REF / "vllm_rlt" / "__init__.py").exists():
        pytest.skip("the unmodified reference is not installed under baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    import vllm_rlt  # noqa: F401

    return vllm_rlt


@pytest.fixture
def ref():
    """The reference package; the graph proxy class and the routing modules
    are restored after the test."""
    vllm_rlt = _reference()
    from vllm_rlt.kernels import prefill_metadata, routing
    from vllm_rlt.worker import cuda_graph

    restores = []

    def b200(cache):
        attention = rb.install(cache, graph_proxy_class=cuda_graph._DeviceCache)
        restores.append(backend_mod.install_routing(routing, prefill_metadata))
        return attention

    vllm_rlt.b200 = b200
    yield vllm_rlt
    for restore in reversed(restores):
        restore()
    backend_mod.uninstall_graph_proxy(cuda_graph._DeviceCache)
    del vllm_rlt.b200


def _tiny_model(ref, head_dim, seed):
    from vllm_rlt.models import OuroConfig, OuroForCausalLM

    torch.manual_seed(seed)
    config = replace(OuroConfig.tiny(), head_dim=head_dim)
    return OuroForCausalLM(config).to("cuda", torch.bfloat16)


def _engine(ref, model, *, layout, mode="sync", static=False, graphs=False, backend="triton",
            exit_config=None, blocks=64, b200=True):
    from vllm_rlt import CacheConfig, ExecutionConfig, SchedulerConfig
    from vllm_rlt.engine.llm_engine import LLMEngine

    engine = LLMEngine(
        model,
        cache_config=CacheConfig(num_blocks=blocks, block_size=16, layout=layout),
        scheduler_config=SchedulerConfig(max_num_seqs=3, max_num_batched_tokens=8,
                                         prefill_chunk_size=4),
        execution_config=ExecutionConfig(async_scheduling=mode != "sync",
                                         multi_stream=mode == "multi", static_buffers=static,
                                         pad_to_power_of_two=static, cuda_graphs=graphs),
        exit_config=exit_config,
        attention_backend=backend,
    )
    # the pools come from torch.empty; zero them so unwritten slots compare equal
    engine.cache_manager.key_cache.zero_()
    engine.cache_manager.value_cache.zero_()
    if b200:
        attention = ref.b200(engine.cache_manager)
        assert engine.cache_manager.attention is attention
        assert engine.cache_manager.attention.info["arch"] == "sm_100a"
    return engine


def _drain(engine, limit=400):
    finished = {}
    for _ in range(limit):
        if not engine.has_unfinished_requests():
            break
        for out in engine.step():
            if out.finished:
                finished[out.request_id] = (tuple(out.token_ids), tuple(out.exit_depths))
    assert not engine.has_unfinished_requests()
    return finished


def _launch_counts():
    launches = {**backend_mod.ROUTING_LAUNCHES, **backend_mod.PREFILL_LAUNCHES}
    return {name: adapter.calls for name, adapter in launches.items()}


@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("layout", ["last_exited", "shared"])
@pytest.mark.parametrize("mode", ["sync", "async", "multi"])
@pytest.mark.parametrize("static", [False, True])
def test_reference_graph_replay_matches_eager_on_b200(ref, head_dim, layout, mode, static):
    """tests/test_cuda_graph.py:24-71 on the B200 backend, plus identical pools."""
    from vllm_rlt import ExitConfig, SamplingParams

    model = _tiny_model(ref, head_dim, 321)
    outputs, pools = [], []
    before = _launch_counts()
    for graphs in (False, True):
        engine = _engine(ref, model, layout=layout, mode=mode, static=static, graphs=graphs,
                         exit_config=ExitConfig("ouro_delayed"))
        rounds = []
        for reuse in range(2):
            for i in range(3):
                engine.add_request(str(i), [2 + i, 3, 4] * (i + 1 + reuse),
                                   SamplingParams(max_tokens=5 + i, min_loops=2,
                                                  exit_threshold=0.2, ignore_eos=True))
            rounds.append(_drain(engine))
            assert engine.cache_manager.num_used_blocks == 0
        if graphs:
            assert engine.model_runner.graphs.captures > 0
            assert engine.model_runner.graphs.replays > engine.model_runner.graphs.captures
        torch.cuda.synchronize()
        assert engine.cache_manager.attention.check_errors() == []
        outputs.append(rounds)
        pools.append((engine.cache_manager.key_cache.clone(),
                      engine.cache_manager.value_cache.clone()))
    assert outputs[0] == outputs[1]
    assert all(len(r) == 3 for r in outputs[0])
    # The same kernels on the same inputs: every written KV byte agrees.
    assert torch.equal(pools[0][0].view(torch.int16), pools[1][0].view(torch.int16))
    assert torch.equal(pools[0][1].view(torch.int16), pools[1][1].view(torch.int16))
    after = _launch_counts()
    if mode != "sync":
        # the runner's routing launches went through the sm_100a adapters
        assert after["metadata_kernel"] > before["metadata_kernel"]
        assert after["gather_kernel"] > before["gather_kernel"]
        assert after["scatter_kernel"] > before["scatter_kernel"]
        if layout == "last_exited":
            assert after["finalize_kernel"] > before["finalize_kernel"]


_TORCH_OUTPUTS = {}


def _trace_run(ref, model, layout, backend, mode, static, graphs, b200):
    from vllm_rlt import ExitConfig, SamplingParams

    traces = {str(i): [4, 2 + i % 3, 4, 2, 3, 4] for i in range(3)}
    engine = _engine(ref, model, layout=layout, mode=mode, static=static, graphs=graphs,
                     backend=backend, exit_config=ExitConfig("trace", depths_by_request=traces),
                     blocks=48, b200=b200)
    for i in range(3):
        engine.add_request(str(i), [2, 3, 4, 5] * (i + 1),
                           SamplingParams(max_tokens=6, min_loops=1, ignore_eos=True))
    finished = _drain(engine, 300)
    assert len(finished) == 3
    assert engine.cache_manager.num_used_blocks == 0
    if b200:
        torch.cuda.synchronize()
        assert engine.cache_manager.attention.check_errors() == []
    return finished


@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("layout", ["last_exited", "shared"])
@pytest.mark.parametrize("static", [False, True])
def test_reference_engine_matches_its_own_backends(ref, head_dim, layout, static):
    """tests/test_flash_attention.py:92-132 on the B200 backend: every mode,
    eager and graphed, generates the tokens and exit depths of the
    reference's stock GPU engine (its Triton backend, same static-buffer
    setting) -- and those of its torch backend wherever the reference's two
    paths agree with each other (where they do not, the torch path's bf16
    logits hold an exact tie, so the greedy pick depends on rounding)."""
    model = _tiny_model(ref, head_dim, 123)
    key = (head_dim, layout)
    if key not in _TORCH_OUTPUTS:
        _TORCH_OUTPUTS[key] = _trace_run(ref, model, layout, "torch", "sync", False, False, False)
    torch_outputs = _TORCH_OUTPUTS[key]
    stock = _trace_run(ref, model, layout, "triton", "sync", static, False, False)
    for mode, graphs in (("sync", False), ("async", False), ("multi", False), ("sync", True),
                         ("async", True), ("multi", True)):
        got = _trace_run(ref, model, layout, "triton", mode, static, graphs, True)
        assert got == stock, (mode, graphs)
        for rid, (tokens, depths) in torch_outputs.items():
            if stock[rid] == (tokens, depths):
                assert got[rid] == (tokens, depths), (mode, graphs, rid)
    # head_dim 64 (no logit ties on this model): all three agree outright
    if head_dim == 64:
        assert stock == torch_outputs


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fragmented_mixed_depth_rows_match_dense(ref, dtype):
    """tests/test_prepared_kv.py:30-82 through the cache manager on the GPU."""
    from vllm_rlt.core.kv_cache_manager import KVCacheManager

    torch.manual_seed(71)
    cache = KVCacheManager(num_layers=3, num_kv_heads=1, head_dim=4, num_blocks=36,
                           block_size=2, max_loops=4, device="cuda", dtype=dtype,
                           backend="triton")
    ref.b200(cache)
    for name, size in (("left", 4), ("protected", 2), ("right", 4)):
        assert cache.allocate(name, size)
    cache.key_cache.fill_(-99)
    cache.value_cache.fill_(-98)
    cache.free("left")
    cache.free("right")
    assert cache.allocate("a", 5) and cache.allocate("b", 3)
    ids = ["a"] * 10 + ["b"] * 3
    depths = [0] * 5 + [3] * 5 + [1] * 3
    positions = list(range(5)) * 2 + list(range(3))
    batch = cache._prepare_batch(ids, depths, positions)
    assert batch.block_tables.shape == (13, 3) and batch.block_tables[-1, -1].item() == -1
    keys = torch.randn(13, 1, 4, device="cuda").to(dtype)
    values = torch.randn(13, 1, 4, device="cuda").to(dtype)
    query = torch.randn(13, 2, 4, device="cuda").to(dtype)
    protected_pages = [p for t in cache._allocations["protected"].block_tables for p in t]
    protected = (cache.key_cache[protected_pages].clone(),
                 cache.value_cache[protected_pages].clone())
    for layer in range(cache.num_layers):
        layer_values = values + layer
        cache._write_prepared(layer, batch, keys, layer_values)
        actual = cache._attend_prepared(layer, batch, query)
        expected = torch.empty(13, 2, 4, dtype=torch.float64)
        for row, (name, depth, position) in enumerate(zip(ids, depths, positions)):
            selected = [i for i, address in enumerate(zip(ids, depths, positions))
                        if address[:2] == (name, depth) and address[2] <= position]
            dense_k = keys[selected].double().cpu().repeat_interleave(2, dim=1)
            dense_v = layer_values[selected].double().cpu().repeat_interleave(2, dim=1)
            scores = torch.einsum("hd,thd->ht", query[row].double().cpu(), dense_k) / 2.0
            expected[row] = torch.einsum("ht,thd->hd", scores.softmax(-1), dense_v)
        name = DTYPE_NAMES[dtype]
        want = expected.float()
        if dtype != torch.float32:
            want = want.to(dtype)
        assert_close(to_numpy(actual), to_numpy(want), name)
        # the page write is the reference's index-put, bit for bit
        blocks, offsets = batch.write_blocks, batch.write_offsets
        assert torch.equal(cache.key_cache[blocks, layer, offsets], keys)
        assert torch.equal(cache.value_cache[blocks, layer, offsets], layer_values)
    assert torch.equal(cache.key_cache[protected_pages], protected[0])
    assert torch.equal(cache.value_cache[protected_pages], protected[1])
    torch.cuda.synchronize()
    assert cache.attention.check_errors() == []


def _small_cache(ref, blocks=8):
    from vllm_rlt.core.kv_cache_manager import KVCacheManager

    cache = KVCacheManager(num_layers=3, num_kv_heads=1, head_dim=4, num_blocks=blocks,
                           block_size=2, max_loops=4, device="cuda", dtype=torch.float32,
                           backend="triton")
    ref.b200(cache)
    return cache


@pytest.mark.parametrize("stale_kind", ["free", "same_id_reallocation", "wrong_manager"])
def test_routed_write_keeps_stale_batch_checks(ref, stale_kind):
    """tests/test_prepared_kv.py:110-139: a stale batch never reaches the pool."""
    cache = _small_cache(ref)
    cache.allocate("a", 4)
    batch = cache._prepare_batch(["a"], [0], [0])
    if stale_kind == "wrong_manager":
        target = _small_cache(ref)
        target.allocate("a", 4)
    else:
        target = cache
        cache.free("a")
        if stale_kind == "same_id_reallocation":
            cache.allocate("a", 4)
    target.key_cache.fill_(17)
    target.value_cache.fill_(19)
    before = target.key_cache.clone(), target.value_cache.clone()
    tensor = torch.ones(1, 1, 4, device="cuda")
    with pytest.raises((ValueError, RuntimeError), match="different cache|stale"):
        target._write_prepared(0, batch, tensor, tensor)
    with pytest.raises((ValueError, RuntimeError), match="different cache|stale"):
        target._attend_prepared(0, batch, tensor)
    torch.cuda.synchronize()
    assert torch.equal(target.key_cache, before[0]) and torch.equal(target.value_cache, before[1])


def test_routed_write_keeps_prefix_and_read_only_checks(ref):
    """tests/test_prepared_kv.py:152-190 on the routed write."""
    cache = _small_cache(ref, blocks=36)
    cache.allocate("a", 4)
    batch = cache._prepare_batch(["a", "a"], [0, 0], [2, 0])
    values = torch.ones(2, 1, 4, device="cuda")
    for layer in range(cache.num_layers):
        with pytest.raises(RuntimeError, match="uninitialized"):
            cache._attend_prepared(layer, batch, values)
    cache._write_prepared(0, batch, values, values)
    with pytest.raises(RuntimeError, match="uninitialized"):
        cache._attend_prepared(0, batch, values)
    cache.write(0, ["a"], [0], [1], values[:1], values[:1])
    torch.testing.assert_close(cache._attend_prepared(0, batch, values), values)
    with pytest.raises(RuntimeError, match="layer 1"):
        cache._attend_prepared(1, batch, values)
    read_only = cache._prepare_batch(["a", "a"], [0, 0], [0, 0], for_write=False)
    with pytest.raises(ValueError, match="read-only"):
        cache._write_prepared(0, read_only, values, values)
    with pytest.raises(ValueError, match="KV heads"):
        cache._write_prepared(0, batch, torch.ones(2, 2, 4, device="cuda"), values)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("head_dim", [64, 128])
def test_packed_prefill_ragged_prefixes_and_depths(ref, dtype, head_dim):
    """tests/test_flash_attention.py:146-189 with the B200 backend installed:
    the packed prefill against the reference's torch oracle over per-token
    rows, at the 2e-3 (+1 ulp) bound."""
    from vllm_rlt.core.kv_cache_manager import KVCacheManager
    from vllm_rlt.kernels.paged_attention import torch_paged_attention

    torch.manual_seed(712)
    cache = KVCacheManager(2, 2, head_dim, 80, 16, 4, "cuda", dtype, "triton")
    ref.b200(cache)
    assert cache.attention.generation == 4
    for rid in ["hole", "a", "b", "c"]:
        cache.allocate(rid, 65)
    cache.free("hole")
    ids, depths, positions = [], [], []
    for rid, depth, prefix, count in [("a", 0, 0, 19), ("b", 2, 17, 7), ("c", 3, 31, 18)]:
        for layer in range(2):
            if prefix:
                kv = torch.randn(prefix, 2, head_dim, device="cuda", dtype=dtype)
                cache.write(layer, [rid] * prefix, [depth] * prefix, list(range(prefix)), kv, -kv)
        ids.extend([rid] * count)
        depths.extend([depth] * count)
        positions.extend(range(prefix, prefix + count))
    batch = cache._prepare_batch(ids, depths, positions, packed_prefill=True)
    flat = cache._prepare_batch(ids, depths, positions)
    assert batch.block_tables.shape[0] == 3 and flat.block_tables.shape[0] == len(ids)
    for layer in range(2):
        k = torch.randn(len(ids), 2, head_dim, device="cuda", dtype=dtype)
        v = torch.randn_like(k)
        q = torch.randn(len(ids), 4, head_dim, device="cuda", dtype=dtype)
        cache._write_prepared(layer, batch, k, v)
        expected = torch_paged_attention(q, cache.key_cache[:, layer], cache.value_cache[:, layer],
                                         flat.block_tables, flat.context_lengths)
        actual = cache._attend_prepared(layer, batch, q)
        assert_close(to_numpy(actual), to_numpy(expected), DTYPE_NAMES[dtype])
    torch.cuda.synchronize()
    assert cache.attention.check_errors() == []


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("heads", [2, 4])
def test_ragged_strided_decode_vs_reference_oracle(ref, dtype, heads):
    """tests/test_flash_attention.py:50-70: strided layer views, an empty row."""
    from vllm_rlt.kernels.paged_attention import torch_paged_attention

    torch.manual_seed(9)
    keys = torch.randn(12, 3, 16, 2, 128, device="cuda", dtype=dtype)[:, 1]
    values = torch.randn(12, 3, 16, 2, 128, device="cuda", dtype=dtype)[:, 1]
    q = torch.randn(4, heads, 128, device="cuda", dtype=dtype)
    tables = torch.tensor([[7, 2, 9], [3, 0, 0], [1, 8, 6], [0, 0, 0]], device="cuda",
                          dtype=torch.int32)
    lengths = torch.tensor([35, 1, 47, 0], device="cuda", dtype=torch.int32)
    attention = rb.B200PagedAttention(q.device, dtype, 128, 16)
    expected = torch_paged_attention(q, keys, values, tables, lengths)
    actual = attention(q, keys, values, tables, lengths)
    assert_close(to_numpy(actual), to_numpy(expected), DTYPE_NAMES[dtype])
    assert torch.isfinite(actual).all() and torch.count_nonzero(actual[-1]) == 0


def test_decode_same_queries_match_across_batch_sizes(ref):
    """tests/test_flash_attention.py:192-208: a row's bits do not depend on the
    rest of the batch (long enough rows to take the split-KV path)."""
    generator = torch.Generator(device="cuda").manual_seed(1234)
    dtype = torch.bfloat16
    keys = torch.randn(260, 2, 16, 4, 128, generator=generator, device="cuda", dtype=dtype)[:, 1]
    values = torch.randn(260, 2, 16, 4, 128, generator=generator, device="cuda",
                         dtype=dtype)[:, 1]
    q = torch.randn(4, 16, 128, generator=generator, device="cuda", dtype=dtype)
    tables = torch.arange(260, device="cuda", dtype=torch.int32).view(4, 65)
    lengths = torch.tensor([1025, 1029, 1025, 1031], device="cuda", dtype=torch.int32)
    attention = rb.B200PagedAttention(q.device, dtype, 128, 16)
    together = attention(q, keys, values, tables, lengths)
    for rows in ([2, 3], [3, 0], [1]):
        separate = attention(q[rows], keys, values, tables[rows], lengths[rows])
        assert torch.equal(separate, together[rows])
    from vllm_rlt.kernels.paged_attention import torch_paged_attention

    expected = torch_paged_attention(q, keys, values, tables, lengths)
    assert_close(to_numpy(together), to_numpy(expected), "bf16")


def test_install_leaves_no_triton_on_the_async_path(ref):
    """With the backend and the routing adapters installed, one async engine
    step sequence launches no reference Triton kernel: every routing kernel
    name in the reference's modules resolves to an sm_100a adapter."""
    from vllm_rlt.kernels import prefill_metadata, routing

    from vllm_rlt import ExitConfig

    model = _tiny_model(ref, 64, 5)
    engine = _engine(ref, model, layout="last_exited", mode="async",
                     exit_config=ExitConfig("ouro_delayed"))
    for name in backend_mod.ROUTING_LAUNCHES:
        assert isinstance(getattr(routing, name), backend_mod._GridLaunch)
    for name in backend_mod.PREFILL_LAUNCHES:
        assert isinstance(getattr(prefill_metadata, name), backend_mod._GridLaunch)
    from vllm_rlt import SamplingParams

    before = _launch_counts()
    engine.add_request("x", [2, 3, 4, 5, 6], SamplingParams(max_tokens=4, ignore_eos=True))
    assert len(_drain(engine)) == 1
    after = _launch_counts()
    assert after["metadata_kernel"] > before["metadata_kernel"]
