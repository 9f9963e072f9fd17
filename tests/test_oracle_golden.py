"""Pin the CPU oracle to the reference's own outputs (golden vectors).

Every fixture under tests/golden/ was produced by running the reference
(vllm-rlt) itself: its KV cache manager, its torch attention oracle and its
Triton kernels under Triton's CPU interpreter. These tests check that the
numpy restatement in ``oracle/`` reproduces them: KV pools bit-exactly (by
digest), metadata bit-exactly, attention within fp32 rounding.
"""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from helpers import (NumpyWriter, assert_close, digest, load, prefill_case, prefill_names,
                     query_inputs, replay_pool, scenario_names)
from vllm_rlt_b200 import workloads

SCENARIOS = scenario_names()


def rebuild(name):
    fx = load(name)
    layers, hkv, hq, d, num_blocks, page, loops, seed = (int(x) for x in fx["dims"])
    writer = NumpyWriter((num_blocks, layers, page, hkv, d), str(fx["dtype"]))
    replay_pool(fx, name, writer)
    return fx, writer


@pytest.mark.parametrize("name", SCENARIOS)
def test_replayed_pool_matches_reference_digest(name):
    fx, writer = rebuild(name)
    assert digest(writer.key) == str(fx["key_digest"])
    assert digest(writer.value) == str(fx["value_digest"])


@pytest.mark.parametrize("name", SCENARIOS)
def test_oracle_attention_matches_reference(name):
    fx, writer = rebuild(name)
    dtype = str(fx["dtype"])
    qi = query_inputs(fx)
    layer = qi["layer"]
    out = oracle.paged_attention(qi["q"], writer.key[:, layer], writer.value[:, layer],
                                 qi["block_tables"], qi["context_lengths"], dtype)
    # Both sides are fp32 math on the same inputs; only summation order differs.
    tight = dict(atol=1e-6, rtol=1e-6, ulps=0) if dtype == "f32" else {}
    assert_close(out, qi["out"], dtype, **tight)


@pytest.mark.parametrize("name", SCENARIOS)
def test_reference_triton_kernel_agrees_with_reference_torch(name):
    fx = load(name)
    qi = query_inputs(fx)
    assert_close(qi["triton_out"], qi["out"], str(fx["dtype"]))


@pytest.mark.parametrize("name", SCENARIOS)
def test_oracle_depth_page_resolution_matches_prepare_batch(name):
    fx = load(name)
    layers, hkv, hq, d, num_blocks, page, loops, seed = (int(x) for x in fx["dims"])
    layout = str(fx["layout"])
    tables = fx["alloc_tables"]
    qi = query_inputs(fx)
    rows = qi["rows"]
    by_request = {}
    for rid in set(rows[:, 0].tolist()):
        by_request[rid] = [[int(b) for b in plane if b >= 0] for plane in tables[rid]]
    prepared = oracle.prepare_rows([by_request[r] for r in rows[:, 0].tolist()], loops,
                                   rows[:, 1].tolist(), rows[:, 2].tolist(), page, layout)
    np.testing.assert_array_equal(prepared["block_tables"], qi["block_tables"])
    np.testing.assert_array_equal(prepared["context_lengths"], qi["context_lengths"])
    np.testing.assert_array_equal(prepared["write_blocks"], fx["q0_write_blocks"])
    np.testing.assert_array_equal(prepared["write_offsets"], fx["q0_write_offsets"])


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_config1_plan_matches_reference_allocator(dtype):
    """The workload generator hands out pages exactly as the reference's
    allocator does, and the plan's padded tables equal _prepare_batch's."""
    fx = load(f"config1_{dtype}")
    plan = workloads.config1_plan(0)
    for r in range(plan.num_rows):
        for plane in range(plan.planes):
            pages = plan.plane_tables[r][plane]
            np.testing.assert_array_equal(fx["alloc_tables"][r, plane, : len(pages)], pages)
    np.testing.assert_array_equal(plan.block_tables(), fx["q0_block_tables"])
    np.testing.assert_array_equal(plan.context_lengths, fx["q0_context_lengths"])


@pytest.mark.parametrize("name", prefill_names())
def test_oracle_packed_prefill_matches_reference(name):
    fx, writer, inputs = prefill_case(name, NumpyWriter)
    dtype = str(fx["dtype"])
    spec = fx["spec"].tolist()
    tables = {rid: [list(fx["alloc_tables"][rid, p]) for p in range(4)] for rid, _, _, _ in spec}
    ids, depths, positions = [], [], []
    for rid, depth, prefix, count in spec:
        ids += [rid] * count
        depths += [depth] * count
        positions += list(range(prefix, prefix + count))
    packed = oracle.prepare_rows([tables[r] for r in ids], 4, depths, positions, 16, "last_exited",
                                 packed=True)
    np.testing.assert_array_equal(packed["block_tables"], fx["block_tables"])
    np.testing.assert_array_equal(packed["context_lengths"], fx["context_lengths"])
    np.testing.assert_array_equal(packed["cu_seqlens_q"], fx["cu_seqlens_q"])
    np.testing.assert_array_equal(packed["write_blocks"], fx["write_blocks"])
    np.testing.assert_array_equal(packed["write_offsets"], fx["write_offsets"])
    for layer, (k, v, q) in enumerate(inputs):
        oracle.kv_write(writer.key, writer.value, layer, fx["write_blocks"], fx["write_offsets"],
                        k, v)
        out = oracle.paged_prefill(q, writer.key[:, layer], writer.value[:, layer],
                                   fx["block_tables"], fx["context_lengths"], fx["cu_seqlens_q"],
                                   dtype)
        tight = dict(atol=1e-6, rtol=1e-6, ulps=0) if dtype == "f32" else {}
        assert_close(out, fx[f"out{layer}"], dtype, **tight)
    assert digest(writer.key) == str(fx["key_digest"])
    assert digest(writer.value) == str(fx["value_digest"])


@pytest.mark.parametrize("planes", [4, 1])
def test_oracle_metadata_matches_reference_triton(planes):
    fx = load("routing")
    tag = f"meta_p{planes}"
    slots, planes_, width, page, size, n, out_width = fx[f"{tag}_dims"].tolist()
    prior = dict(
        slots=np.full(size, -7, np.int64), positions=np.full(size, -7, np.int64),
        lengths=np.full(size, -7, np.int32), blocks=np.full(size, -7, np.int64),
        offsets=np.full(size, -7, np.int64), out_tables=np.full((size, width), -7, np.int32),
    )
    res = oracle.metadata(fx[f"{tag}_desc"], fx[f"{tag}_tables"], prior, n, size, width, page,
                          planes_, out_width)
    for key in prior:
        np.testing.assert_array_equal(res[key], fx[f"{tag}_{key}"], err_msg=key)


def test_oracle_finalize_matches_reference_triton():
    fx = load("routing")
    blocks, layers, page, hkv, d, planes, width, slots = fx["fin_dims"].tolist()
    key = fx["fin_key_before"].copy()
    value = fx["fin_value_before"].copy()
    oracle.finalize(fx["fin_desc"], fx["fin_tables"], key, value, planes, page)
    np.testing.assert_array_equal(key, fx["fin_key_after"])
    np.testing.assert_array_equal(value, fx["fin_value_after"])


def test_oracle_finalize_token_equals_batched_finalize():
    """The eager exit copy (kv_cache_manager.py:601-611) and the batched
    kernel (routing.py:79-109) agree, row by row."""
    fx = load("routing")
    blocks, layers, page, hkv, d, planes, width, slots = fx["fin_dims"].tolist()
    key = fx["fin_key_before"].copy()
    value = fx["fin_value_before"].copy()
    for slot, depth, pos in fx["fin_desc"].tolist():
        oracle.finalize_token(key, value, fx["fin_tables"][slot], pos, depth, planes, page)
    np.testing.assert_array_equal(key, fx["fin_key_after"])
    np.testing.assert_array_equal(value, fx["fin_value_after"])


def test_oracle_prefill_metadata_matches_reference_triton():
    fx = load("routing")
    target, target32 = oracle.stage_prefill(fx["stage_source"])
    np.testing.assert_array_equal(target, fx["stage_target"])
    np.testing.assert_array_equal(target32, fx["stage_target32"])
    n, width, page = fx["expand_dims"].tolist()
    blocks, offsets = oracle.expand_prefill(fx["expand_positions"], fx["expand_sequences"],
                                            fx["expand_tables"], width, page)
    np.testing.assert_array_equal(blocks, fx["expand_blocks"])
    np.testing.assert_array_equal(offsets, fx["expand_offsets"])


def test_oracle_gather_scatter_matches_reference_triton():
    fx = load("routing")
    got = oracle.gather(fx["gather_pool"], fx["gather_slots"], 5, 8)
    # the reference kernel writes zeros into padding rows of the output
    np.testing.assert_array_equal(got, fx["gather_out"])
    after = oracle.scatter(fx["scatter_values"], fx["scatter_slots"], fx["scatter_before"], 4)
    np.testing.assert_array_equal(after, fx["scatter_after"])
