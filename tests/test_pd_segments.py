"""Prefill/decode KV transport host logic (CPU): the segment lists and their
partition into transfers equal the reference's own outputs
(tests/golden/pd_segments.json, made by tests/golden/make_pd_golden.py from
vllm_rlt/pd/transport.py:18-72), and they cover exactly the valid tokens of
every plane, layer, K and V."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from vllm_rlt_b200.pd import kv_segments, partition_segments, pool_info

CASES = json.loads((Path(__file__).parent / "golden" / "pd_segments.json").read_text())


@pytest.mark.parametrize("index", range(len(CASES)))
def test_segments_match_reference(index):
    case = CASES[index]
    segments = kv_segments(case["info"], case["tables"], case["start"], case["end"]).tolist()
    assert segments == case["segments"]
    for limits in case["partitions"]:
        parts = [[local.tolist(), remote.tolist(), size]
                 for local, remote, size in partition_segments(
                     segments, segments, limits["byte_limit"], limits["descriptor_limit"])]
        assert parts == limits["parts"]
        for local, _, size in parts:
            assert size <= limits["byte_limit"] and len(local) <= limits["descriptor_limit"]


@pytest.mark.parametrize("index", range(len(CASES)))
def test_segments_cover_exactly_the_valid_tokens(index):
    case = CASES[index]
    info, tables, start, end = case["info"], case["tables"], case["start"], case["end"]
    page = info["block_size"]
    expected = set()
    for table in tables:
        for token in range(start, end):
            for layer in range(info["num_layers"]):
                for base in (info["key_ptr"], info["value_ptr"]):
                    pos = (base + table[token // page] * info["block_bytes"]
                           + layer * info["layer_bytes"] + (token % page) * info["token_bytes"])
                    expected.add((pos, pos + info["token_bytes"]))
    covered = set()
    for address, size, _ in kv_segments(info, tables, start, end).tolist():
        for pos in range(address, address + size, info["token_bytes"]):
            covered.add((pos, pos + info["token_bytes"]))
    assert covered == expected


def test_invalid_ranges_and_blocks_raise():
    case = CASES[0]
    info, tables = case["info"], case["tables"]
    for start, end in ((3, 3), (-1, 2), (5, 4)):
        with pytest.raises(ValueError, match="token range"):
            kv_segments(info, tables, start, end)
    with pytest.raises(ValueError, match="past the"):
        kv_segments(info, tables, 0, len(tables[0]) * info["block_size"] + 1)
    bad = [list(t) for t in tables]
    bad[0][0] = info["num_blocks"]
    with pytest.raises(ValueError, match="outside the pool"):
        kv_segments(info, bad, 0, 1)
    with pytest.raises(ValueError, match="different byte layouts"):
        partition_segments([(0, 16, 0)], [(0, 32, 0)], 64, 4)
    assert partition_segments([], [], 64, 4) == []


def test_partition_against_a_byte_stream_walk():
    """Random segment lists and limits: the transfers tile the byte stream in
    order, each within both limits, every byte exactly once, and only the
    byte bound ever splits a segment."""
    rng = np.random.default_rng(0)
    for _ in range(200):
        n = int(rng.integers(1, 40))
        sizes = rng.integers(1, 300, size=n)
        src = np.stack([np.cumsum(sizes) * 7, sizes, np.zeros(n, dtype=np.int64)], 1)
        dst = src + np.array([1 << 30, 0, 1])
        byte_limit, descriptor_limit = int(rng.integers(1, 700)), int(rng.integers(1, 9))
        parts = partition_segments(src, dst, byte_limit, descriptor_limit)
        flat = []
        for local, remote, size in parts:
            assert 0 < size <= byte_limit and len(local) <= descriptor_limit
            assert int(local[:, 1].sum()) == size
            assert (remote[:, 0] - local[:, 0] == 1 << 30).all() and (remote[:, 2] == 1).all()
            # a transfer closes only at its byte limit or its descriptor limit (or the end)
            full = size == byte_limit or len(local) == descriptor_limit
            assert full or (local is parts[-1][0])
            flat.extend(local.tolist())
        covered = []
        for address, size, _ in flat:
            covered.extend(range(address, address + size))
        want = []
        for address, size, _ in src.tolist():
            want.extend(range(address, address + size))
        assert covered == want


def test_pool_info_geometry():
    k = torch.zeros(8, 3, 4, 2, 16, dtype=torch.bfloat16)
    info = pool_info(k, torch.zeros_like(k), 4)
    assert info["block_bytes"] == 3 * 4 * 2 * 16 * 2
    assert info["layer_bytes"] == 4 * 2 * 16 * 2
    assert info["token_bytes"] == 2 * 16 * 2
    assert info["num_layers"] == 3 and info["num_blocks"] == 8
