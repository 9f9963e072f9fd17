"""Shared-prefix decode on the B200 vs the oracle's paged attention.

Rows whose block tables begin with the same physical pages (prefix caching)
are attended through ``paged_attention_shared``, which reads the shared
pages once per group; the result must equal the oracle (and the plain decode
kernel) on the same tables and lengths."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import vllm_rlt_b200 as rb
from gpu_helpers import TORCH, to_numpy
from helpers import assert_close
from test_shared_prefix_plan import make_case
from vllm_rlt_b200 import _lib

pytestmark = pytest.mark.gpu


def run_case(dtype, d, hkv, group, page, rows=12, width=24, groups=((0, 1, 2, 3, 4), (6, 7)),
             shared=(5, 3), seed=0, empty_rows=(), chunk_tokens=64):
    tables, lengths, num_blocks = make_case(seed, page=page, rows=rows, width=width, groups=groups,
                                            shared=shared)
    for r in empty_rows:
        lengths[r] = 0
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    td = TORCH[dtype]
    # a 5-D pool [blocks, layers, page, Hkv, D]; attention sees the layer view
    pool_k = torch.randn(num_blocks, 2, page, hkv, d, generator=g, device="cuda").to(td)
    pool_v = torch.randn(num_blocks, 2, page, hkv, d, generator=g, device="cuda").to(td)
    key, value = pool_k[:, 1], pool_v[:, 1]
    q = torch.randn(rows, hkv * group, d, generator=g, device="cuda").to(td)
    t = torch.from_numpy(tables).cuda()
    n = torch.from_numpy(lengths).cuda()
    plan = rb.plan_shared_prefix(tables, lengths, page, hkv * group, hkv, "cuda",
                                 chunk_tokens=chunk_tokens)
    backend = rb.B200PagedAttention("cuda", td, d, page)
    out = rb.paged_attention_shared(q, key, value, t, plan, context_lengths=n)
    plain = rb.paged_attention(q, key, value, t, n)
    torch.cuda.synchronize()
    assert backend.check_errors() == []
    expected = oracle.paged_attention(to_numpy(q), to_numpy(key), to_numpy(value), tables, lengths,
                                      dtype)
    return out, plain, expected, plan


@pytest.mark.parametrize("dtype", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("d", [64, 128])
def test_shared_prefix_decode_matches_oracle(dtype, d):
    out, plain, expected, plan = run_case(dtype, d, hkv=2, group=2, page=16)
    assert plan.read_tokens < plan.logical_tokens
    assert_close(to_numpy(out), expected, dtype)
    assert_close(to_numpy(out), to_numpy(plain), dtype)


@pytest.mark.parametrize("group,page", [(1, 16), (4, 8), (8, 32)])
def test_gqa_and_page_sizes(group, page):
    out, _, expected, _ = run_case("bf16", 128, hkv=2, group=group, page=page, seed=3)
    assert_close(to_numpy(out), expected, "bf16")


@pytest.fixture(params=[2, 1], ids=["tma", "cp_async"])
def staging(request):
    """The chunk kernel's K/V staging (rlt_shared_prefix_select): 2 = tiled
    TMA loads where the page size allows (the default), 1 = cp.async."""
    lib = _lib.load()
    previous = lib.rlt_shared_prefix_select(request.param)
    yield request.param
    lib.rlt_shared_prefix_select(previous)


@pytest.mark.parametrize("page,chunk,group,width,shared",
                         [(16, 512, 1, 24, (20, 12)), (16, 200, 8, 24, (20, 12)),
                          (8, 100, 1, 40, (30, 20)), (64, 512, 4, 12, (10, 6)),
                          (48, 512, 2, 24, (20, 12)), (5, 333, 1, 80, (70, 40))])
def test_chunks_of_many_sub_tiles(page, chunk, group, width, shared, staging):
    """Chunks longer than one staged sub-tile, including chunk starts inside a
    page and pages that do not divide the sub-tile (cp.async staging there):
    the cp.async loader steps each token's page and in-page offset from one
    sub-tile to the next; the TMA loader starts at the page holding the
    chunk's first token and masks the tokens outside the chunk."""
    out, plain, expected, plan = run_case("bf16", 128, hkv=2, group=group, page=page, width=width,
                                          shared=shared, seed=5, chunk_tokens=chunk)
    chunks = plan.chunks.cpu().numpy()
    assert (chunks[:, 2] - chunks[:, 1]).max() > 64
    assert_close(to_numpy(out), expected, "bf16")
    assert_close(to_numpy(out), to_numpy(plain), "bf16")


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("d", [64, 128])
def test_tma_and_cp_async_staging_agree(dtype, d):
    """Page-aligned chunks: both stagings put the same tokens in the same
    sub-tile slices, so their results are bit-identical."""
    lib = _lib.load()
    outs = []
    for mode in (2, 1):
        previous = lib.rlt_shared_prefix_select(mode)
        try:
            out, _, expected, _ = run_case(dtype, d, hkv=2, group=2, page=16, width=24,
                                           shared=(20, 12), seed=9, chunk_tokens=256)
        finally:
            lib.rlt_shared_prefix_select(previous)
        assert_close(to_numpy(out), expected, dtype)
        outs.append(out)
    assert torch.equal(outs[0], outs[1])


def test_large_group_split_into_member_blocks_and_empty_rows():
    """A 30-row group (Ouro geometry, 16 KV heads, no GQA) is attended in
    member blocks of 32; empty rows produce zeros."""
    out, _, expected, plan = run_case("bf16", 128, hkv=16, group=1, page=16, rows=40, width=20,
                                      groups=(tuple(range(30)), (31, 32, 33)), shared=(12, 4),
                                      seed=5, empty_rows=(35,))
    assert_close(to_numpy(out), expected, "bf16")
    assert not to_numpy(out[35]).any()
    assert plan.read_tokens * 2 < plan.logical_tokens  # 30 rows read a 192-token prefix once


def test_no_shared_pages_equals_plain_decode():
    out, plain, expected, plan = run_case("bf16", 128, hkv=2, group=1, page=16, groups=(),
                                          shared=(), seed=9)
    assert plan.groups == [] and plan.read_tokens == plan.logical_tokens
    assert_close(to_numpy(out), expected, "bf16")


@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_decode_log_sum_exp(dtype):
    """rlt_paged_decode_lse: same output as the plain decode, and the base-2
    log-sum-exp of the scaled scores (rows short and long enough to split,
    and an empty row)."""
    tables, lengths, num_blocks = make_case(13, rows=9, width=40, groups=(), shared=())
    lengths[4] = 0
    long_row = int(np.argmax((tables >= 0).sum(axis=1)))
    lengths[long_row] = int((tables[long_row] >= 0).sum()) * 16  # its whole table: several splits
    assert lengths[long_row] > 256
    g = torch.Generator(device="cuda").manual_seed(3)
    td = TORCH[dtype]
    key = torch.randn(num_blocks, 16, 2, 128, generator=g, device="cuda").to(td)
    value = torch.randn(num_blocks, 16, 2, 128, generator=g, device="cuda").to(td)
    q = torch.randn(9, 4, 128, generator=g, device="cuda").to(td)
    t = torch.from_numpy(tables).cuda()
    n = torch.from_numpy(lengths).cuda()
    backend = rb.B200PagedAttention("cuda", td, 128, 16)
    out, lse = rb.paged_attention_lse(q, key, value, t, n)
    plain = rb.paged_attention(q, key, value, t, n)
    torch.cuda.synchronize()
    assert backend.check_errors() == []
    assert torch.equal(out, plain)
    qf = q.float().cpu().numpy().astype(np.float64)
    kf = key.float().cpu().numpy().astype(np.float64)
    for r in range(9):
        if lengths[r] == 0:
            assert torch.isinf(lse[r]).all() and (lse[r] < 0).all()
            continue
        pos = np.arange(lengths[r])
        k = np.repeat(kf[tables[r, pos // 16], pos % 16], 2, axis=1)  # [T, Hq, D]
        s = np.einsum("hd,thd->ht", qf[r], k) / np.sqrt(128)
        want = np.log2(np.exp(s - s.max(axis=1, keepdims=True)).sum(axis=1)) + s.max(axis=1) / np.log(2)
        np.testing.assert_allclose(lse[r].cpu().numpy(), want, rtol=0, atol=2e-4)


def test_plan_stays_valid_as_rows_grow_and_replays_in_a_graph():
    """A plan made once keeps serving the batch while its rows grow (each
    call derives the suffix tables and lengths on the device): decode steps
    that append tokens -- within the rows' pages and onto fresh pages --
    eagerly and as replays of one captured CUDA graph whose length and table
    buffers are updated in place."""
    page, hkv, d = 16, 4, 128
    tables, lengths, num_blocks = make_case(21, page=page, rows=10, width=30,
                                            groups=((0, 1, 2, 3), (5, 6, 7)), shared=(6, 4))
    lengths = np.minimum(lengths, 20 * page).astype(np.int32)  # room to grow
    for r in range(10):  # drop table entries beyond the (shortened) context
        tables[r, -(-int(lengths[r]) // page):] = -1
    spare = iter(range(num_blocks, num_blocks + 10 * 30))  # fresh pages appended on growth
    pool_blocks = num_blocks + 10 * 30
    g = torch.Generator(device="cuda").manual_seed(4)
    key = torch.randn(pool_blocks, page, hkv, d, generator=g, device="cuda").to(torch.bfloat16)
    value = torch.randn(pool_blocks, page, hkv, d, generator=g, device="cuda").to(torch.bfloat16)
    q = torch.randn(10, hkv, d, generator=g, device="cuda").to(torch.bfloat16)
    plan = rb.plan_shared_prefix(tables, lengths, page, hkv, hkv, "cuda", chunk_tokens=64)
    t = torch.from_numpy(tables).cuda()
    n = torch.from_numpy(lengths).cuda()
    out = torch.empty_like(q)
    backend = rb.B200PagedAttention("cuda", torch.bfloat16, d, page)

    def grow(steps):
        for _ in range(steps):
            for r in range(10):
                if lengths[r] % page == 0:
                    tables[r, lengths[r] // page] = next(spare)
                lengths[r] += 1

    def check():
        torch.cuda.synchronize()
        assert backend.check_errors() == []
        want = oracle.paged_attention(to_numpy(q), to_numpy(key), to_numpy(value), tables,
                                      lengths, "bf16")
        assert_close(to_numpy(out), want, "bf16")

    rb.paged_attention_shared(q, key, value, t, plan, context_lengths=n, out=out)
    check()
    grow(17)  # eager, a plan from 17 steps ago
    t.copy_(torch.from_numpy(tables))
    n.copy_(torch.from_numpy(lengths))
    rb.paged_attention_shared(q, key, value, t, plan, context_lengths=n, out=out)
    check()
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        rb.paged_attention_shared(q, key, value, t, plan, context_lengths=n, out=out)
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        rb.paged_attention_shared(q, key, value, t, plan, context_lengths=n, out=out)
    for steps in (1, 15, 3):
        grow(steps)
        t.copy_(torch.from_numpy(tables))
        n.copy_(torch.from_numpy(lengths))
        graph.replay()
        check()


def test_stale_plan_is_reported():
    """A row whose context shrank below its shared pages is outside the plan:
    the call flags it (status bit 1) instead of reading past the context."""
    tables, lengths, num_blocks = make_case(2, rows=6, width=16, groups=((0, 1, 2),), shared=(5,))
    g = torch.Generator(device="cuda").manual_seed(5)
    key = torch.randn(num_blocks, 16, 2, 64, generator=g, device="cuda").to(torch.bfloat16)
    q = torch.randn(6, 2, 64, generator=g, device="cuda").to(torch.bfloat16)
    plan = rb.plan_shared_prefix(tables, lengths, 16, 2, 2, "cuda")
    shrunk = lengths.copy()
    shrunk[1] = 3 * 16  # below the group's 5 shared pages
    backend = rb.B200PagedAttention("cuda", torch.bfloat16, 64, 16)
    rb.paged_attention_shared(q, key, key, torch.from_numpy(tables).cuda(), plan,
                              context_lengths=torch.from_numpy(shrunk).cuda())
    torch.cuda.synchronize()
    assert backend.check_errors() == [_lib.STATUS_BITS[1]]
