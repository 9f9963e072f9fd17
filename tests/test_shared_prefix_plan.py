"""Host planning of the shared-prefix decode (CPU).

Invariants of ``plan_arrays``: every row's context [0, ctx) is covered exactly
once, by its shared-prefix chunks plus its suffix (read through its suffix
table); a range read through another row's table uses the same physical pages
as the row's own table; slots are contiguous per row; no chunk exceeds 32
(member, query head) pairs. A numpy execution of the plan (suffix attention
with its log-sum-exp, prefix chunk partials, the merge) matches the oracle's
paged attention."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from vllm_rlt_b200.kernels.shared_prefix import MAX_PAIRS, find_shared_prefixes, plan_arrays


def make_case(seed, page=16, rows=12, width=24, groups=((0, 1, 2, 3, 4), (6, 7)), shared=(5, 3),
              short_row=None):
    rng = np.random.default_rng(seed)
    num_blocks = 2 * rows * width + 8
    perm = rng.permutation(num_blocks)
    tables = np.full((rows, width), -1, dtype=np.int32)
    lengths = rng.integers(1, width * page, size=rows).astype(np.int32)
    cursor = 0
    for r in range(rows):
        n = -(-int(lengths[r]) // page)
        tables[r, :n] = perm[cursor:cursor + n]
        cursor += n
    for members, pages in zip(groups, shared):
        lead = members[0]
        for m in members:
            lengths[m] = min(max(lengths[m], pages * page + int(rng.integers(1, 3 * page))),
                             width * page)
            n = -(-int(lengths[m]) // page)
            fresh = perm[cursor:cursor + n]
            cursor += n
            tables[m, :] = -1
            tables[m, :n] = fresh
        for m in members:
            tables[m, :pages] = tables[lead, :pages]
    if short_row is not None:
        r, n_tokens = short_row
        lengths[r] = n_tokens
    return tables, lengths, num_blocks


def check_plan(tables, lengths, page, group, chunk_tokens=64):
    (chunks, members, slots, row_slots, suffix_tables, suffix_lengths, groups, logical,
     read) = plan_arrays(tables, lengths, page, group, chunk_tokens)
    rows = tables.shape[0]
    assert row_slots[0] == 0 and row_slots[-1] == len(members)
    covered = [np.zeros(max(int(n), 0), dtype=np.int32) for n in lengths]
    seen_slots = set()
    for c, (table_row, b, e, mb, mc) in enumerate(chunks):
        assert 0 < mc and mc * group <= MAX_PAIRS
        assert 0 <= b < e
        for i in range(mc):
            row, slot = members[mb + i], slots[mb + i]
            assert row_slots[row] <= slot < row_slots[row + 1]
            assert slot not in seen_slots
            seen_slots.add(slot)
            assert e <= lengths[row]
            covered[row][b:e] += 1
            pages = np.arange(b // page, (e - 1) // page + 1)
            assert (tables[table_row, pages] == tables[row, pages]).all()
    for r in range(rows):
        n = int(suffix_lengths[r])
        prefix = int(lengths[r]) - n if n else int(lengths[r])
        if n:
            covered[r][prefix:] += 1
            assert prefix % page == 0
            pages = np.arange(0, (n - 1) // page + 1)
            assert (suffix_tables[r, pages] == tables[r, prefix // page + pages]).all()
        assert (covered[r] == 1).all(), f"row {r} coverage {covered[r]}"
    assert logical == int(np.clip(lengths, 0, None).sum())
    return chunks, members, slots, row_slots, groups, logical, read, suffix_tables, suffix_lengths


def run_plan(q, key, value, tables, lengths, page, group, chunk_tokens=64):
    """numpy execution of the plan: the suffix attention with its base-e
    log-sum-exp, chunk partials (o, m, l), then the merge."""
    (chunks, members, slots, row_slots, suffix_tables, suffix_lengths,
     *_) = plan_arrays(tables, lengths, page, group, chunk_tokens)
    n, hq, d = q.shape
    scale = 1.0 / np.sqrt(d)
    so = np.zeros((n, hq, d))
    slse = np.full((n, hq), -np.inf)
    for r in range(n):
        ln = int(suffix_lengths[r])
        if ln == 0:
            continue
        pos = np.arange(ln)
        blocks = suffix_tables[r, pos // page]
        k = np.repeat(key[blocks, pos % page].astype(np.float64), group, axis=1)
        v = np.repeat(value[blocks, pos % page].astype(np.float64), group, axis=1)
        s = np.einsum("hd,thd->ht", q[r].astype(np.float64), k) * scale
        m = s.max(axis=1)
        p = np.exp(s - m[:, None])
        so[r] = np.einsum("ht,thd->hd", p, v) / p.sum(axis=1)[:, None]
        slse[r] = m + np.log(p.sum(axis=1))
    po = np.zeros((row_slots[-1], hq, d))
    pm = np.full((row_slots[-1], hq), -np.inf)
    pl = np.zeros((row_slots[-1], hq))
    for table_row, b, e, mb, mc in chunks:
        pos = np.arange(b, e)
        blocks = tables[table_row, pos // page]
        k = key[blocks, pos % page].astype(np.float64)  # [T, Hkv, D]
        v = value[blocks, pos % page].astype(np.float64)
        k = np.repeat(k, group, axis=1)
        v = np.repeat(v, group, axis=1)
        for i in range(mc):
            row, slot = members[mb + i], slots[mb + i]
            s = np.einsum("hd,thd->ht", q[row].astype(np.float64), k) * scale
            m = s.max(axis=1)
            p = np.exp(s - m[:, None])
            po[slot] = np.einsum("ht,thd->hd", p, v)
            pm[slot], pl[slot] = m, p.sum(axis=1)
    out = so.copy()
    for r in range(n):
        s0, s1 = row_slots[r], row_slots[r + 1]
        if s1 == s0:
            continue
        mx = np.maximum(pm[s0:s1].max(axis=0), slse[r])
        w = np.exp(pm[s0:s1] - mx)
        wx = np.exp(slse[r] - mx)
        num = (po[s0:s1] * w[:, :, None]).sum(axis=0) + so[r] * wx[:, None]
        out[r] = num / ((pl[s0:s1] * w).sum(axis=0) + wx)[:, None]
    return out


def test_groups_found_by_common_leading_pages():
    tables, lengths, _ = make_case(0)
    groups = dict((tuple(r), s) for r, s in find_shared_prefixes(tables, lengths, 16))
    assert groups[(0, 1, 2, 3, 4)] >= 5
    assert groups[(6, 7)] >= 3


def test_no_sharing_reads_every_context_once():
    tables, lengths, _ = make_case(1, groups=(), shared=())
    _, _, _, _, groups, logical, read, _, _ = check_plan(tables, lengths, 16, 1)
    assert groups == [] and read == logical


@pytest.mark.parametrize("group", [1, 2, 4, 8])
def test_plan_invariants_and_dedupe(group):
    tables, lengths, _ = make_case(2, rows=40, groups=(tuple(range(0, 30)), (31, 32, 33)),
                                   shared=(8, 2))
    chunks, members, slots, row_slots, groups, logical, read, _, _ = check_plan(tables, lengths, 16,
                                                                               group)
    assert read < logical
    # a 30-row group is split into member blocks of at most 32 // group rows
    prefix_chunks = [c for c in chunks if c[4] > 1]
    assert max(c[4] for c in prefix_chunks) == min(30, MAX_PAIRS // group)


def test_divergent_tables_share_only_the_common_run():
    tables, lengths, _ = make_case(3, groups=((0, 1, 2),), shared=(4,))
    tables[2, 2] = tables.max() + 1  # row 2 diverges at its third page
    groups = find_shared_prefixes(tables, lengths, 16)
    assert [(r, s) for r, s in groups if 0 in r] == [([0, 1, 2], 2)]
    check_plan(tables, lengths, 16, 1)


def test_short_member_caps_the_shared_run():
    tables, lengths, _ = make_case(4, groups=((0, 1, 2, 3),), shared=(6,), short_row=(3, 40))
    groups = find_shared_prefixes(tables, lengths, 16)
    assert [(r, s) for r, s in groups if 0 in r] == [([0, 1, 2, 3], 40 // 16)]
    check_plan(tables, lengths, 16, 1)


def test_empty_rows_get_no_slots():
    tables, lengths, _ = make_case(5)
    lengths[9] = 0
    chunks, members, slots, row_slots, *_, suffix_lengths = check_plan(tables, lengths, 16, 1)
    assert row_slots[9] == row_slots[10] and suffix_lengths[9] == 0


@pytest.mark.parametrize("group", [1, 3])
def test_plan_execution_matches_oracle(group):
    rng = np.random.default_rng(6)
    page, hkv, d = 16, 2, 32
    tables, lengths, num_blocks = make_case(7, rows=10, width=12, groups=((0, 1, 2, 3), (5, 6)),
                                            shared=(4, 2))
    key = rng.standard_normal((num_blocks, page, hkv, d)).astype(np.float32)
    value = rng.standard_normal((num_blocks, page, hkv, d)).astype(np.float32)
    q = rng.standard_normal((10, hkv * group, d)).astype(np.float32)
    got = run_plan(q, key, value, tables, lengths, page, group, chunk_tokens=48)
    want = oracle.paged_attention(q, key, value, tables, lengths, "f32")
    np.testing.assert_allclose(got, want, atol=1e-5, rtol=1e-5)


def test_chunk_length_fits_one_resident_wave():
    """choose_chunk_tokens: the smallest length (512 doubled) whose (chunk, KV
    head) CTAs fit in one resident wave of the chunk kernel (2 per SM)."""
    from vllm_rlt_b200.kernels.shared_prefix import choose_chunk_tokens

    # 16 groups of 16 rows sharing 2,560 tokens, 16 KV heads, no GQA
    groups = [(list(range(16 * g, 16 * g + 16)), 160) for g in range(16)]
    # 512: 5 x 16 x 16 = 1280 CTAs, 1024: 768, 2048: 512, 4096: 256 <= 296
    assert choose_chunk_tokens(groups, 16, 1, 16, 148) == 4096
    assert choose_chunk_tokens(groups, 16, 1, 16, 500) == 1024  # 1000 slots: 768 CTAs
    # a small shared prefix keeps short chunks (more CTAs for little work)
    assert choose_chunk_tokens([([0, 1], 100)], 16, 1, 16, 148) == 512
    # member blocks multiply the CTAs (40 members at group 1 are 2 blocks); no
    # chunk grows past the longest prefix
    assert choose_chunk_tokens([(list(range(40)), 64)], 16, 1, 8, 4) == 1024
    assert choose_chunk_tokens([], 16, 1, 16, 148) == 512
