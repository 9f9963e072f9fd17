"""Decode attention on the B200 vs the reference (golden vectors) and the oracle.

Bar: attention within max-abs 1e-5 (fp32) / 2e-3 (+1 output ulp, 16-bit)
of the reference's torch path on the same inputs; KV pools written by the
CUDA write/exit-copy kernels bit-identical to the reference's pools.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
import vllm_rlt_b200 as rb
from gpu_helpers import TORCH, CudaWriter, to_numpy, to_torch
from helpers import assert_close, digest, load, query_inputs, replay_pool, scenario_names
from vllm_rlt_b200 import _lib, workloads

pytestmark = pytest.mark.gpu

SCENARIOS = scenario_names()


def rebuild_on_gpu(name):
    fx = load(name)
    layers, hkv, hq, d, num_blocks, page, loops, seed = (int(x) for x in fx["dims"])
    writer = CudaWriter((num_blocks, layers, page, hkv, d), str(fx["dtype"]))
    replay_pool(fx, name, writer)
    writer.flush()
    return fx, writer


@pytest.mark.parametrize("name", SCENARIOS)
def test_scenario_pool_and_attention_match_reference(name):
    fx, writer = rebuild_on_gpu(name)
    key, value = writer.numpy()
    # KV page writes and LAST-EXITED exit copies: bit-exact with the reference.
    assert digest(key) == str(fx["key_digest"])
    assert digest(value) == str(fx["value_digest"])
    dtype = str(fx["dtype"])
    qi = query_inputs(fx)
    layer = qi["layer"]
    q = to_torch(qi["q"], dtype)
    tables = torch.from_numpy(qi["block_tables"]).cuda()
    lengths = torch.from_numpy(qi["context_lengths"]).cuda()
    out = rb.b200_paged_attention(q, writer.key[:, layer], writer.value[:, layer], tables, lengths)
    torch.cuda.synchronize()
    assert rb.B200PagedAttention("cuda", TORCH[dtype], q.shape[-1], 1).check_errors() == []
    assert_close(to_numpy(out), qi["out"], dtype)


def random_pool(num_blocks, layers, page, hkv, d, dtype, seed=0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    shape = (num_blocks, layers, page, hkv, d)
    key = torch.randn(shape, generator=g, device="cuda", dtype=torch.float32).to(TORCH[dtype])
    value = torch.randn(shape, generator=g, device="cuda", dtype=torch.float32).to(TORCH[dtype])
    return key, value


def oracle_rows(q, key_layer, value_layer, tables, lengths, rows, dtype):
    """Oracle output of the selected rows, reading only those rows' pages."""
    outs = []
    page = key_layer.shape[1]
    for r in rows:
        n = int(lengths[r])
        pages = math.ceil(n / page)
        ids = tables[r, :pages].long()
        k = to_numpy(key_layer[ids])
        v = to_numpy(value_layer[ids])
        t = np.arange(pages, dtype=np.int32)[None]
        outs.append(oracle.paged_attention(to_numpy(q[r : r + 1]), k, v, t, np.array([n]), dtype)[0])
    return np.stack(outs)


def run_case(rows, hq, hkv, d, page, dtype, lengths, layers=3, layer=1, seed=0, width=None,
             pad=-1):
    """Random pool, random fragmented tables; returns everything for checks."""
    lengths = np.asarray(lengths, dtype=np.int32)
    pages_needed = [math.ceil(int(n) / page) for n in lengths]
    width = max(pages_needed + [1]) if width is None else width
    num_blocks = sum(pages_needed) + 7
    rng = np.random.default_rng(seed)
    perm = rng.permutation(num_blocks)
    tables = np.full((rows, width), pad, dtype=np.int32)
    cursor = 0
    for r, n in enumerate(pages_needed):
        tables[r, :n] = perm[cursor : cursor + n]
        cursor += n
    key, value = random_pool(num_blocks, layers, page, hkv, d, dtype, seed)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    q = torch.randn((rows, hq, d), generator=g, device="cuda").to(TORCH[dtype])
    t_tables = torch.from_numpy(tables).cuda()
    t_lengths = torch.from_numpy(lengths).cuda()
    out = rb.paged_attention(q, key[:, layer], value[:, layer], t_tables, t_lengths)
    torch.cuda.synchronize()
    return q, key[:, layer], value[:, layer], t_tables, t_lengths, out


@pytest.mark.parametrize("dtype", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("d", [32, 64, 128, 256, 7, 48])
@pytest.mark.parametrize("group", [1, 2, 3, 8])
def test_head_dims_gqa_and_dtypes_vs_oracle(dtype, d, group):
    if dtype == "f32" and d == 256:
        d = 200  # exercises the generic kernel at fp32
    hkv = 2
    lengths = [1, 15, 16, 17, 33, 100, 257, 600]
    q, k, v, tables, lengths_t, out = run_case(len(lengths), hkv * group, hkv, d, 16, dtype,
                                               lengths)
    expected = oracle_rows(q, k, v, tables, lengths_t, range(len(lengths)), dtype)
    assert_close(to_numpy(out), expected, dtype)


@pytest.mark.parametrize("page", [1, 2, 3, 5, 8, 16, 32])
def test_page_sizes_vs_oracle(page):
    lengths = [1, 2, 7, 31, 64, 65, 300]
    q, k, v, tables, lengths_t, out = run_case(len(lengths), 4, 4, 128, page, "bf16", lengths)
    expected = oracle_rows(q, k, v, tables, lengths_t, range(len(lengths)), "bf16")
    assert_close(to_numpy(out), expected, "bf16")


def test_split_boundaries_and_long_rows_vs_oracle():
    """Lengths around the split chunk (256), the split alignment (32) and the
    split cap (128 splits -> longer splits beyond 32768 tokens); the longer
    rows finish their merge in whichever split CTA arrives last."""
    lengths = [255, 256, 257, 287, 288, 289, 511, 512, 513, 8191, 8192, 8193, 9000, 20000,
               32768, 32769, 40000]
    q, k, v, tables, lengths_t, out = run_case(len(lengths), 16, 16, 128, 16, "bf16", lengths,
                                               layers=1, layer=0)
    expected = oracle_rows(q, k, v, tables, lengths_t, range(len(lengths)), "bf16")
    assert_close(to_numpy(out), expected, "bf16")


def test_batch_beyond_one_schedule_pass_vs_oracle():
    """2,500 rows: the one-CTA schedule kernel orders and scans the rows in
    three passes of 1,024 (batches up to 1,024 rows take its one-pass path);
    sampled rows of every split count, including the first and last scheduled,
    against the oracle, and the same rows alone through a one-pass call."""
    rng = np.random.default_rng(5)
    lengths = rng.integers(1, 1200, size=2500).astype(np.int32)
    lengths[[3, 1700, 2499]] = [9000, 4500, 257]
    q, k, v, tables, lengths_t, out = run_case(len(lengths), 4, 2, 128, 16, "bf16", lengths,
                                               layers=1, layer=0, seed=3)
    picks = sorted(set([0, 3, 1023, 1024, 1700, 2047, 2048, 2499]
                       + rng.choice(len(lengths), 24, replace=False).tolist()))
    expected = oracle_rows(q, k, v, tables, lengths_t, picks, "bf16")
    assert_close(to_numpy(out[picks]), expected, "bf16")
    idx = torch.tensor(picks, device="cuda")
    alone = rb.paged_attention(q[idx], k, v, tables[idx], lengths_t[idx])
    assert torch.equal(alone, out[idx])


def test_fp32_long_rows_vs_oracle():
    lengths = [1, 300, 1000, 4097]
    q, k, v, tables, lengths_t, out = run_case(len(lengths), 16, 16, 128, 16, "f32", lengths,
                                               layers=1, layer=0)
    expected = oracle_rows(q, k, v, tables, lengths_t, range(len(lengths)), "f32")
    assert_close(to_numpy(out), expected, "f32")


def test_zero_length_rows_are_zero_and_padding_is_never_read():
    lengths = [0, 5, 0, 40]
    # pad with a huge id: reading it would be caught by the status word
    q, k, v, tables, lengths_t, out = run_case(len(lengths), 4, 2, 128, 16, "bf16", lengths,
                                               width=8, pad=2**30)
    assert torch.count_nonzero(out[0]) == 0 and torch.count_nonzero(out[2]) == 0
    assert torch.isfinite(out).all()
    assert rb.B200PagedAttention("cuda", torch.bfloat16, 128, 16).check_errors() == []
    expected = oracle_rows(q, k, v, tables, lengths_t, [1, 3], "bf16")
    assert_close(to_numpy(out[[1, 3]]), expected, "bf16")


@pytest.mark.parametrize("dtype", ["f16", "bf16"])
@pytest.mark.parametrize("heads", [2, 4])
def test_ragged_strided_layer_view(dtype, heads):
    """Layer slicing leaves a non-contiguous block stride, as in the real
    cache (reference tests/test_flash_attention.py:50-70)."""
    g = torch.Generator(device="cuda").manual_seed(9)
    td = TORCH[dtype]
    keys = torch.randn(12, 3, 16, 2, 128, generator=g, device="cuda").to(td)[:, 1]
    values = torch.randn(12, 3, 16, 2, 128, generator=g, device="cuda").to(td)[:, 1]
    q = torch.randn(4, heads, 128, generator=g, device="cuda").to(td)
    tables = torch.tensor([[7, 2, 9], [3, 0, 0], [1, 8, 6], [0, 0, 0]], device="cuda",
                          dtype=torch.int32)
    lengths = torch.tensor([35, 1, 47, 0], device="cuda", dtype=torch.int32)
    out = rb.B200PagedAttention(q.device, td, 128, 16)(q, keys, values, tables, lengths)
    expected = oracle.paged_attention(to_numpy(q), to_numpy(keys), to_numpy(values),
                                      tables.cpu().numpy(), lengths.cpu().numpy(), dtype)
    assert_close(to_numpy(out), expected, dtype)
    assert torch.isfinite(out).all()
    assert torch.count_nonzero(out[-1]) == 0


def test_int32_block_ids_use_64bit_physical_offsets():
    """Block id x block stride beyond 2^31 elements must address correctly
    (reference tests/test_attention_64bit.py)."""
    if torch.cuda.mem_get_info()[0] < 9 * 2**30:
        pytest.skip("needs 9 GiB free")
    shape = (2049, 1, 1, 16)
    strides = (2**20, 16, 16, 1)
    key = torch.empty_strided(shape, strides, device="cuda", dtype=torch.float16)
    value = torch.empty_strided(shape, strides, device="cuda", dtype=torch.float16)
    key[0].zero_()
    value[0].fill_(-3)
    key[2048].fill_(1)
    expected = torch.arange(16, device="cuda", dtype=torch.float16).view(1, 1, 16)
    value[2048].copy_(expected)
    query = torch.ones((1, 1, 16), device="cuda", dtype=torch.float16)
    table = torch.tensor([[2048]], device="cuda", dtype=torch.int32)
    lengths = torch.tensor([1], device="cuda", dtype=torch.int32)
    actual = rb.paged_attention(query, key, value, table, lengths)
    torch.cuda.synchronize()
    torch.testing.assert_close(actual, expected, rtol=0, atol=0)


def test_batch_invariance_bit_identical_rows():
    """A row's output never depends on the other rows of the batch
    (reference tests/test_flash_attention.py:192-208)."""
    lengths = [1025, 1029, 1025, 1031, 3000, 17]
    q, k, v, tables, lengths_t, together = run_case(len(lengths), 16, 16, 128, 16, "bf16",
                                                    lengths, layers=2, layer=1)
    for rows in ([2, 3], [3, 0], [1], [5, 4]):
        sub_tables = tables[rows][:, : math.ceil(max(lengths[r] for r in rows) / 16)]
        separate = rb.paged_attention(q[rows], k, v, sub_tables.contiguous(), lengths_t[rows])
        torch.testing.assert_close(separate, together[rows], rtol=0, atol=0)


def test_bad_metadata_is_reported_not_dereferenced():
    """Out-of-pool block ids and over-long lengths raise status bits; the
    kernel skips them instead of reading outside the pool."""
    lengths = [20, 5]
    q, k, v, tables, lengths_t, _ = run_case(2, 4, 4, 128, 16, "bf16", lengths, width=2)
    backend = rb.B200PagedAttention("cuda", torch.bfloat16, 128, 16)
    backend.check_errors()
    bad_tables = tables.clone()
    bad_tables[0, 1] = k.shape[0] + 5  # outside the pool
    out = backend(q, k, v, bad_tables, lengths_t)
    torch.cuda.synchronize()
    assert "block id outside the KV pool" in backend.check_errors()
    assert torch.isfinite(out).all()
    too_long = torch.tensor([20, 999], dtype=torch.int32, device="cuda")
    out = backend(q, k, v, tables, too_long)
    torch.cuda.synchronize()
    assert any("context length" in e for e in backend.check_errors())
    assert torch.count_nonzero(out[1]) == 0


def test_config2_subset_vs_oracle_and_properties():
    """The benchmark workload at full size: 256 rows, LAST-EXITED planes,
    lognormal contexts up to 8192. Sampled rows (shortest, longest, random)
    against the oracle; all rows finite and batch-invariant."""
    plan = workloads.config2_plan(0)
    key, value = random_pool(plan.num_blocks, 1, 16, 16, 128, "bf16", seed=3)
    tables = torch.from_numpy(plan.block_tables()).cuda()
    lengths = torch.from_numpy(plan.context_lengths).cuda()
    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn((plan.num_rows, 16, 128), generator=g, device="cuda").to(torch.bfloat16)
    out = rb.paged_attention(q, key[:, 0], value[:, 0], tables, lengths)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    order = np.argsort(plan.context_lengths)
    rows = sorted(set([int(order[0]), int(order[-1]), int(order[-2])]
                      + np.random.default_rng(1).choice(plan.num_rows, 9, replace=False).tolist()))
    expected = oracle_rows(q, key[:, 0], value[:, 0], tables, plan.context_lengths, rows, "bf16")
    assert_close(to_numpy(out[rows]), expected, "bf16")
    again = rb.paged_attention(q, key[:, 0], value[:, 0], tables, lengths)
    torch.testing.assert_close(again, out, rtol=0, atol=0)  # deterministic


def test_status_word_first_made_under_inference_mode_can_be_cleared():
    """The reference's graph runner calls the backend under
    torch.inference_mode; the per-device status word it may create there must
    stay an ordinary tensor that a later check outside that mode can clear."""
    device = torch.device("cuda", 0)
    _lib._status.pop(0, None)
    with torch.inference_mode():
        word = _lib.status_word(device)
        word.fill_(2)
    assert not word.is_inference()
    assert _lib.read_status(device) == [_lib.STATUS_BITS[2]]
    assert _lib.read_status(device) == []


def test_split_partial_ring_wraps_around():
    """More (row, split) pairs than the split-partial ring holds: 300 rows of
    7,400-8,192 tokens give ~9,300 pairs against a 4,096-slot ring, so slots
    are reused (each waits until the row that used it before has merged) and
    rows' runs of slots straddle the ring's end (split counts of 29-32 do not
    divide the ring). Every sampled row against the oracle, no status bit
    (no wait timed out), results deterministic."""
    rng = np.random.default_rng(12)
    rows, page, hkv, d = 300, 16, 2, 128
    lengths = rng.integers(7400, 8193, size=rows).astype(np.int32)
    pages = [math.ceil(int(n) / page) for n in lengths]
    width = max(pages)
    num_blocks = sum(pages)
    perm = rng.permutation(num_blocks).astype(np.int32)
    tables = np.full((rows, width), -1, dtype=np.int32)
    c = 0
    for r, n in enumerate(pages):
        tables[r, :n] = perm[c : c + n]
        c += n
    key, value = random_pool(num_blocks, 1, page, hkv, d, "bf16", seed=8)
    g = torch.Generator(device="cuda").manual_seed(9)
    q = torch.randn((rows, hkv, d), generator=g, device="cuda").to(torch.bfloat16)
    t = torch.from_numpy(tables).cuda()
    n = torch.from_numpy(lengths).cuda()
    splits = [min(math.ceil(int(x) / 256), 128) for x in lengths]
    assert sum(s for s in splits if s > 1) > 2 * 4096  # wraps the ring twice over
    backend = rb.B200PagedAttention("cuda", torch.bfloat16, d, page)
    out = rb.paged_attention(q, key[:, 0], value[:, 0], t, n)
    torch.cuda.synchronize()
    assert backend.check_errors() == []
    sample = sorted(set(rng.choice(rows, 14, replace=False).tolist() + [0, rows - 1]))
    expected = oracle_rows(q, key[:, 0], value[:, 0], t, lengths, sample, "bf16")
    assert_close(to_numpy(out[sample]), expected, "bf16")
    again = rb.paged_attention(q, key[:, 0], value[:, 0], t, n)
    torch.cuda.synchronize()
    assert torch.equal(again, out)
