"""Packed chunked prefill on the B200 vs the reference (golden vectors)."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
import vllm_rlt_b200 as rb
from gpu_helpers import TORCH, CudaWriter, to_numpy, to_torch
from helpers import assert_close, digest, prefill_case, prefill_names
from vllm_rlt_b200 import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name", prefill_names())
def test_packed_prefill_matches_reference(name):
    fx, writer, inputs = prefill_case(name, CudaWriter)
    writer.flush()
    dtype = str(fx["dtype"])
    d = inputs[0][2].shape[-1]
    blocks = torch.from_numpy(fx["write_blocks"]).cuda()
    offsets = torch.from_numpy(fx["write_offsets"]).cuda()
    backend = rb.B200PagedAttention("cuda", TORCH[dtype], d, 16)
    for layer, (k, v, q) in enumerate(inputs):
        rb.write_kv(writer.key, writer.value, layer, blocks, offsets, to_torch(k, dtype),
                    to_torch(v, dtype))
        out = backend.prefill(to_torch(q, dtype), writer.key[:, layer], writer.value[:, layer],
                              torch.from_numpy(fx["block_tables"]).cuda(),
                              torch.from_numpy(fx["context_lengths"]).cuda(),
                              torch.from_numpy(fx["cu_seqlens_q"]).cuda(), int(fx["max_seqlen_q"]))
        torch.cuda.synchronize()
        assert backend.check_errors() == []
        assert_close(to_numpy(out), fx[f"out{layer}"], dtype)
    key, value = writer.numpy()
    assert digest(key) == str(fx["key_digest"])
    assert digest(value) == str(fx["value_digest"])


def test_tensor_core_path_selection():
    lib = _lib.load()
    assert lib.rlt_paged_prefill_uses_tensor_cores(_lib.BF16, 128, 16) == 1
    assert lib.rlt_paged_prefill_uses_tensor_cores(_lib.F16, 128, 32) == 1
    assert lib.rlt_paged_prefill_uses_tensor_cores(_lib.F32, 128, 16) == 0
    assert lib.rlt_paged_prefill_uses_tensor_cores(_lib.BF16, 64, 16) == 0
    assert lib.rlt_paged_prefill_uses_tensor_cores(_lib.BF16, 128, 5) == 0


def _prefix_reuse_case(dtype, page=16, hkv=4, seed=7, prompt=(300, 517, 64, 1000),
                       prefix=(0, 256, 17, 640), chunk_cap=200):
    rng = np.random.default_rng(seed)
    d = 128
    chunk = [min(chunk_cap, p - s) for p, s in zip(prompt, prefix)]
    lengths = [s + c for s, c in zip(prefix, chunk)]
    width = max(math.ceil(n / page) for n in lengths)
    num_blocks = sum(math.ceil(n / page) for n in lengths) + 3
    perm = rng.permutation(num_blocks)
    tables = np.full((len(lengths), width), -1, dtype=np.int32)
    c = 0
    for i, n in enumerate(lengths):
        pages = math.ceil(n / page)
        tables[i, :pages] = perm[c : c + pages]
        c += pages
    g = torch.Generator(device="cuda").manual_seed(5)
    td = TORCH[dtype]
    key = torch.randn(num_blocks, 1, page, hkv, d, generator=g, device="cuda").to(td)
    value = torch.randn(num_blocks, 1, page, hkv, d, generator=g, device="cuda").to(td)
    cu = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    q = torch.randn(int(cu[-1]), hkv, d, generator=g, device="cuda").to(td)
    out = rb.paged_prefill(q, key[:, 0], value[:, 0], torch.from_numpy(tables).cuda(),
                           torch.tensor(lengths, dtype=torch.int32, device="cuda"),
                           torch.from_numpy(cu).cuda(), max(chunk))
    expected = oracle.paged_prefill(to_numpy(q), to_numpy(key[:, 0]), to_numpy(value[:, 0]),
                                    tables, np.array(lengths), cu, dtype)
    return out, expected


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_chunked_prefill_with_prefix_reuse_vs_oracle(dtype):
    """Config-4-shaped (scaled down): several sequences, chunk after a reused
    prefix, fragmented tables, GQA 1, head_dim 128."""
    out, expected = _prefix_reuse_case(dtype)
    assert_close(to_numpy(out), expected, dtype)


# The reference's own bound for its tensor-core prefill (FA4, which rounds P
# to the input dtype before the PV product) against the fp32 torch path:
# tests/test_flash_attention.py:66-67 and :187-188. Kernel versions 1-5 round
# P to bf16 the same way; on these cases their largest bf16 error is 2.4e-3
# beyond one output ulp (a query row that attends only four keys), so they
# are held to this bound for bf16. Versions 6 and 7, which split P into a bf16
# hi + lo pair where few keys are attended (6) or everywhere (7), and every
# fp16 version are held to the stated bound: max-abs 2e-3 plus one ulp.
FA4_TOLERANCE = {"bf16": dict(atol=0.015, rtol=0.02, ulps=0), "f16": {}}
ROUNDED_P_VERSIONS = (1, 2, 3, 4, 5)


def _with_version(version, fn):
    lib = _lib.load()
    previous = lib.rlt_prefill_tc_select(version)
    try:
        result = fn()
        torch.cuda.synchronize()
    finally:
        lib.rlt_prefill_tc_select(previous)
    return result


@pytest.mark.parametrize("page", [16, 64])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_each_tensor_core_kernel_vs_oracle(dtype, page):
    """Every tensor-core prefill kernel (1: single tile; 2: two tiles, P in
    shared memory; 3: two tiles, P in TMEM; 4: as 3 with each row's softmax
    split over two warps by key-column half; 5: as 3 with the softmax
    warpgroups' registers raised so a row's scores stay in registers for one
    pass; 6: as 5 with bf16 P split into hi + lo in query tiles whose rows
    attend fewer than 512 keys; 7: as 6 in every tile; 8: as 6 with 64-key
    steps and two S buffers per query tile) on long chunks that run many key
    tiles, with ragged tails and a chunk shorter than one tile. Kernels 2 and
    3 differ only in where P is held, so their outputs are bit-identical."""
    case = dict(page=page, seed=11, prompt=(1500, 2100, 90, 777), prefix=(0, 700, 30, 1),
                chunk_cap=1100)
    outs = {}
    for version in (1, 2, 3, 4, 5, 6, 7, 8):
        out, expected = _with_version(version, lambda: _prefix_reuse_case(dtype, **case))
        if version in ROUNDED_P_VERSIONS:
            assert_close(to_numpy(out), expected, dtype, **FA4_TOLERANCE[dtype])
        else:
            assert_close(to_numpy(out), expected, dtype)
        outs[version] = out
    assert torch.equal(outs[2], outs[3])
    if dtype == "f16":  # fp16's P is never split: 6 and 7 are 5
        assert torch.equal(outs[5], outs[6]) and torch.equal(outs[5], outs[7])


@pytest.mark.parametrize("dtype,d,group", [("bf16", 128, 1), ("f16", 128, 2), ("f32", 64, 1)])
def test_prefill_batch_invariance_bit_identical_sequences(dtype, d, group):
    """A sequence's prefill output does not depend on which other sequences
    share the launch (the decode counterpart is the reference's
    tests/test_flash_attention.py:192-208): every tile's reduction order is
    a function of its own sequence. Covers the tensor-core kernel (bf16 /
    fp16, head_dim 128, GQA 1 and 2) and the CUDA-core path (fp32)."""
    rng = np.random.default_rng(21)
    page, hkv = 16, 2
    prefix = [0, 300, 1100, 40]
    chunk = [700, 260, 333, 17]
    lengths = [s + c for s, c in zip(prefix, chunk)]
    width = max(math.ceil(n / page) for n in lengths)
    num_blocks = sum(math.ceil(n / page) for n in lengths) + 2
    perm = rng.permutation(num_blocks)
    tables = np.full((4, width), -1, dtype=np.int32)
    c = 0
    for i, n in enumerate(lengths):
        tables[i, : math.ceil(n / page)] = perm[c : c + math.ceil(n / page)]
        c += math.ceil(n / page)
    g = torch.Generator(device="cuda").manual_seed(9)
    td = TORCH[dtype]
    key = torch.randn(num_blocks, page, hkv, d, generator=g, device="cuda").to(td)
    value = torch.randn(num_blocks, page, hkv, d, generator=g, device="cuda").to(td)
    q = [torch.randn(n, hkv * group, d, generator=g, device="cuda").to(td) for n in chunk]

    def run(rows):
        cu = np.concatenate([[0], np.cumsum([chunk[r] for r in rows])]).astype(np.int32)
        out = rb.paged_prefill(torch.cat([q[r] for r in rows]), key, value,
                               torch.from_numpy(tables[rows]).cuda(),
                               torch.tensor([lengths[r] for r in rows], dtype=torch.int32,
                                            device="cuda"),
                               torch.from_numpy(cu).cuda(), max(chunk[r] for r in rows))
        torch.cuda.synchronize()
        return [out[cu[i] : cu[i + 1]] for i in range(len(rows))]

    together = run([0, 1, 2, 3])
    for rows in ([2, 3], [3, 0], [1], [2]):
        for r, part in zip(rows, run(rows)):
            assert torch.equal(part, together[r]), (rows, r)


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
@pytest.mark.parametrize("version", [1, 5, 6, 8])
def test_pool_garbage_past_the_context_never_reaches_the_output(dtype, version):
    """Pages are copied whole, so the last context page's slots past the
    context come along; a pool allocated without initialisation may hold NaN
    there (the reference's KVCacheManager allocates its pools with
    torch.empty). Every slot the context does not cover is NaN here; the
    output must equal the oracle, which reads only the context."""
    rng = np.random.default_rng(17)
    page, hkv, d = 16, 2, 128
    prefix, chunk = [0, 37, 5], [23, 91, 140]
    lengths = [s + c for s, c in zip(prefix, chunk)]
    width = max(math.ceil(n / page) for n in lengths)
    num_blocks = sum(math.ceil(n / page) for n in lengths) + 2
    perm = rng.permutation(num_blocks)
    tables = np.full((3, width), -1, dtype=np.int32)
    c = 0
    for i, n in enumerate(lengths):
        tables[i, : math.ceil(n / page)] = perm[c : c + math.ceil(n / page)]
        c += math.ceil(n / page)
    td = TORCH[dtype]
    g = torch.Generator(device="cuda").manual_seed(3)
    key = torch.full((num_blocks, page, hkv, d), float("nan"), device="cuda", dtype=td)
    value = torch.full_like(key, float("nan"))
    for i, n in enumerate(lengths):
        pos = torch.arange(n, device="cuda")
        blocks = torch.from_numpy(tables[i]).cuda().long()[pos // page]
        key[blocks, pos % page] = torch.randn(n, hkv, d, generator=g, device="cuda").to(td)
        value[blocks, pos % page] = torch.randn(n, hkv, d, generator=g, device="cuda").to(td)
    cu = np.concatenate([[0], np.cumsum(chunk)]).astype(np.int32)
    q = torch.randn(int(cu[-1]), hkv, d, generator=g, device="cuda").to(td)
    out = _with_version(version, lambda: rb.paged_prefill(
        q, key, value, torch.from_numpy(tables).cuda(),
        torch.tensor(lengths, dtype=torch.int32, device="cuda"), torch.from_numpy(cu).cuda(),
        max(chunk)))
    assert torch.isfinite(out).all()
    expected = oracle.paged_prefill(to_numpy(q), to_numpy(key), to_numpy(value), tables,
                                    np.array(lengths), cu, dtype)
    tol = FA4_TOLERANCE[dtype] if version in ROUNDED_P_VERSIONS else {}
    assert_close(to_numpy(out), expected, dtype, **tol)
