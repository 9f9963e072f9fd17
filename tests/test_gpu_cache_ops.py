"""KV write, exit copy, routing metadata, prefill metadata and slot
gather/scatter on the B200: bit-exact against the reference's Triton kernels
(golden vectors from Triton's CPU interpreter) and the oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import vllm_rlt_b200 as rb
from gpu_helpers import to_numpy, to_torch
from helpers import load

pytestmark = pytest.mark.gpu


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("planes", [4, 1])
@pytest.mark.parametrize("uva", [False, True])
def test_metadata_matches_reference_triton(planes, uva):
    fx = load("routing")
    tag = f"meta_p{planes}"
    slots, planes_, width, page, size, n, out_width = fx[f"{tag}_dims"].tolist()
    desc = torch.from_numpy(fx[f"{tag}_desc"])
    desc = desc.pin_memory() if uva else desc.cuda()  # mapped pinned host descriptor
    out = dict(
        slots=torch.full((size,), -7, dtype=torch.int64, device="cuda"),
        positions=torch.full((size,), -7, dtype=torch.int64, device="cuda"),
        lengths=torch.full((size,), -7, dtype=torch.int32, device="cuda"),
        blocks=torch.full((size,), -7, dtype=torch.int64, device="cuda"),
        offsets=torch.full((size,), -7, dtype=torch.int64, device="cuda"),
        out_tables=torch.full((size, width), -7, dtype=torch.int32, device="cuda"),
    )
    rb.metadata(desc, cuda(fx[f"{tag}_tables"]), out["slots"], out["positions"], out["lengths"],
                out["blocks"], out["offsets"], out["out_tables"], n, size, page, planes_,
                out_width)
    torch.cuda.synchronize()
    for key, value in out.items():
        np.testing.assert_array_equal(value.cpu().numpy(), fx[f"{tag}_{key}"], err_msg=key)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_finalize_matches_reference_triton(dtype):
    fx = load("routing")
    blocks, layers, page, hkv, d, planes, width, slots = fx["fin_dims"].tolist()
    key_np, value_np = fx["fin_key_before"], fx["fin_value_before"]
    if dtype == "bf16":
        key_np, value_np = oracle.f32_to_bf16(key_np), oracle.f32_to_bf16(value_np)
    key = to_torch(key_np, dtype)
    value = to_torch(value_np, dtype)
    rb.finalize(cuda(fx["fin_desc"]), cuda(fx["fin_tables"]), key, value)
    exp_k, exp_v = key_np.copy(), value_np.copy()
    oracle.finalize(fx["fin_desc"], fx["fin_tables"], exp_k, exp_v, planes, page)
    if dtype == "f32":  # the reference's own kernel output for this dtype
        np.testing.assert_array_equal(exp_k, fx["fin_key_after"])
    np.testing.assert_array_equal(to_numpy(key), exp_k)
    np.testing.assert_array_equal(to_numpy(value), exp_v)


def test_kv_write_matches_index_put_on_strided_inputs():
    """key_cache[blocks, layer, offsets] = k[:n], with k a strided view and
    extra padding rows beyond n (reference kv_cache_manager.py:531-532)."""
    g = torch.Generator(device="cuda").manual_seed(0)
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        pool = torch.randn(30, 4, 8, 2, 64, generator=g, device="cuda").to(dtype)
        vpool = torch.randn(30, 4, 8, 2, 64, generator=g, device="cuda").to(dtype)
        qkv = torch.randn(11, 3, 2, 64, generator=g, device="cuda").to(dtype)
        k, v = qkv[:, 1], qkv[:, 2]  # non-contiguous row stride
        blocks = torch.tensor([3, 29, 0, 7, 7, 12, 3, 18, 1], dtype=torch.int64, device="cuda")
        offsets = torch.tensor([0, 7, 5, 1, 2, 6, 3, 0, 4], dtype=torch.int64, device="cuda")
        exp_k, exp_v = pool.clone(), vpool.clone()
        exp_k[blocks, 2, offsets] = k[: len(blocks)]
        exp_v[blocks, 2, offsets] = v[: len(blocks)]
        rb.write_kv(pool, vpool, 2, blocks, offsets, k, v)
        assert torch.equal(pool, exp_k) and torch.equal(vpool, exp_v)


def test_kv_write_bad_address_reports_status():
    pool = torch.zeros(4, 1, 4, 1, 16, device="cuda", dtype=torch.bfloat16)
    vpool = torch.zeros_like(pool)
    k = torch.ones(2, 1, 16, device="cuda", dtype=torch.bfloat16)
    backend = rb.B200PagedAttention("cuda", torch.bfloat16, 16, 4)
    backend.check_errors()
    rb.write_kv(pool, vpool, 0, torch.tensor([9, 1], device="cuda"), torch.tensor([0, 2], device="cuda"), k, k)
    torch.cuda.synchronize()
    assert "block id outside the KV pool" in backend.check_errors()
    assert torch.count_nonzero(pool) == 16  # only the valid row landed


def test_stage_and_expand_prefill_match_reference_triton():
    fx = load("routing")
    source = cuda(fx["stage_source"])
    target = torch.zeros_like(source)
    target32 = torch.zeros(len(source), dtype=torch.int32, device="cuda")
    rb.stage_prefill(source, target, target32, len(source))
    np.testing.assert_array_equal(target.cpu().numpy(), fx["stage_target"])
    np.testing.assert_array_equal(target32.cpu().numpy(), fx["stage_target32"])
    n, width, page = fx["expand_dims"].tolist()
    blocks = torch.full((n,), -7, dtype=torch.int64, device="cuda")
    offsets = torch.full((n,), -7, dtype=torch.int64, device="cuda")
    rb.expand_prefill(cuda(fx["expand_positions"]), cuda(fx["expand_sequences"]),
                      cuda(fx["expand_tables"]), blocks, offsets, n, width, page)
    np.testing.assert_array_equal(blocks.cpu().numpy(), fx["expand_blocks"])
    np.testing.assert_array_equal(offsets.cpu().numpy(), fx["expand_offsets"])


def test_gather_scatter_match_reference_triton():
    fx = load("routing")
    pool = to_torch(fx["gather_pool"], "bf16")
    out = torch.full((8, 300), 5.0, dtype=torch.bfloat16, device="cuda")
    rb.gather(pool, cuda(fx["gather_slots"]), out, 5, 8)
    np.testing.assert_array_equal(to_numpy(out), fx["gather_out"])
    tokens = cuda(fx["scatter_before"])
    rb.scatter(cuda(fx["scatter_values"]), cuda(fx["scatter_slots"]), tokens, 4)
    np.testing.assert_array_equal(tokens.cpu().numpy(), fx["scatter_after"])
