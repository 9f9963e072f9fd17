"""rlt_paged_decode_noalloc: decode attention for callers that cannot allocate.

Callers such as a serving runtime that has reserved all device memory for
its own pool, or a host that forbids driver allocations once it is running,
cannot hand the decode kernel a freshly allocated split-KV workspace. The
no-allocation entry point uses a fixed device array inside the library
instead. These tests call it through the C ABI and check it against the
workspace-taking entry point, rlt_paged_decode, on two calls in a row (the
second call reuses the shared array the first one left behind), and check
that a launch shape too large for the array is refused without a launch.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from helpers import assert_close
from vllm_rlt_b200 import _lib

pytestmark = pytest.mark.gpu

RLT_E_SCRATCH = -8


def make_inputs(seed, rows, lengths, hq=16, hkv=16, d=128, page=16, width=None):
    rng = np.random.default_rng(seed)
    pages = [math.ceil(int(n) / page) for n in lengths]
    width = max(pages) if width is None else width
    num_blocks = sum(pages) + 5
    perm = rng.permutation(num_blocks)
    tables = np.full((rows, width), -1, dtype=np.int32)
    c = 0
    for r, n in enumerate(pages):
        tables[r, :n] = perm[c : c + n]
        c += n
    g = torch.Generator(device="cuda").manual_seed(seed)
    key = torch.randn(num_blocks, 2, page, hkv, d, generator=g, device="cuda").to(torch.bfloat16)
    value = torch.randn(num_blocks, 2, page, hkv, d, generator=g, device="cuda").to(torch.bfloat16)
    q = torch.randn(rows, hq, d, generator=g, device="cuda").to(torch.bfloat16)
    return dict(q=q, k=key[:, 1], v=value[:, 1], tables=torch.from_numpy(tables).cuda(),
                lengths=torch.tensor(lengths, dtype=torch.int32, device="cuda"))


def shape_args(x):
    q, k, v, tables = x["q"], x["k"], x["v"], x["tables"]
    rows, hq, d = q.shape
    return [rows, hq, k.shape[2], d, k.shape[1], tables.shape[1], k.shape[0],
            q.stride(0), q.stride(1), k.stride(0), k.stride(1), k.stride(2),
            v.stride(0), v.stride(1), v.stride(2), tables.stride(0)]


def decode_with_workspace(lib, x):
    out = torch.empty_like(x["q"])
    rows, hq, d = x["q"].shape
    need = lib.rlt_paged_decode_workspace_bytes(rows, hq, d, x["k"].shape[1], x["tables"].shape[1])
    ws = torch.empty(max(need, 16), dtype=torch.uint8, device="cuda")
    code = lib.rlt_paged_decode(
        x["q"].data_ptr(), x["k"].data_ptr(), x["v"].data_ptr(), x["tables"].data_ptr(),
        x["lengths"].data_ptr(), out.data_ptr(), ws.data_ptr(), need, None, _lib.BF16,
        *shape_args(x), out.stride(0), out.stride(1), x["q"].shape[-1] ** -0.5,
        torch.cuda.current_stream().cuda_stream)
    assert code == 0
    return out


def decode_no_alloc(lib, x, out):
    return lib.rlt_paged_decode_noalloc(
        x["q"].data_ptr(), x["k"].data_ptr(), x["v"].data_ptr(), x["tables"].data_ptr(),
        x["lengths"].data_ptr(), out.data_ptr(), None, _lib.BF16,
        *shape_args(x), out.stride(0), out.stride(1), x["q"].shape[-1] ** -0.5,
        torch.cuda.current_stream().cuda_stream)


def test_no_alloc_matches_workspace_entry_point_on_two_calls():
    lib = _lib.load()
    first = make_inputs(1, 40, list(np.random.default_rng(1).integers(1, 3000, size=40)))
    second = make_inputs(2, 24, list(np.random.default_rng(2).integers(200, 4000, size=24)))
    expected, got = [], []
    for x in (first, second):
        rows, hq, d = x["q"].shape
        need = lib.rlt_paged_decode_workspace_bytes(rows, hq, d, 16, x["tables"].shape[1])
        assert 0 < need <= 16 << 20  # multi-split rows that fit the static scratch
        expected.append(decode_with_workspace(lib, x))
        got.append(torch.full_like(x["q"], float("nan")))
    # two no-allocation calls in a row: the second reuses the shared scratch
    assert decode_no_alloc(lib, first, got[0]) == 0
    assert decode_no_alloc(lib, second, got[1]) == 0
    torch.cuda.synchronize()
    to_u16 = lambda t: t.cpu().view(torch.int16).numpy().view(np.uint16)  # noqa: E731
    for a, b in zip(got, expected):
        assert_close(to_u16(a), to_u16(b), "bf16")
        assert torch.equal(a, b)  # same kernels and split plan: identical bits
    # and directly against the CPU oracle for a few rows of the second call
    rows = [0, 7, 23]
    x = second
    want = oracle.paged_attention(to_u16(x["q"][rows]), to_u16(x["k"]), to_u16(x["v"]),
                                  x["tables"][rows].cpu().numpy(),
                                  x["lengths"][rows].cpu().numpy(), "bf16")
    assert_close(to_u16(got[1][rows]), want, "bf16")


def test_no_alloc_refuses_shapes_beyond_its_static_scratch():
    lib = _lib.load()
    # 64 query heads of head_dim 256 at table width 512 (page 16): the ring of
    # split partials (1024 slots x 64 heads x 258 fp32) needs 68 MB.
    x = make_inputs(3, 64, [100] * 64, hq=64, hkv=8, d=256, width=512)
    assert lib.rlt_paged_decode_workspace_bytes(64, 64, 256, 16, 512) > 16 << 20
    out = torch.zeros_like(x["q"])
    assert decode_no_alloc(lib, x, out) == RLT_E_SCRATCH
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0  # nothing was launched
