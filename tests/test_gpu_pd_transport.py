"""KV page transport on the GPU: a request's tokens [start, end) at every
depth plane, layer, K and V land bit-exactly in the peer pool's pages, nothing
else in the peer pool changes; in-flight back-pressure; a second GPU as the
peer when the box has one."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from vllm_rlt_b200.pd import PageTransport

pytestmark = pytest.mark.gpu


def pools(device, blocks=40, layers=3, page=16, heads=2, dim=64, dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    k = torch.randn(blocks, layers, page, heads, dim, generator=g).to(dtype).to(device)
    v = torch.randn(blocks, layers, page, heads, dim, generator=g).to(dtype).to(device)
    return k, v


def tables_for(rng, planes, pages, blocks):
    perm = rng.permutation(blocks)
    return [list(map(int, perm[p * pages:(p + 1) * pages])) for p in range(planes)]


def run_transfer(dst_device, start, end, planes=4, page=16, seed=1):
    rng = np.random.default_rng(seed)
    pages = -(-end // page)
    src_k, src_v = pools("cuda:0", blocks=planes * pages + 4, page=page, seed=seed)
    dst_k, dst_v = pools(dst_device, blocks=planes * pages + 6, page=page, seed=seed + 100)
    before_k, before_v = dst_k.clone(), dst_v.clone()
    local = tables_for(rng, planes, pages, src_k.shape[0])
    remote = tables_for(rng, planes, pages, dst_k.shape[0])
    transport = PageTransport(src_k, src_v, page, transfer_chunk_bytes=1 << 16,
                              descriptor_limit=7, max_inflight_bytes=1 << 30)
    transport.connect("decode", dst_k, dst_v)
    assert transport.submit("req", 0, "decode", local, remote, start, end)
    assert transport.busy("req")
    torch.cuda.synchronize()
    done = transport.poll()
    assert [t.transfer_id for t in done] == ["req"] and not transport.busy("req")
    transport.close()
    want_k, want_v = before_k.clone(), before_v.clone()
    for lt, rt in zip(local, remote):
        for token in range(start, end):
            lb, rb = lt[token // page], rt[token // page]
            want_k[rb, :, token % page] = src_k[lb, :, token % page].to(dst_device)
            want_v[rb, :, token % page] = src_v[lb, :, token % page].to(dst_device)
    assert torch.equal(dst_k, want_k)
    assert torch.equal(dst_v, want_v)


@pytest.mark.parametrize("start,end", [(0, 64), (0, 70), (5, 37), (33, 34)])
def test_transfer_same_device(start, end):
    run_transfer("cuda:0", start, end)


def test_backpressure_and_geometry_checks():
    src_k, src_v = pools("cuda:0")
    dst_k, dst_v = pools("cuda:0", seed=3)
    transport = PageTransport(src_k, src_v, 16, transfer_chunk_bytes=1 << 12,
                              max_inflight_bytes=1 << 14)
    transport.connect("decode", dst_k, dst_v)
    tables = [[0, 1, 2, 3]]
    # 64 tokens x 3 layers x 2 heads x 64 dims x 2 B x (K, V) = 96 KiB > 16 KiB budget
    assert not transport.submit("big", 0, "decode", tables, tables, 0, 64)
    assert not transport.pending
    other_k = torch.zeros(40, 2, 16, 2, 64, dtype=torch.bfloat16, device="cuda:0")
    with pytest.raises(ValueError, match="different KV geometry"):
        transport.connect("bad", other_k, torch.zeros_like(other_k))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs a second GPU")
@pytest.mark.parametrize("start,end", [(0, 64), (7, 61)])
def test_transfer_to_peer_gpu(start, end):
    run_transfer("cuda:1", start, end)
