"""Every kernel is capturable in a CUDA graph: static metadata buffers of the
fixed graph width (vllm_rlt/worker/cuda_graph.py:77-94), lengths that change
between replays, replay == eager."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import vllm_rlt_b200 as rb

pytestmark = pytest.mark.gpu


def test_decode_and_kv_write_capture_replay_matches_eager():
    torch.manual_seed(0)
    page, hkv, hq, d, layers = 16, 16, 16, 128, 2
    rows, graph_width = 8, 4096  # ceil(65536 / 16): the reference's graph table width
    num_blocks = 1600  # 8 rows x at most 188 pages, disjoint per row
    key = torch.randn(num_blocks, layers, page, hkv, d, device="cuda").to(torch.bfloat16)
    value = torch.randn_like(key)
    static = dict(
        q=torch.zeros(rows, hq, d, device="cuda", dtype=torch.bfloat16),
        k=torch.zeros(rows, hkv, d, device="cuda", dtype=torch.bfloat16),
        v=torch.zeros(rows, hkv, d, device="cuda", dtype=torch.bfloat16),
        blocks=torch.zeros(rows, dtype=torch.int64, device="cuda"),
        offsets=torch.zeros(rows, dtype=torch.int64, device="cuda"),
        tables=torch.zeros(rows, graph_width, dtype=torch.int32, device="cuda"),
        lengths=torch.zeros(rows, dtype=torch.int32, device="cuda"),
    )
    backend = rb.B200PagedAttention("cuda", torch.bfloat16, d, page)

    def step():
        outs = []
        for layer in range(layers):
            rb.write_kv(key, value, layer, static["blocks"], static["offsets"], static["k"],
                        static["v"])
            outs.append(backend(static["q"], key[:, layer], value[:, layer], static["tables"],
                                static["lengths"]))
        return outs

    def load_inputs(seed):
        rng = np.random.default_rng(seed)
        lengths = rng.integers(1, 3000, size=rows)
        perm = rng.permutation(num_blocks)
        tables = np.zeros((rows, graph_width), dtype=np.int32)
        c = 0
        blocks, offsets = [], []
        for r, n in enumerate(lengths):
            pages = math.ceil(int(n) / page)
            tables[r, :pages] = perm[c : c + pages]
            c += pages
            blocks.append(tables[r, (int(n) - 1) // page])
            offsets.append((int(n) - 1) % page)
        static["tables"].copy_(torch.from_numpy(tables))
        static["lengths"].copy_(torch.from_numpy(lengths.astype(np.int32)))
        static["blocks"].copy_(torch.tensor(blocks))
        static["offsets"].copy_(torch.tensor(offsets))
        for name in ("q", "k", "v"):
            static[name].copy_(torch.randn_like(static[name], dtype=torch.float32))

    load_inputs(1)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(stream)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        graph_out = step()
    for seed in (2, 3):
        load_inputs(seed)
        pool_before = (key.clone(), value.clone())
        graph.replay()
        torch.cuda.synchronize()
        replayed = [o.clone() for o in graph_out]
        replay_pool = (key.clone(), value.clone())
        key.copy_(pool_before[0])
        value.copy_(pool_before[1])
        eager = step()
        torch.cuda.synchronize()
        for a, b in zip(replayed, eager):
            torch.testing.assert_close(a, b, rtol=0, atol=0)
        assert torch.equal(replay_pool[0], key) and torch.equal(replay_pool[1], value)
    assert backend.check_errors() == []


@pytest.mark.parametrize("d", [64, 128])  # CUDA-core path, tensor-core path
def test_prefill_capture(d):
    torch.manual_seed(1)
    page, hkv = 16, 4
    key = torch.randn(64, 1, page, hkv, d, device="cuda").to(torch.float16)
    value = torch.randn_like(key)
    tables = torch.arange(64, dtype=torch.int32, device="cuda").view(4, 16)
    lengths = torch.tensor([40, 100, 17, 256], dtype=torch.int32, device="cuda")
    cu = torch.tensor([0, 5, 9, 26, 40], dtype=torch.int32, device="cuda")
    q = torch.randn(40, hkv, d, device="cuda").to(torch.float16)
    eager = rb.paged_prefill(q, key[:, 0], value[:, 0], tables, lengths, cu, 17)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        rb.paged_prefill(q, key[:, 0], value[:, 0], tables, lengths, cu, 17)
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(graph):
        out = rb.paged_prefill(q, key[:, 0], value[:, 0], tables, lengths, cu, 17)
    graph.replay()
    torch.cuda.synchronize()
    torch.testing.assert_close(out, eager, rtol=0, atol=0)
