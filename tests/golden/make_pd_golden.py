"""Golden vectors for the prefill/decode KV page transport's segment logic.

Run where the reference source is available:

    python tests/golden/make_pd_golden.py --reference /path/to/vllm-rlt

It imports the reference's ``kv_segments`` and ``partition_segments``
(vllm_rlt/pd/transport.py:18-72) and its ``KVCacheManager`` (for real
allocation tables at every depth plane), runs them on seeded cases -- full
and partial blocks, one and several planes, token ranges that start and end
inside blocks, byte and descriptor limits that split segments -- and writes
the inputs and outputs to ``pd_segments.json`` beside this script.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent


def cases():
    # (layers, page, planes, blocks, heads, head_dim, request tokens, [(start, end)], limits)
    yield (3, 4, 4, 24, 4, 4, 9, [(2, 9), (0, 9), (0, 4), (4, 8), (5, 6)], [(333, 3), (10**9, 10**6), (64, 2)])
    yield (2, 16, 1, 40, 2, 8, 70, [(0, 70), (16, 64), (17, 63), (69, 70)], [(4096, 4), (1000, 7)])
    yield (24, 16, 4, 64, 4, 16, 50, [(0, 50), (13, 37), (48, 50)], [(1 << 20, 8), (5000, 3)])


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    sys.path.insert(0, args.reference)
    from vllm_rlt.core.kv_cache_manager import KVCacheManager
    from vllm_rlt.pd.transport import kv_segments, partition_segments

    out = []
    for layers, page, planes, blocks, heads, dim, tokens, ranges, limits in cases():
        cache = KVCacheManager(layers, heads, dim, blocks, page, planes)
        cache.allocate("a", tokens)
        k = cache.key_cache
        element = k.element_size()
        info = dict(
            block_size=page, num_blocks=blocks, num_layers=layers, device=0,
            block_bytes=k.stride(0) * element, layer_bytes=k.stride(1) * element,
            token_bytes=k.stride(2) * element, key_ptr=1 << 20, value_ptr=1 << 40,
        )
        tables = [list(map(int, t)) for t in cache._get_allocation("a").block_tables]
        for start, end in ranges:
            segments = [list(s) for s in kv_segments(info, tables, start, end)]
            parts = []
            for byte_limit, descriptor_limit in limits:
                split = [[[list(x) for x in local], [list(x) for x in remote], size]
                         for local, remote, size in partition_segments(
                             [tuple(s) for s in segments], [tuple(s) for s in segments],
                             byte_limit, descriptor_limit)]
                parts.append(dict(byte_limit=byte_limit, descriptor_limit=descriptor_limit,
                                  parts=split))
            out.append(dict(info=info, tables=tables, start=start, end=end, segments=segments,
                            partitions=parts))
    path = HERE / "pd_segments.json"
    path.write_text(json.dumps(out))
    print(f"wrote {len(out)} cases to {path} ({path.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
