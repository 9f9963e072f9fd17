"""Generate golden vectors from the reference implementation (vllm-rlt).

Run in a container where the reference source is available:

    python tests/golden/make_golden.py --reference /path/to/vllm-rlt

It imports the reference package and runs, on the CPU:
  * its KV cache manager (allocate / write / finalize_token / _prepare_batch),
  * its torch attention oracle (torch_paged_attention),
  * its Triton kernels (paged attention, metadata, finalize, prefill metadata,
    gather/scatter) through Triton's CPU interpreter (TRITON_INTERPRET=1).

Fixtures stay small: K/V values are drawn from a seeded numpy generator in a
recorded order, so a test rebuilds the pool by replaying the recorded writes
and checks the rebuilt pool against the reference pool's SHA-256 digest
before using it. Outputs are stored in full.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"  # must precede any triton import

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from vllm_rlt_b200 import workloads  # noqa: E402

TORCH_DTYPES = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}


def storage(t: torch.Tensor) -> np.ndarray:
    """Tensor -> numpy storage form (bf16 as uint16 bits)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def digest(t: torch.Tensor) -> str:
    return hashlib.sha256(storage(t).tobytes()).hexdigest()


def values(rng, shape, dtype):
    return torch.from_numpy(rng.standard_normal(shape, dtype=np.float32)).to(TORCH_DTYPES[dtype])


# ----------------------------------------------------------------- scenarios


def scenario(name, *, layers, hkv, hq, d, num_blocks, page, loops, dtype, layout, ops, queries,
             seed, free_order=None, scale_values=None):
    """Replay ``ops`` on a reference KVCacheManager and record everything.

    ops: list of tuples
      ("alloc", rid, max_tokens) | ("free", rid)
      ("write", layer, rid, depth, pos)        -- values drawn in order
      ("finalize", rid, pos, exit_depth)
    queries: list of (layer, [(rid, depth, pos), ...]); q drawn per query.
    """
    from vllm_rlt.core.kv_cache_manager import KVCacheManager
    from vllm_rlt.kernels.paged_attention import torch_paged_attention
    from vllm_rlt.kernels.triton_attention import paged_attention as triton_paged_attention

    cache = KVCacheManager(layers, hkv, d, num_blocks, page, loops, "cpu", TORCH_DTYPES[dtype],
                           "torch", layout)
    cache.key_cache.zero_()
    cache.value_cache.zero_()
    if free_order is not None:
        cache._free_blocks = list(reversed([int(b) for b in free_order]))
    rng = np.random.default_rng([seed, 1])
    rids = {}
    op_codes = []  # (kind, a, b, c, e) int rows
    for op in ops:
        kind = op[0]
        if kind == "alloc":
            rid = rids.setdefault(op[1], len(rids))
            assert cache.allocate(op[1], op[2])
            op_codes.append((0, rid, op[2], 0, 0))
        elif kind == "free":
            cache.free(op[1])
            op_codes.append((1, rids[op[1]], 0, 0, 0))
        elif kind == "write":
            _, layer, rid_name, depth, pos = op
            k = values(rng, (1, hkv, d), dtype)
            v = values(rng, (1, hkv, d), dtype)
            if scale_values is not None:
                k, v = scale_values(k, v, rid_name, depth)
            cache.write(layer, [rid_name], [depth], [pos], k, v)
            op_codes.append((2, layer, rids[rid_name], depth, pos))
        elif kind == "finalize":
            _, rid_name, pos, exit_depth = op
            cache.finalize_token(rid_name, pos, exit_depth)
            op_codes.append((3, rids[rid_name], pos, exit_depth, 0))
        else:
            raise ValueError(kind)
    names = sorted(rids, key=rids.get)
    tables = np.full((len(names), cache.storage_depths, num_blocks), -1, dtype=np.int32)
    for name_, index in rids.items():
        if name_ in cache._allocations:
            for plane, table in enumerate(cache._allocations[name_].block_tables):
                tables[index, plane, : len(table)] = table
    out = {
        "dims": np.array([layers, hkv, hq, d, num_blocks, page, loops, seed], dtype=np.int64),
        "layout": np.array(layout),
        "dtype": np.array(dtype),
        "ops": np.array(op_codes, dtype=np.int64).reshape(-1, 5),
        "alloc_tables": tables,
        "key_digest": np.array(digest(cache.key_cache)),
        "value_digest": np.array(digest(cache.value_cache)),
    }
    for qi, (layer, rows) in enumerate(queries):
        ids = [r[0] for r in rows]
        depths = [r[1] for r in rows]
        positions = [r[2] for r in rows]
        batch = cache._prepare_batch(ids, depths, positions, for_write=False)
        q = values(rng, (len(rows), hq, d), dtype)
        expected = torch_paged_attention(q, cache.key_cache[:, layer], cache.value_cache[:, layer],
                                         batch.block_tables, batch.context_lengths)
        triton_out = triton_paged_attention(q, cache.key_cache[:, layer],
                                            cache.value_cache[:, layer], batch.block_tables,
                                            batch.context_lengths)
        out[f"q{qi}_layer"] = np.array(layer)
        out[f"q{qi}_rows"] = np.array([[rids[i], dd, p] for i, dd, p in rows], dtype=np.int64)
        out[f"q{qi}_q"] = storage(q)
        out[f"q{qi}_block_tables"] = batch.block_tables.numpy()
        out[f"q{qi}_context_lengths"] = batch.context_lengths.numpy()
        out[f"q{qi}_write_blocks"] = batch.write_blocks.numpy()
        out[f"q{qi}_write_offsets"] = batch.write_offsets.numpy()
        out[f"q{qi}_out"] = storage(expected)
        out[f"q{qi}_triton_out"] = storage(triton_out)
    np.savez_compressed(HERE / f"{name}.npz", **out)
    print(f"{name}: {len(op_codes)} ops, {len(queries)} queries")


def config1_ops(plan):
    ops = [("alloc", f"r{r}", int(plan.context_lengths[r])) for r in range(plan.num_rows)]
    for item in workloads.write_schedule(plan):
        if item[0] == "write":
            _, r, depth, pos = item
            ops.append(("write", 0, f"r{r}", depth, pos))
        else:
            _, r, pos, e = item
            ops.append(("finalize", f"r{r}", pos, e))
    rows = [(f"r{r}", int(plan.query_depths[r]), int(plan.context_lengths[r]) - 1)
            for r in range(plan.num_rows)]
    return ops, [(0, rows)]


def make_config1(dtype):
    plan = workloads.config1_plan(0)
    ops, queries = config1_ops(plan)
    scenario(f"config1_{dtype}", layers=1, hkv=16, hq=16, d=128, num_blocks=1024, page=16,
             loops=4, dtype=dtype, layout="last_exited", ops=ops, queries=queries, seed=11,
             free_order=plan.free_order)


def make_mixed(dtype, d):
    """Mixed requests/depths over fragmented tables, GQA 6q/2kv
    (reference tests/test_attention.py:57-83)."""
    ops = [("alloc", "retained", 4), ("alloc", "hole", 8), ("alloc", "a", 7), ("free", "hole"),
           ("alloc", "b", 6)]
    for rid, length in [("a", 7), ("b", 6)]:
        for depth in range(3):
            for pos in range(length):
                ops.append(("write", 1, rid, depth, pos))

    def shift(k, v, rid, depth):
        return k + depth * 0.5, v + (4 if rid == "a" else -4)

    queries = [(1, [("a", 2, 6), ("b", 0, 4), ("a", 1, 2), ("b", 2, 5)])]
    scenario(f"mixed_{dtype}_d{d}", layers=2, hkv=2, hq=6, d=d, num_blocks=48, page=3, loops=3,
             dtype=dtype, layout="last_exited", ops=ops, queries=queries, seed=48,
             scale_values=shift)


def make_long(dtype):
    """Several online-softmax tiles and irregular page boundaries
    (reference tests/test_attention.py:90-106), GQA 2q/1kv, page 5."""
    ops = [("alloc", "long", 71)] + [("write", 0, "long", 1, p) for p in range(71)]

    def scale(k, v, rid, depth):
        return k * 8, v

    queries = [(0, [("long", 1, p) for p in [0, 31, 32, 70]])]
    scenario(f"long_{dtype}", layers=1, hkv=1, hq=2, d=32, num_blocks=30, page=5, loops=2,
             dtype=dtype, layout="last_exited", ops=ops, queries=queries, seed=89,
             scale_values=scale)


def make_shared(dtype):
    """SHARED layout: every depth overwrites plane 0 (docs/kv_layout_computation.md)."""
    ops = [("alloc", "x", 40), ("alloc", "y", 23)]
    for rid, length in [("x", 40), ("y", 23)]:
        for pos in range(length):
            for depth in range(3):
                ops.append(("write", 0, rid, depth, pos))
    queries = [(0, [("x", 2, 39), ("y", 1, 22), ("x", 0, 17), ("y", 2, 0)])]
    scenario(f"shared_{dtype}", layers=1, hkv=2, hq=4, d=64, num_blocks=8, page=16, loops=3,
             dtype=dtype, layout="shared", ops=ops, queries=queries, seed=5)


def make_prefill(dtype, d=64, spec=None, max_tokens=65, blocks=80, tag="", store_inputs=True):
    """Packed chunked prefill with prefixes at unequal depths crossing page
    boundaries (reference tests/test_flash_attention.py:146-189): the packed
    batch's metadata from _prepare_batch(packed_prefill=True) and the expected
    output from torch_paged_attention over the flat per-token tables."""
    from types import SimpleNamespace

    from vllm_rlt.core.kv_cache_manager import KVCacheManager
    from vllm_rlt.kernels.paged_attention import torch_paged_attention

    td = TORCH_DTYPES[dtype]
    cache = KVCacheManager(2, 2, d, blocks, 16, 4, "cpu", td, "torch")
    cache.attention = SimpleNamespace(generation=4)
    cache.key_cache.zero_()
    cache.value_cache.zero_()
    rng = np.random.default_rng([712, 2])
    for rid in ["hole", "a", "b", "c"]:
        cache.allocate(rid, max_tokens)
    cache.free("hole")
    ids, depths, positions = [], [], []
    spec = spec or [("a", 0, 0, 19), ("b", 2, 17, 7), ("c", 3, 31, 18)]
    for rid, depth, prefix, count in spec:
        for layer in range(2):
            if prefix:
                kv = values(rng, (prefix, 2, d), dtype)
                cache.write(layer, [rid] * prefix, [depth] * prefix, list(range(prefix)), kv, -kv)
        ids.extend([rid] * count)
        depths.extend([depth] * count)
        positions.extend(range(prefix, prefix + count))
    batch = cache._prepare_batch(ids, depths, positions, packed_prefill=True)
    flat = cache._prepare_batch(ids, depths, positions)
    out = {
        "spec": np.array([[["a", "b", "c"].index(r), d, p, c] for r, d, p, c in spec]),
        "dtype": np.array(dtype),
        "block_tables": batch.block_tables.numpy(),
        "context_lengths": batch.context_lengths.numpy(),
        "cu_seqlens_q": batch.cu_seqlens_q.numpy(),
        "max_seqlen_q": np.array(batch.max_seqlen_q),
        "write_blocks": batch.write_blocks.numpy(),
        "write_offsets": batch.write_offsets.numpy(),
        "position_ids": batch.position_ids.numpy(),
        "flat_block_tables": flat.block_tables.numpy(),
        "flat_context_lengths": flat.context_lengths.numpy(),
        "alloc_tables": np.array([list(cache._allocations[r].block_tables) for r in "abc"],
                                 dtype=np.int32),
    }
    for layer in range(2):
        k = values(rng, (len(ids), 2, d), dtype)
        v = values(rng, (len(ids), 2, d), dtype)
        q = values(rng, (len(ids), 4, d), dtype)
        cache._write_prepared(layer, batch, k, v)
        expected = torch_paged_attention(q, cache.key_cache[:, layer], cache.value_cache[:, layer],
                                         flat.block_tables, flat.context_lengths)
        if store_inputs:  # otherwise re-drawn from the seeded generator by the test
            out[f"k{layer}"] = storage(k)
            out[f"v{layer}"] = storage(v)
            out[f"q{layer}"] = storage(q)
        out[f"out{layer}"] = storage(expected)
    out["key_digest"] = np.array(digest(cache.key_cache))
    out["value_digest"] = np.array(digest(cache.value_cache))
    out["prefix_seed"] = np.array([712, 2])
    out["geometry"] = np.array([d, blocks, max_tokens])
    np.savez_compressed(HERE / f"prefill{tag}_{dtype}.npz", **out)
    print(f"prefill{tag}_{dtype}: {len(ids)} tokens")


def make_routing():
    """Reference Triton routing kernels run by the CPU interpreter."""
    from vllm_rlt.kernels.prefill_metadata import expand_prefill, stage_prefill
    from vllm_rlt.kernels.routing import (finalize_kernel, gather_kernel, metadata_kernel,
                                          scatter_kernel)

    rng = np.random.default_rng(2024)
    out = {}
    # metadata_kernel: resident tables [slots, planes, width]
    for planes in (4, 1):
        slots, width, page, size, n, out_width = 6, 64, 16, 9, 6, 40
        tables = torch.from_numpy(rng.integers(0, 5000, size=(slots, planes, width)).astype(np.int32))
        desc = torch.from_numpy(np.stack([
            rng.integers(0, slots, size=size),
            rng.integers(0, planes, size=size),
            rng.integers(0, out_width * page, size=size),
        ], axis=1).astype(np.int64))
        sentinel = dict(
            slots=torch.full((size,), -7, dtype=torch.int64),
            positions=torch.full((size,), -7, dtype=torch.int64),
            lengths=torch.full((size,), -7, dtype=torch.int32),
            blocks=torch.full((size,), -7, dtype=torch.int64),
            offsets=torch.full((size,), -7, dtype=torch.int64),
            out_tables=torch.full((size, width), -7, dtype=torch.int32),
        )
        res = {k: v.clone() for k, v in sentinel.items()}
        metadata_kernel[(size,)](desc, tables, res["slots"], res["positions"], res["lengths"],
                                 res["blocks"], res["offsets"], res["out_tables"], n, size, width,
                                 page, planes, out_width, 256)
        tag = f"meta_p{planes}"
        out[f"{tag}_tables"] = tables.numpy()
        out[f"{tag}_desc"] = desc.numpy()
        out[f"{tag}_dims"] = np.array([slots, planes, width, page, size, n, out_width])
        for k, v in res.items():
            out[f"{tag}_{k}"] = v.numpy()
    # finalize_kernel on a small 5-D pool [blocks, layers, page, hkv, d]
    blocks, layers, page, hkv, d, planes, width, slots = 64, 3, 4, 2, 8, 4, 5, 3
    key = torch.from_numpy(rng.standard_normal((blocks, layers, page, hkv, d), dtype=np.float32))
    value = torch.from_numpy(rng.standard_normal((blocks, layers, page, hkv, d), dtype=np.float32))
    perm = rng.permutation(blocks)[: slots * planes * width]
    tables = torch.from_numpy(perm.reshape(slots, planes, width).astype(np.int32))
    desc = torch.tensor([[0, 0, 5], [1, 2, 19], [2, 1, 0], [0, 3, 7]], dtype=torch.int64)
    out["fin_key_before"] = key.numpy().copy()
    out["fin_value_before"] = value.numpy().copy()
    out["fin_tables"] = tables.numpy()
    out["fin_desc"] = desc.numpy()
    channels = hkv * d
    finalize_kernel[(len(desc), planes, -(-layers * channels // 256))](
        desc, tables, key, value, width, planes, page, layers, channels, *key.stride()[:3], 256)
    out["fin_key_after"] = key.numpy()
    out["fin_value_after"] = value.numpy()
    out["fin_dims"] = np.array([blocks, layers, page, hkv, d, planes, width, slots])
    # stage_prefill / expand_prefill
    source = torch.from_numpy(np.concatenate([
        rng.integers(-5, 2**40, size=37), np.array([2**33 + 5, -(2**31) - 3])]).astype(np.int64))
    target = torch.zeros_like(source)
    target32 = torch.zeros(len(source), dtype=torch.int32)
    stage_prefill[(1,)](source, target, target32, len(source), 256)
    out["stage_source"] = source.numpy()
    out["stage_target"] = target.numpy()
    out["stage_target32"] = target32.numpy()
    n, width, page, seqs = 50, 7, 16, 4
    positions = torch.from_numpy(rng.integers(0, width * page, size=n).astype(np.int64))
    sequences = torch.from_numpy(rng.integers(0, seqs, size=n).astype(np.int64))
    ptables = torch.from_numpy(rng.integers(0, 900, size=seqs * width).astype(np.int32))
    eblocks = torch.full((n,), -7, dtype=torch.int64)
    eoffsets = torch.full((n,), -7, dtype=torch.int64)
    expand_prefill[(1,)](positions, sequences, ptables, eblocks, eoffsets, n, width, page, 256)
    out["expand_positions"] = positions.numpy()
    out["expand_sequences"] = sequences.numpy()
    out["expand_tables"] = ptables.numpy()
    out["expand_dims"] = np.array([n, width, page])
    out["expand_blocks"] = eblocks.numpy()
    out["expand_offsets"] = eoffsets.numpy()
    # gather / scatter of a bf16 hidden pool and an int64 token pool
    pool = torch.from_numpy(rng.standard_normal((10, 300), dtype=np.float32)).to(torch.bfloat16)
    slots_t = torch.tensor([7, 2, 9, 0, 3, 3, 3, 3], dtype=torch.int64)
    gathered = torch.full((8, 300), 5.0, dtype=torch.bfloat16)
    gather_kernel[(8, 2)](pool, slots_t, gathered, 5, 300, pool.stride(0), gathered.stride(0), 256)
    out["gather_pool"] = storage(pool)
    out["gather_slots"] = slots_t.numpy()
    out["gather_out"] = storage(gathered)
    tokens = torch.from_numpy(rng.integers(0, 49152, size=(10, 1)).astype(np.int64))
    upd = torch.from_numpy(rng.integers(0, 49152, size=(4, 1)).astype(np.int64))
    slots_s = torch.tensor([4, 1, 8, 6], dtype=torch.int64)
    out["scatter_before"] = tokens.numpy().copy()
    scatter_kernel[(4, 1)](upd, slots_s, tokens, 1, upd.stride(0), tokens.stride(0), 256)
    out["scatter_values"] = upd.numpy()
    out["scatter_slots"] = slots_s.numpy()
    out["scatter_after"] = tokens.numpy()
    np.savez_compressed(HERE / "routing.npz", **out)
    print("routing: metadata, finalize, stage/expand, gather/scatter")


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path of the vllm-rlt source tree")
    args = parser.parse_args()
    sys.path.insert(0, str(Path(args.reference).resolve()))
    torch.manual_seed(0)
    torch.set_num_threads(8)
    for dtype in ("f32", "bf16"):
        make_config1(dtype)
    for dtype in ("f32", "f16", "bf16"):
        for d in (7, 32, 64, 128):
            make_mixed(dtype, d)
        make_long(dtype)
        make_shared(dtype)
        make_prefill(dtype)
    for dtype in ("f16", "bf16"):
        # head_dim 128, chunks crossing 128-query tiles, prefixes crossing pages
        make_prefill(dtype, d=128, spec=[("a", 0, 0, 150), ("b", 2, 17, 7), ("c", 3, 131, 260)],
                     max_tokens=400, blocks=400, tag="128", store_inputs=False)
    make_routing()


if __name__ == "__main__":
    main()
