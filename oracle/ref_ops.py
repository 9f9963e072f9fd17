"""numpy restatement of the reference's paged-KV attention path (test oracle).

Every function cites the reference file:line it restates (paths relative to
the vllm-rlt project root). Arrays use storage form: float32, float16, or
uint16 holding bfloat16 bits (numpy has no bfloat16); the ``dtype`` argument
names which ("f32", "f16", "bf16").
"""

from __future__ import annotations

import math

import numpy as np

DTYPES = ("f32", "f16", "bf16")


# ---------------------------------------------------------------- dtype helpers


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bfloat16 bits -> float32 (exact: bf16 is the top half of an fp32)."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 bits, round to nearest even (torch's .to(bfloat16))."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = (u + (((u >> 16) & 1) + 0x7FFF)) >> 16
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    out = rounded.astype(np.uint16)
    out[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)  # quiet NaN, sign kept
    return out


def to_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return bf16_to_f32(x)
    return np.asarray(x).astype(np.float32)


def from_f32(x: np.ndarray, dtype: str) -> np.ndarray:
    if dtype == "bf16":
        return f32_to_bf16(x)
    if dtype == "f16":
        return np.asarray(x, dtype=np.float32).astype(np.float16)
    return np.asarray(x, dtype=np.float32)


def storage_dtype(dtype: str):
    return {"f32": np.float32, "f16": np.float16, "bf16": np.uint16}[dtype]


# ------------------------------------------------------------------ attention


def paged_attention(q, key_cache, value_cache, block_tables, context_lengths, dtype):
    """vllm_rlt/kernels/paged_attention.py:12-36 (torch_paged_attention).

    q [N, Hq, D]; key_cache/value_cache are layer views [blocks, page, Hkv, D]
    (any strides); block_tables int [N, W]; context_lengths int [N]. Per row:
    gather positions 0..len-1 through the table (block = table[pos // page],
    offset = pos % page), repeat KV heads for GQA, fp32 scores scaled by
    1/sqrt(D), softmax, weighted sum of V, cast to the input dtype; len 0
    gives zeros (:25-27).
    """
    n, hq, d = q.shape
    page, hkv = key_cache.shape[1], key_cache.shape[2]
    groups = hq // hkv
    scale = np.float32(1.0 / math.sqrt(d))
    out = np.zeros(q.shape, dtype=storage_dtype(dtype))
    tables = np.asarray(block_tables)
    lengths = np.asarray(context_lengths).tolist()
    for row, length in enumerate(lengths):
        if length == 0:
            continue
        positions = np.arange(length)
        blocks = tables[row, positions // page].astype(np.int64)
        offsets = positions % page
        keys = to_f32(key_cache[blocks, offsets], dtype)  # [L, Hkv, D]
        values = to_f32(value_cache[blocks, offsets], dtype)
        if groups > 1:
            keys = np.repeat(keys, groups, axis=1)
            values = np.repeat(values, groups, axis=1)
        query = to_f32(q[row], dtype)  # [Hq, D]
        # scores[h, t] = q[h] . k[t, h]  (batched over heads)
        scores = np.matmul(keys.transpose(1, 0, 2), query[:, :, None])[:, :, 0] * scale
        scores = scores - scores.max(axis=1, keepdims=True)
        weights = np.exp(scores, dtype=np.float32)
        weights /= weights.sum(axis=1, keepdims=True)
        result = np.matmul(weights[:, None, :], values.transpose(1, 0, 2))[:, 0, :]
        out[row] = from_f32(result, dtype)
    return out


def paged_prefill(q, key_cache, value_cache, block_tables, context_lengths, cu_seqlens_q, dtype):
    """Packed chunked prefill with bottom-right causal alignment.

    vllm_rlt/kernels/flash_attention.py:66-96 (FlashPagedAttention.prefill):
    sequence s owns queries cu[s]..cu[s+1]-1 and keys 0..len_s-1 through table
    s; query i of the chunk (0-based) sees keys up to len_s - qlen_s + i
    (prefix_length = seqlen_k - seqlen_q). The reference's own test checks it
    against per-token decode rows (tests/test_flash_attention.py:169-186),
    which is how this restatement computes it.
    """
    cu = np.asarray(cu_seqlens_q).astype(np.int64)
    lengths = np.asarray(context_lengths).astype(np.int64)
    tables = np.asarray(block_tables)
    n_tok = q.shape[0]
    row_tables = np.zeros((n_tok, tables.shape[1]), dtype=tables.dtype)
    row_lengths = np.zeros(n_tok, dtype=np.int64)
    for s in range(len(cu) - 1):
        qlen = cu[s + 1] - cu[s]
        for i in range(qlen):
            row_tables[cu[s] + i] = tables[s]
            row_lengths[cu[s] + i] = max(0, lengths[s] - qlen + i + 1)
    return paged_attention(q, key_cache, value_cache, row_tables, row_lengths, dtype)


# ------------------------------------------------------------ cache metadata


def prepare_rows(block_tables_by_plane, planes, depths, positions, page, layout, packed=False):
    """Depth/page resolution of vllm_rlt/core/kv_cache_manager.py:398-478.

    block_tables_by_plane[r][plane] is row r's allocation table for that
    plane (its request's ``block_tables``). plane = depth for LAST-EXITED,
    0 for SHARED (:350-351). Returns write blocks/offsets, per-row (or, when
    packed, per-sequence) tables padded with -1 to width = max(pos//page + 1),
    context lengths = pos + 1, and cu_seqlens_q when packed (:424-444).
    ``planes`` is accepted for symmetry with the reference's storage depths.
    """
    del planes
    plane_of = (lambda depth: depth) if layout == "last_exited" else (lambda depth: 0)
    rows = list(zip(block_tables_by_plane, depths, positions))
    blocks = [t[plane_of(d)][p // page] for t, d, p in rows]
    offsets = [p % page for _, _, p in rows]
    width = max((p // page + 1 for _, _, p in rows), default=0)
    table_rows, cumulative = rows, None
    if packed:
        ends, cumulative = [], [0]
        for index, (tables, depth, position) in enumerate(rows):
            key = (id(tables), depth)
            prev = rows[index - 1] if index else None
            if index and key == (id(prev[0]), prev[1]):
                if position != prev[2] + 1:
                    raise ValueError("packed prefill positions must be contiguous")
                ends[-1] = (tables, depth, position)
                cumulative[-1] = index + 1
            else:
                ends.append((tables, depth, position))
                cumulative.append(index + 1)
        table_rows = ends
    tables_out = np.full((len(table_rows), width), -1, dtype=np.int32)
    for i, (tables, depth, _) in enumerate(table_rows):
        t = list(tables[plane_of(depth)][:width])
        tables_out[i, : len(t)] = t
    return dict(
        write_blocks=np.asarray(blocks, dtype=np.int64),
        write_offsets=np.asarray(offsets, dtype=np.int64),
        block_tables=tables_out,
        context_lengths=np.asarray([p + 1 for _, _, p in table_rows], dtype=np.int32),
        position_ids=np.asarray([p for _, _, p in rows], dtype=np.int64),
        cu_seqlens_q=None if cumulative is None else np.asarray(cumulative, dtype=np.int32),
    )


def kv_write(key_cache, value_cache, layer, write_blocks, write_offsets, k, v):
    """vllm_rlt/core/kv_cache_manager.py:531-532 (and the graph copy at
    vllm_rlt/worker/cuda_graph.py:16-19), in place on the 5-D pools:
    key_cache[write_blocks, layer, write_offsets] = k[:n]."""
    blocks = np.asarray(write_blocks, dtype=np.int64)
    offsets = np.asarray(write_offsets, dtype=np.int64)
    n = len(blocks)
    key_cache[blocks, layer, offsets] = k[:n]
    value_cache[blocks, layer, offsets] = v[:n]


def finalize_token(key_cache, value_cache, plane_tables, position, exit_depth, max_loops, page):
    """vllm_rlt/core/kv_cache_manager.py:601-611 (LAST-EXITED eager exit copy):
    copy the exit plane's page row (all layers) into each deeper plane.
    plane_tables[plane] is the request's table for that plane."""
    logical, offset = divmod(position, page)
    source = plane_tables[exit_depth][logical]
    for depth in range(exit_depth + 1, max_loops):
        destination = plane_tables[depth][logical]
        key_cache[destination, :, offset] = key_cache[source, :, offset]
        value_cache[destination, :, offset] = value_cache[source, :, offset]


def finalize(descriptor, tables, key_cache, value_cache, planes, page):
    """vllm_rlt/kernels/routing.py:79-109 (finalize_kernel): descriptor rows
    (slot, depth, pos); tables [slots, planes, width]; for every target plane
    in (depth, planes) copy the token's K/V of all layers from plane depth."""
    desc = np.asarray(descriptor, dtype=np.int64).reshape(-1, 3)
    tables = np.asarray(tables)
    for slot, depth, pos in desc.tolist():
        source = int(tables[slot, depth, pos // page])
        for target in range(depth + 1, planes):
            dest = int(tables[slot, target, pos // page])
            key_cache[dest, :, pos % page] = key_cache[source, :, pos % page]
            value_cache[dest, :, pos % page] = value_cache[source, :, pos % page]


def metadata(descriptor, tables, outputs, n, size, width, page, planes, out_width):
    """vllm_rlt/kernels/routing.py:7-41 (metadata_kernel), grid = size rows.

    ``outputs`` holds the prior contents of slots, positions, lengths, blocks,
    offsets, out_tables (the kernel leaves blocks/offsets of padding rows
    untouched); returns updated copies. tables is [slots, planes, width].
    """
    desc = np.asarray(descriptor, dtype=np.int64).reshape(-1, 3)
    flat = np.asarray(tables).reshape(-1)
    res = {key: np.array(value, copy=True) for key, value in outputs.items()}
    for row in range(size):
        valid = row < n
        slot, depth, pos = (int(x) for x in desc[row]) if valid else (0, 0, 0)
        plane = depth if planes > 1 else 0
        base = (slot * planes + plane) * width
        res["slots"][row] = slot
        res["positions"][row] = pos
        res["lengths"][row] = pos + 1 if valid else 0
        if valid:
            res["blocks"][row] = flat[base + pos // page]
            res["offsets"][row] = pos % page
        res["out_tables"].reshape(-1)[row * width : row * width + out_width] = (
            flat[base : base + out_width] if valid else 0
        )
    return res


def stage_prefill(source):
    """vllm_rlt/kernels/prefill_metadata.py:7-12: int64 copy and int32 copy
    (two's-complement truncation, like Triton's store of int64 into int32)."""
    src = np.asarray(source, dtype=np.int64)
    return src.copy(), src.astype(np.int32)


def expand_prefill(positions, sequences, tables_flat, width, page):
    """vllm_rlt/kernels/prefill_metadata.py:15-32:
    block = tables[seq * width + pos // page], offset = pos % page."""
    pos = np.asarray(positions, dtype=np.int64)
    seq = np.asarray(sequences, dtype=np.int64)
    flat = np.asarray(tables_flat).reshape(-1)
    blocks = flat[seq * width + pos // page].astype(np.int64)
    return blocks, pos % page


def gather(pool, slots, n, size):
    """vllm_rlt/kernels/routing.py:44-59: out[row] = pool[slots[row]] for
    row < n, zeros for n <= row < size."""
    pool = np.asarray(pool)
    out = np.zeros((size,) + pool.shape[1:], dtype=pool.dtype)
    idx = np.asarray(slots, dtype=np.int64)[:n]
    out[:n] = pool[idx]
    return out


def scatter(values, slots, pool, n):
    """vllm_rlt/kernels/routing.py:62-76: pool[slots[row]] = values[row], row < n."""
    pool = np.array(pool, copy=True)
    idx = np.asarray(slots, dtype=np.int64)[:n]
    pool[idx] = np.asarray(values)[:n]
    return pool
