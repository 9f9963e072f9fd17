"""Decode attention that reads prefix-shared KV pages once per group of rows.

Prefix caching in the reference (vllm_rlt/core/kv_cache_manager.py:211-251)
publishes complete prompt pages by content hash and hands the same physical
pages to later requests (``_refs[b] += 1``), so rows of a decode batch can
start their block tables with identical page ids. The plain decode kernel,
like the reference's, reads such pages once per row. Here:

* ``find_shared_prefixes`` groups rows by identical leading page ids (the
  longest common run of full pages, capped by the shortest member context);
* ``plan_shared_prefix`` turns each group's shared prefix into chunks -- a
  token range of the group's first table row plus the member rows that attend
  to it -- with one partial slot per (member, chunk), rows' slots contiguous;
  the chunk length defaults to ``choose_chunk_tokens`` (the smallest whose
  chunk CTAs fit one resident wave of the chunk kernel);
  and gives every row a suffix table (its own table shifted past its shared
  pages) and suffix length for the tokens only it reads;
* ``paged_attention_shared`` derives each row's suffix table and length on
  the device from the call's own tables and lengths
  (``rlt_shared_prefix_suffix``), runs the prefix chunks on a side stream
  (each chunk's K/V read once and attended by all its members) beside the
  plain decode kernel on the suffix tables (``rlt_paged_decode_lse``: the
  suffix result lands in the output, its log-sum-exp beside it), and merges
  the chunk partials into the output after both.

The result equals ``paged_attention`` on the same tables and lengths (fp32
online softmax in a different order: within fp32 rounding). The plan is built
on the host from host copies of the tables and lengths, once per batch
layout; it stays valid while the rows grow, so a captured CUDA graph can
replay the call step after step. Rebuild it when the batch's rows change.
"""

from __future__ import annotations

from collections import defaultdict
from dataclasses import dataclass, field

import numpy as np
import torch

from .. import _lib
from .paged_attention import _as_int32, _validate

MAX_PAIRS = 32  # (member row, query head) pairs per chunk CTA


def find_shared_prefixes(tables: np.ndarray, lengths: np.ndarray, page: int, min_rows: int = 2):
    """[(rows, shared_pages)] for groups of >= min_rows rows whose tables begin
    with the same physical pages. shared_pages is the longest common run of
    page ids over the group, counted in pages that lie fully inside every
    member's context."""
    tables = np.asarray(tables)
    lengths = np.asarray(lengths, dtype=np.int64)
    full = lengths // page
    by_first = defaultdict(list)
    for row in range(tables.shape[0]):
        if full[row] >= 1 and tables[row, 0] >= 0:
            by_first[int(tables[row, 0])].append(row)
    groups = []
    for rows in by_first.values():
        if len(rows) < min_rows:
            continue
        idx = np.asarray(rows)
        limit = int(min(full[idx].min(), tables.shape[1]))
        same = (tables[idx, :limit] == tables[idx[0], :limit]).all(axis=0)
        shared = limit if same.all() else int(np.argmin(same))
        if shared >= 1:
            groups.append((rows, shared))
    return groups


@dataclass
class SharedPrefixPlan:
    chunks: torch.Tensor        # int32 [C, 5]: table row, token begin, token end, member begin, count
    members: torch.Tensor       # int32 [M]: member row ids
    member_slots: torch.Tensor  # int32 [M]: partial slot of (member, chunk)
    row_slots: torch.Tensor     # int32 [N + 1]: row r owns slots row_slots[r]..row_slots[r+1]
    suffix_tables: torch.Tensor   # int32 [N, W]: row's table after its shared pages (-1 padded)
    suffix_lengths: torch.Tensor  # int32 [N]: tokens after the shared prefix
    prefix_pages: torch.Tensor    # int32 [N]: the row's shared leading pages (0: none)
    lengths: torch.Tensor         # int32 [N]: the context lengths the plan was built from
    num_rows: int
    num_chunks: int
    num_slots: int
    groups: list = field(default_factory=list)
    logical_tokens: int = 0     # sum of context lengths (token rows a per-row decode reads)
    read_tokens: int = 0        # token rows this plan reads (per KV head)
    chunk_tokens: int = 0       # longest token range of one chunk


def plan_arrays(tables, lengths, page: int, group: int, chunk_tokens: int = 256, min_rows: int = 2,
                groups=None):
    """Host plan as numpy arrays: (chunks [C,5], members, member_slots,
    row_slots, suffix_tables, suffix_lengths, groups, logical_tokens,
    read_tokens). ``group`` = query heads per KV head (GQA). The chunks cover
    the shared prefixes; row r's tokens [prefix_r, ctx_r) are read through
    suffix_tables[r] (tokens renumbered from 0). ``groups``: the rows'
    ``find_shared_prefixes`` result when the caller already has it."""
    tables = np.asarray(tables)
    lengths = np.asarray(lengths, dtype=np.int64)
    rows = tables.shape[0]
    if group < 1 or group > MAX_PAIRS:
        raise ValueError(f"query heads per KV head must be in [1, {MAX_PAIRS}]")
    max_members = MAX_PAIRS // group
    if groups is None:
        groups = find_shared_prefixes(tables, lengths, page, min_rows)
    prefix = np.zeros(rows, dtype=np.int64)
    items = []  # (table row, begin, end, member rows)
    for members, shared in groups:
        tokens = shared * page
        prefix[members] = tokens
        for start in range(0, len(members), max_members):
            items.append((members[0], 0, tokens, members[start:start + max_members]))
    suffix_tables = np.full(tables.shape, -1, dtype=np.int32)
    for row in range(rows):
        skip = int(prefix[row]) // page
        suffix_tables[row, : tables.shape[1] - skip] = tables[row, skip:]
    suffix_lengths = np.clip(lengths - prefix, 0, None).astype(np.int32)
    chunk_list = []
    for table_row, begin, end, members in items:
        for b in range(begin, end, chunk_tokens):
            chunk_list.append((table_row, b, min(b + chunk_tokens, end), members))
    counts = np.zeros(rows, dtype=np.int64)
    for _, _, _, members in chunk_list:
        counts[members] += 1
    row_slots = np.zeros(rows + 1, dtype=np.int64)
    np.cumsum(counts, out=row_slots[1:])
    cursor = row_slots[:-1].copy()
    chunks = np.zeros((len(chunk_list), 5), dtype=np.int32)
    member_rows, member_slots = [], []
    read_tokens = 0
    for c, (table_row, b, e, members) in enumerate(chunk_list):
        chunks[c] = (table_row, b, e, len(member_rows), len(members))
        for m in members:
            member_rows.append(m)
            member_slots.append(cursor[m])
            cursor[m] += 1
        read_tokens += e - b
    read_tokens += int(suffix_lengths.sum())
    return (chunks, np.asarray(member_rows, dtype=np.int32), np.asarray(member_slots, dtype=np.int32),
            row_slots.astype(np.int32), suffix_tables, suffix_lengths, groups,
            int(lengths.clip(min=0).sum()), int(read_tokens))


# Chunk CTAs one SM holds at once (the chunk kernel's launch bounds).
CHUNK_CTAS_PER_SM = 2


def choose_chunk_tokens(groups, page: int, group: int, num_kv_heads: int, num_sms: int,
                        smallest: int = 512) -> int:
    """The smallest chunk length (``smallest`` doubled until it fits) whose
    (chunk, KV head) CTAs fit in one resident wave of the chunk kernel.

    The chunk kernel runs beside the suffix decode, and one resident wave of
    long chunks leaves the decode the SMs' remaining slots for the whole call:
    on the prefix-cached configs[1] batch (16 groups of 16 rows, 1-4K shared
    tokens) the overlapped call took 287 us with 512-token chunks, 265 us with
    2048 and 261 us with 4096 (one wave), while the chunk kernel alone is
    fastest with many short chunks."""
    max_members = MAX_PAIRS // group
    work = [(int(shared) * page, -(-len(members) // max_members)) for members, shared in groups]
    slots = CHUNK_CTAS_PER_SM * max(1, int(num_sms))
    chunk = smallest
    longest = max((tokens for tokens, _ in work), default=smallest)
    while chunk < longest:
        ctas = sum(-(-tokens // chunk) * blocks for tokens, blocks in work) * num_kv_heads
        if ctas <= slots:
            break
        chunk *= 2
    return chunk


def _num_sms(device) -> int:
    device = torch.device(device)
    if device.type == "cuda" and torch.cuda.is_available():
        return torch.cuda.get_device_properties(device).multi_processor_count
    return 148  # B200


def plan_shared_prefix(block_tables, context_lengths, page_size: int, num_q_heads: int,
                       num_kv_heads: int, device, chunk_tokens: int | None = None) -> SharedPrefixPlan:
    """Build the plan on the host (tables/lengths may be tensors on any
    device or numpy arrays) and upload it to ``device``. ``chunk_tokens``
    None picks the chunk length with ``choose_chunk_tokens``."""
    tables = block_tables.cpu().numpy() if torch.is_tensor(block_tables) else np.asarray(block_tables)
    lengths = (context_lengths.cpu().numpy() if torch.is_tensor(context_lengths)
               else np.asarray(context_lengths))
    if num_q_heads % num_kv_heads:
        raise ValueError("query heads must be a positive multiple of KV heads")
    groups = find_shared_prefixes(tables, np.asarray(lengths, dtype=np.int64), page_size)
    if chunk_tokens is None:
        chunk_tokens = choose_chunk_tokens(groups, page_size, num_q_heads // num_kv_heads,
                                           num_kv_heads, _num_sms(device))
    (chunks, members, slots, row_slots, suffix_tables, suffix_lengths, groups, logical,
     read) = plan_arrays(tables, lengths, page_size, num_q_heads // num_kv_heads, chunk_tokens,
                         groups=groups)

    def up(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(device)

    clipped = np.clip(np.asarray(lengths, dtype=np.int64), 0, None)
    prefix_pages = ((clipped - suffix_lengths) // page_size).astype(np.int32)
    return SharedPrefixPlan(
        chunks=up(chunks if len(chunks) else np.zeros((0, 5), np.int32)),
        members=up(members), member_slots=up(slots), row_slots=up(row_slots),
        suffix_tables=up(suffix_tables), suffix_lengths=up(suffix_lengths),
        prefix_pages=up(prefix_pages), lengths=up(clipped.astype(np.int32)),
        num_rows=int(tables.shape[0]), num_chunks=int(len(chunks)), num_slots=int(row_slots[-1]),
        groups=groups, logical_tokens=logical, read_tokens=read, chunk_tokens=int(chunk_tokens))


_SIDE_STREAMS = {}


def _side_stream(device):
    index = device.index if device.index is not None else torch.cuda.current_device()
    stream = _SIDE_STREAMS.get(index)
    if stream is None:
        stream = torch.cuda.Stream(device=torch.device("cuda", index))
        _SIDE_STREAMS[index] = stream
    return stream


def paged_attention_shared(q, key_cache, value_cache, block_tables, plan: SharedPrefixPlan,
                           *, context_lengths=None, out=None):
    """Decode attention over the plan; same inputs and result as
    ``paged_attention``.

    The plan's groups and chunks stay valid while its rows grow: each call
    derives the rows' suffix tables and lengths on the device from the call's
    own ``block_tables`` and ``context_lengths`` (the plan's lengths when
    none are given), so a captured CUDA graph can replay the call step after
    step. Rebuild the plan when the batch's rows change. The prefix chunks
    run on a second stream while the plain decode kernel computes the
    suffixes; the merge joins them on the caller's stream."""
    lengths = _as_int32(context_lengths) if context_lengths is not None else plan.lengths
    _validate(q, key_cache, value_cache, block_tables, lengths)
    if q.shape[-1] not in (64, 128):
        raise ValueError("the shared-prefix decode supports head_dim 64 or 128")
    if plan.num_rows != q.shape[0]:
        raise ValueError("the plan was built for a different number of rows")
    if q.stride(-1) != 1:
        q = q.contiguous()
    output = torch.empty_like(q) if out is None else out
    rows, hq, d = q.shape
    if rows == 0:
        return output
    lib = _lib.load()
    device = q.device
    page, hkv = key_cache.shape[1], key_cache.shape[2]
    status = _lib.status_word(device).data_ptr()
    stream = _lib.stream_of(device)
    scale = d ** -0.5
    tables = _as_int32(block_tables)
    width = tables.shape[1]
    # 0. this call's suffix tables and lengths
    suffix = torch.empty((rows, width), dtype=torch.int32, device=device)
    suffix_lengths = torch.empty(rows, dtype=torch.int32, device=device)
    code = lib.rlt_shared_prefix_suffix(
        tables.data_ptr(), lengths.data_ptr(), plan.prefix_pages.data_ptr(), suffix.data_ptr(),
        suffix_lengths.data_ptr(), status, rows, width, page, tables.stride(0), stream)
    _lib.check(code, "shared-prefix suffix metadata")
    dtype_code = _lib.DTYPE_CODES[q.dtype]

    def shared(phases, launch_stream, workspace, lse):
        return lib.rlt_paged_decode_shared_phases(
            q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), tables.data_ptr(),
            plan.chunks.data_ptr(), plan.members.data_ptr(), plan.member_slots.data_ptr(),
            plan.row_slots.data_ptr(), _lib.ptr(lse), output.data_ptr(), workspace.data_ptr(),
            workspace.numel(), status, dtype_code,
            rows, hq, hkv, d, page, width, key_cache.shape[0],
            plan.num_chunks, plan.num_slots, plan.members.numel(),
            q.stride(0), q.stride(1),
            key_cache.stride(0), key_cache.stride(1), key_cache.stride(2),
            value_cache.stride(0), value_cache.stride(1), value_cache.stride(2),
            tables.stride(0), output.stride(0), output.stride(1), scale, phases, launch_stream)

    # 1. the shared prefixes, read once per group, on the side stream
    need = lib.rlt_paged_decode_shared_workspace_bytes(plan.num_slots, hq, d)
    workspace = torch.empty(max(need, 16), dtype=torch.uint8, device=device)
    overlap = plan.num_chunks > 0
    if overlap:
        current = torch.cuda.current_stream(device)
        side = _side_stream(device)
        fork = torch.cuda.Event()
        fork.record(current)
        side.wait_event(fork)
        _lib.check(shared(1, side.cuda_stream, workspace, None),
                   "shared-prefix paged decode attention (prefix chunks)")
        workspace.record_stream(side)
    # 2. each row's own tokens after its shared prefix: the plain decode kernel
    lse = torch.empty((rows, hq), dtype=torch.float32, device=device)
    need = lib.rlt_paged_decode_workspace_bytes(rows, hq, d, page, width)
    decode_ws = torch.empty(need, dtype=torch.uint8, device=device) if need else None
    code = lib.rlt_paged_decode_lse(
        q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), suffix.data_ptr(),
        suffix_lengths.data_ptr(), output.data_ptr(), _lib.ptr(decode_ws), need, status,
        dtype_code, rows, hq, hkv, d, page, width, key_cache.shape[0],
        q.stride(0), q.stride(1),
        key_cache.stride(0), key_cache.stride(1), key_cache.stride(2),
        value_cache.stride(0), value_cache.stride(1), value_cache.stride(2),
        suffix.stride(0), output.stride(0), output.stride(1), scale, lse.data_ptr(), stream,
    )
    _lib.check(code, "shared-prefix paged decode attention (suffixes)")
    # 3. the merge, once both are done
    if overlap:
        join = torch.cuda.Event()
        join.record(side)
        current.wait_event(join)
        _lib.check(shared(2, stream, workspace, lse), "shared-prefix paged decode attention (merge)")
    return output
