"""Seeded synthetic workloads for the paged decode path.

Shapes and value distributions follow the benchmark configurations of the
reference's hot path (Ouro-1.4B geometry: 16 query heads = 16 KV heads,
head_dim 128, page 16, LAST-EXITED with 4 depth planes). No dataset is
involved: every input is drawn from numpy's PCG64 generator with a fixed seed
so a test, the bench and the golden-vector script draw identical inputs.

Page tables are handed out the way the reference allocator does
(vllm_rlt/core/kv_cache_manager.py:253-293 with ``_claim`` at :182-192): a
request of ``max_tokens`` takes ceil(max_tokens/page) pages per plane from
the free list in one claim, plane d getting the d-th run of that claim. The
free list is a seeded permutation of the pool, so tables are fragmented.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np


@dataclass
class DecodePlan:
    """One batch of decode rows over a LAST-EXITED (or SHARED) page pool."""

    num_rows: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    page: int
    planes: int
    num_blocks: int
    context_lengths: np.ndarray  # int32 [rows], = position + 1
    query_depths: np.ndarray  # int64 [rows], 0-based depth (= plane for LAST-EXITED)
    exit_depths: list = field(default_factory=list)  # per row: 0-based exit depth per past position
    plane_tables: list = field(default_factory=list)  # per row: list of per-plane page lists
    layout: str = "last_exited"
    free_order: np.ndarray | None = None  # the pool's page hand-out order

    def plane_of(self, depth: int) -> int:
        return depth if self.layout == "last_exited" else 0

    @property
    def width(self) -> int:
        return max((math.ceil(int(c) / self.page) for c in self.context_lengths), default=0)

    def block_tables(self, width: int | None = None, pad: int = -1) -> np.ndarray:
        """Per-row table of the row's query plane, padded to ``width``
        (vllm_rlt/core/kv_cache_manager.py:445-448)."""
        width = self.width if width is None else width
        out = np.full((self.num_rows, width), pad, dtype=np.int32)
        for r in range(self.num_rows):
            table = self.plane_tables[r][self.plane_of(int(self.query_depths[r]))]
            used = math.ceil(int(self.context_lengths[r]) / self.page)
            out[r, :used] = table[:used]
        return out

    def kv_bytes(self, elem_bytes: int) -> int:
        return int(self.context_lengths.astype(np.int64).sum()) * self.num_kv_heads * self.head_dim * 2 * elem_bytes


def allocate_tables(lengths, planes: int, page: int, free_order: np.ndarray):
    """Reference allocation order: request r claims ceil(len_r/page)*planes
    pages from the front of ``free_order``; plane d gets run d."""
    cursor = 0
    tables = []
    for length in lengths:
        pages = math.ceil(int(length) / page)
        claim = free_order[cursor : cursor + pages * planes]
        if len(claim) < pages * planes:
            raise ValueError("page pool too small for the requested contexts")
        cursor += pages * planes
        tables.append([claim[d * pages : (d + 1) * pages].tolist() for d in range(planes)])
    return tables


def config1_plan(seed: int = 0) -> DecodePlan:
    """CPU-plumbing configuration: 8 rows, 16x128 heads, page 16, context
    lengths uniform in [1, 512], query depth and every past position's exit
    depth uniform in {1..4}, LAST-EXITED with 4 planes. 256 pages per plane
    (a 1024-page pool, one seeded permutation) -- 256 pages in total cannot
    hold 4 planes of these contexts."""
    rng = np.random.default_rng(seed)
    rows, planes, page = 8, 4, 16
    lengths = rng.integers(1, 513, size=rows).astype(np.int32)
    depths = rng.integers(1, 5, size=rows).astype(np.int64) - 1
    exits = [rng.integers(1, 5, size=int(c) - 1).astype(np.int64) - 1 for c in lengths]
    free_order = rng.permutation(1024)
    tables = allocate_tables(lengths, planes, page, free_order)
    return DecodePlan(rows, 16, 16, 128, page, planes, 1024, lengths, depths, exits, tables,
                      free_order=free_order)


def config2_plan(seed: int = 0, rows: int = 256, sigma: float = 0.6) -> DecodePlan:
    """Decode microbenchmark: bf16, 16x128 heads, page 16, context lengths
    log-normal with median 2048 (sigma 0.6), clipped to [128, 8192],
    LAST-EXITED with 4 planes, exit depths uniform in {1..4}, random page
    permutation. The pool holds exactly the pages the rows' 4 planes need."""
    rng = np.random.default_rng(seed)
    planes, page = 4, 16
    lengths = np.clip(np.rint(rng.lognormal(math.log(2048.0), sigma, size=rows)), 128, 8192)
    lengths = lengths.astype(np.int32)
    depths = rng.integers(1, 5, size=rows).astype(np.int64) - 1
    exits = [rng.integers(1, 5, size=int(c) - 1).astype(np.int64) - 1 for c in lengths]
    num_blocks = int(sum(math.ceil(int(c) / page) for c in lengths)) * planes
    free_order = rng.permutation(num_blocks)
    tables = allocate_tables(lengths, planes, page, free_order)
    return DecodePlan(rows, 16, 16, 128, page, planes, num_blocks, lengths, depths, exits, tables,
                      free_order=free_order)


def config5_plan(seed: int = 0, rows: int = 64) -> DecodePlan:
    """Long-context skewed decode, SHARED layout (one plane): context lengths
    Pareto(alpha=1.5) scaled to a minimum of 1024, clipped at 32768."""
    rng = np.random.default_rng(seed)
    page = 16
    lengths = np.clip(np.floor(1024 * (1 + rng.pareto(1.5, size=rows))), 1024, 32768).astype(np.int32)
    depths = rng.integers(1, 5, size=rows).astype(np.int64) - 1
    num_blocks = int(sum(math.ceil(int(c) / page) for c in lengths))
    free_order = rng.permutation(num_blocks)
    tables = allocate_tables(lengths, 1, page, free_order)
    return DecodePlan(
        rows, 16, 16, 128, page, 1, num_blocks, lengths, depths, [], tables, layout="shared",
        free_order=free_order,
    )


def write_schedule(plan: DecodePlan):
    """The LAST-EXITED write/finalize sequence that builds ``plan``'s history:
    for each row r and past position p: writes at depths 0..exit_p, then the
    exit copy from exit_p into deeper planes; then the row's current token at
    its query depth. Yields ("write", r, depth, pos) / ("finalize", r, pos, exit).
    Values are drawn in this order (two [Hkv, D] fp32 normals per write)."""
    for r in range(plan.num_rows):
        pos = int(plan.context_lengths[r]) - 1
        for p in range(pos):
            e = int(plan.exit_depths[r][p])
            for depth in range(e + 1):
                yield ("write", r, depth, p)
            yield ("finalize", r, p, e)
        yield ("write", r, int(plan.query_depths[r]), pos)


@dataclass
class PrefillPlan:
    """Chunked prefill of many prompts over one paged pool."""

    prompt_lengths: np.ndarray  # int64 [requests]
    reused: np.ndarray  # int64 [requests], reused prefix tokens (whole pages)
    tables: np.ndarray  # int32 [requests, width]; leading pages shared with a donor
    num_blocks: int
    chunk: int
    page: int = 16
    num_q_heads: int = 16
    num_kv_heads: int = 16
    head_dim: int = 128

    def rounds(self):
        """Per chunk round: (request ids, chunk starts, chunk lengths)."""
        starts = self.reused.copy()
        while True:
            active = np.nonzero(starts < self.prompt_lengths)[0]
            if len(active) == 0:
                return
            lengths = np.minimum(self.chunk, self.prompt_lengths[active] - starts[active])
            yield active, starts[active].copy(), lengths
            starts[active] += lengths

    def causal_pairs(self) -> int:
        """Query-key pairs attended: sum over computed positions i of (i + 1)."""
        length = self.prompt_lengths.astype(np.int64)
        s = self.reused.astype(np.int64)
        return int(((length * (length + 1) - s * (s + 1)) // 2).sum())

    def flops(self) -> int:
        return 4 * self.head_dim * self.num_q_heads * self.causal_pairs()


def config4_plan(seed: int = 0, requests: int = 64, chunk: int = 2048) -> PrefillPlan:
    """64 prompts with lengths uniform in [512, 8192], chunk 2048,
    bf16 16x128 heads, page 16; each request's number of shared leading pages
    is uniform in [0, 50%] of its pages and those pages point at one donor's
    pages (prefix reuse: they are attended, not recomputed)."""
    rng = np.random.default_rng(seed)
    page = 16
    lengths = rng.integers(512, 8193, size=requests).astype(np.int64)
    pages = (lengths + page - 1) // page
    shared = np.array([rng.integers(0, p // 2 + 1) for p in pages], dtype=np.int64)
    shared = np.minimum(shared, (lengths - 1) // page)  # at least one token to compute
    donor = int(shared.max())
    num_blocks = donor + int((pages - shared).sum())
    order = rng.permutation(num_blocks)
    donor_pages, fresh = order[:donor], order[donor:]
    width = int(pages.max())
    tables = np.full((requests, width), -1, dtype=np.int32)
    cursor = 0
    for r in range(requests):
        tables[r, : shared[r]] = donor_pages[: shared[r]]
        own = int(pages[r] - shared[r])
        tables[r, shared[r] : pages[r]] = fresh[cursor : cursor + own]
        cursor += own
    return PrefillPlan(lengths, shared * page, tables, num_blocks, chunk)


def lpt_assign(kv_bytes, ranks: int):
    """Greedy longest-processing-time assignment of requests to ranks by KV
    bytes: returns a list of request-index lists, one per rank."""
    order = np.argsort(-np.asarray(kv_bytes), kind="stable")
    loads = [0] * ranks
    parts = [[] for _ in range(ranks)]
    for i in order:
        r = min(range(ranks), key=lambda k: (loads[k], k))
        parts[r].append(int(i))
        loads[r] += int(kv_bytes[i])
    return parts
