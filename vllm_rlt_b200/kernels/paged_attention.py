"""Depth-aware paged attention backend on the sm_100a kernels.

Drop-in for the reference's attention backends (vllm_rlt/kernels/
paged_attention.py, triton_attention.py, flash_attention.py): the same call
``attention(q, key_cache_layer, value_cache_layer, block_tables,
context_lengths) -> out`` with the same layouts -- q ``[N, Hq, D]``, the
non-contiguous layer views ``[blocks, page, Hkv, D]`` of the 5-D pool, int32
tables ``[N, W]`` padded with -1 (or 0), int32 lengths -- and the same
``.prefill(...)``, ``.info`` and ``.generation`` surface the reference's
cache manager and CUDA-graph proxy call (vllm_rlt/core/kv_cache_manager.py:
559-586, vllm_rlt/worker/cuda_graph.py:21-29).

Every launch is asynchronous on the current torch stream and allocates only
through torch (output, split-KV workspace), so the calls can be captured in
a CUDA graph. There is no fallback: a missing library or an unsupported
device raises.
"""

from __future__ import annotations

import math

import torch

from .. import _lib

_SUPPORTED = (torch.float32, torch.float16, torch.bfloat16)


def _validate(q, key_cache, value_cache, block_tables, context_lengths):
    if q.device.type != "cuda":
        raise ValueError("the B200 attention backend requires a CUDA device")
    if q.ndim != 3 or key_cache.ndim != 4 or value_cache.ndim != 4:
        raise ValueError("expected q [N, Hq, D] and layer views [blocks, page, Hkv, D]")
    if q.shape[-1] > 256:
        raise ValueError("the B200 attention backend supports head_dim <= 256")
    if q.dtype not in _SUPPORTED:
        raise ValueError("the B200 attention backend requires float32, float16 or bfloat16")
    if key_cache.dtype != q.dtype or value_cache.dtype != q.dtype:
        raise ValueError("q, key_cache and value_cache must share a dtype")
    if key_cache.shape != value_cache.shape or key_cache.shape[-1] != q.shape[-1]:
        raise ValueError("key/value cache shapes must match and end in head_dim")
    if q.shape[1] == 0 or q.shape[1] % key_cache.shape[2]:
        raise ValueError("query heads must be a positive multiple of KV heads")
    if key_cache.stride(-1) != 1 or value_cache.stride(-1) != 1:
        raise ValueError("the head_dim dimension of the KV cache must be contiguous")
    if block_tables.ndim != 2 or block_tables.shape[0] != context_lengths.shape[0]:
        raise ValueError("block_tables must be [rows, width] with one length per row")
    for tensor in (key_cache, value_cache, block_tables, context_lengths):
        if tensor.device != q.device:
            raise ValueError("all attention inputs must live on the same device")


def _as_int32(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.int32:
        t = t.to(torch.int32)
    if t.ndim == 2 and t.stride(1) != 1:
        t = t.contiguous()
    if t.ndim == 1 and t.stride(0) != 1:
        t = t.contiguous()
    return t


def paged_attention(q, key_cache, value_cache, block_tables, context_lengths, *, out=None):
    """Launch the decode kernel: one query row per table row."""
    _validate(q, key_cache, value_cache, block_tables, context_lengths)
    if q.stride(-1) != 1:
        q = q.contiguous()
    output = torch.empty_like(q) if out is None else out
    rows, hq, d = q.shape
    if rows == 0:
        return output
    tables = _as_int32(block_tables)
    lengths = _as_int32(context_lengths)
    lib = _lib.load()
    device = q.device
    page, hkv = key_cache.shape[1], key_cache.shape[2]
    width = tables.shape[1]
    need = lib.rlt_paged_decode_workspace_bytes(rows, hq, d, page, width)
    workspace = torch.empty(need, dtype=torch.uint8, device=device) if need else None
    code = lib.rlt_paged_decode(
        q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), tables.data_ptr(),
        lengths.data_ptr(), output.data_ptr(), _lib.ptr(workspace), need,
        _lib.status_word(device).data_ptr(), _lib.DTYPE_CODES[q.dtype],
        rows, hq, hkv, d, page, width, key_cache.shape[0],
        q.stride(0), q.stride(1),
        key_cache.stride(0), key_cache.stride(1), key_cache.stride(2),
        value_cache.stride(0), value_cache.stride(1), value_cache.stride(2),
        tables.stride(0), output.stride(0), output.stride(1),
        q.shape[-1] ** -0.5, _lib.stream_of(device),
    )
    _lib.check(code, "paged decode attention")
    return output


def paged_attention_lse(q, key_cache, value_cache, block_tables, context_lengths, *, out=None):
    """``paged_attention`` that also returns, per row and query head, the
    base-2 log-sum-exp of the scaled scores (fp32 ``[N, Hq]``; -inf for an
    empty row): what merging attention over disjoint token ranges needs."""
    _validate(q, key_cache, value_cache, block_tables, context_lengths)
    if q.stride(-1) != 1:
        q = q.contiguous()
    output = torch.empty_like(q) if out is None else out
    rows, hq, d = q.shape
    lse = torch.empty((rows, hq), dtype=torch.float32, device=q.device)
    if rows == 0:
        return output, lse
    tables = _as_int32(block_tables)
    lengths = _as_int32(context_lengths)
    lib = _lib.load()
    device = q.device
    page, hkv = key_cache.shape[1], key_cache.shape[2]
    width = tables.shape[1]
    need = lib.rlt_paged_decode_workspace_bytes(rows, hq, d, page, width)
    workspace = torch.empty(need, dtype=torch.uint8, device=device) if need else None
    code = lib.rlt_paged_decode_lse(
        q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), tables.data_ptr(),
        lengths.data_ptr(), output.data_ptr(), _lib.ptr(workspace), need,
        _lib.status_word(device).data_ptr(), _lib.DTYPE_CODES[q.dtype],
        rows, hq, hkv, d, page, width, key_cache.shape[0],
        q.stride(0), q.stride(1),
        key_cache.stride(0), key_cache.stride(1), key_cache.stride(2),
        value_cache.stride(0), value_cache.stride(1), value_cache.stride(2),
        tables.stride(0), output.stride(0), output.stride(1),
        q.shape[-1] ** -0.5, lse.data_ptr(), _lib.stream_of(device),
    )
    _lib.check(code, "paged decode attention (log-sum-exp)")
    return output, lse


def b200_paged_attention(q, key_cache, value_cache, block_tables, context_lengths):
    """Explicit dispatch with no silent fallback, mirroring the reference's
    ``triton_paged_attention`` (vllm_rlt/kernels/paged_attention.py:39-54)."""
    if q.device.type != "cuda":
        raise ValueError("the B200 attention backend requires a CUDA device")
    if q.shape[-1] > 256:
        raise ValueError("the B200 attention backend supports head_dim <= 256")
    return paged_attention(q, key_cache, value_cache, block_tables, context_lengths)


class B200PagedAttention:
    """Attention backend object with the surface of the reference's
    ``FlashPagedAttention`` (vllm_rlt/kernels/flash_attention.py:34-130).

    ``generation`` is 4 because the reference's cache manager and runner only
    route packed chunked prefill to a backend that reports generation 4
    (vllm_rlt/core/kv_cache_manager.py:425, vllm_rlt/worker/model_runner.py:274).
    """

    generation = 4

    def __init__(self, device, dtype, head_dim, block_size, backend="b200"):
        device = torch.device(device)
        if device.type != "cuda" or torch.version.hip:
            raise ValueError("the B200 backend requires an NVIDIA CUDA device")
        if dtype not in _SUPPORTED:
            raise ValueError("the B200 backend requires float32, float16 or bfloat16")
        if head_dim <= 0 or head_dim > 256:
            raise ValueError("the B200 backend requires 0 < head_dim <= 256")
        if block_size <= 0:
            raise ValueError("block_size must be positive")
        major, minor = torch.cuda.get_device_capability(device)
        if major != 10:
            raise ValueError(f"the B200 backend is built for sm_100a; found SM{major}{minor}")
        lib = _lib.load()
        self.device, self.dtype, self.head_dim, self.block_size = device, dtype, head_dim, block_size
        self.info = dict(
            backend=backend,
            generation=self.generation,
            library=str(_lib.LIB_PATH),
            version=lib.rlt_version(),
            arch="sm_100a",
        )

    def __call__(self, q, key_cache, value_cache, block_tables, context_lengths):
        return paged_attention(q, key_cache, value_cache, block_tables, context_lengths)

    def prefill(self, q, key_cache, value_cache, block_tables, context_lengths, cu_seqlens_q,
                max_seqlen_q):
        """Packed chunked prefill with bottom-right causal alignment
        (vllm_rlt/kernels/flash_attention.py:66-96)."""
        from .paged_prefill import paged_prefill

        return paged_prefill(q, key_cache, value_cache, block_tables, context_lengths,
                             cu_seqlens_q, max_seqlen_q)

    def check_errors(self) -> list[str]:
        """Synchronise and return metadata errors the kernels reported."""
        return _lib.read_status(self.device)


def decode_bytes(context_lengths, num_q_heads, num_kv_heads, head_dim, elem_bytes, page=16):
    """Algorithmic HBM bytes of one decode call: K and V of every context
    token read once per KV head, q read and out written once, plus the table
    entries and lengths read."""
    total = int(sum(int(c) for c in context_lengths))
    rows = len(context_lengths)
    pages = int(sum(math.ceil(int(c) / page) for c in context_lengths))
    return (total * num_kv_heads * head_dim * 2 * elem_bytes
            + 2 * rows * num_q_heads * head_dim * elem_bytes + pages * 4 + rows * 4)
