"""Packed chunked-prefill paged causal attention (bottom-right aligned).

Same contract as the reference's ``FlashPagedAttention.prefill``
(vllm_rlt/kernels/flash_attention.py:66-96): q ``[tokens, Hq, D]`` packed by
``cu_seqlens_q`` (int32 ``[S+1]``), one block table per sequence (int32
``[S, W]``), ``context_lengths`` = each sequence's last position + 1 (the
keys of the chunk itself are already in the pool). Output ``[tokens, Hq, D]``.
"""

from __future__ import annotations

import torch

from .. import _lib
from .paged_attention import _as_int32, _validate


def paged_prefill(q, key_cache, value_cache, block_tables, context_lengths, cu_seqlens_q,
                  max_seqlen_q, *, out=None):
    _validate(q, key_cache, value_cache, block_tables, context_lengths)
    if cu_seqlens_q.ndim != 1 or cu_seqlens_q.shape[0] != block_tables.shape[0] + 1:
        raise ValueError("cu_seqlens_q must have one entry per sequence plus one")
    if cu_seqlens_q.device != q.device:
        raise ValueError("cu_seqlens_q must live on the query's device")
    if q.stride(-1) != 1:
        q = q.contiguous()
    output = torch.empty_like(q) if out is None else out
    tokens, hq, d = q.shape
    if tokens == 0:
        return output
    tables = _as_int32(block_tables)
    lengths = _as_int32(context_lengths)
    cu = _as_int32(cu_seqlens_q)
    lib = _lib.load()
    device = q.device
    page, hkv = key_cache.shape[1], key_cache.shape[2]
    width = tables.shape[1]
    need = lib.rlt_paged_prefill_workspace_bytes(tokens, hq, d, page, width)
    workspace = torch.empty(need, dtype=torch.uint8, device=device)
    code = lib.rlt_paged_prefill(
        q.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(), tables.data_ptr(),
        lengths.data_ptr(), cu.data_ptr(), output.data_ptr(), workspace.data_ptr(), need,
        _lib.status_word(device).data_ptr(), _lib.DTYPE_CODES[q.dtype],
        tokens, tables.shape[0], int(max_seqlen_q), hq, hkv, d, page, width, key_cache.shape[0],
        q.stride(0), q.stride(1),
        key_cache.stride(0), key_cache.stride(1), key_cache.stride(2),
        value_cache.stride(0), value_cache.stride(1), value_cache.stride(2),
        tables.stride(0), output.stride(0), output.stride(1),
        d ** -0.5, _lib.stream_of(device),
    )
    _lib.check(code, "paged prefill attention")
    return output
