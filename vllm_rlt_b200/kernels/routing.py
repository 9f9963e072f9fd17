"""Routing-bank metadata and resident-slot gather/scatter on sm_100a.

Argument order follows the reference's Triton kernels and their launch
sites (vllm_rlt/kernels/routing.py:7-76; vllm_rlt/worker/async_state.py:
181-197, 215-234) so a runner can swap the launch for a call.
"""

from __future__ import annotations

import torch

from .. import _lib


def metadata(descriptor, tables, slots, positions, lengths, blocks, offsets, out_tables, n, size,
             page, planes, out_width):
    """Depth/page resolution of one bank (vllm_rlt/kernels/routing.py:7-41).

    descriptor int64 [rows >= n, 3] (device or mapped pinned host); tables
    int32 [slots, planes, width]; outputs: slots/positions/blocks/offsets int64,
    lengths int32, out_tables int32 [rows, width] (row stride = width)."""
    if tables.ndim != 3 or tables.dtype != torch.int32 or not tables.is_contiguous():
        raise ValueError("tables must be a contiguous int32 [slots, planes, width] tensor")
    width = tables.shape[2]
    if out_tables.stride(0) != width or out_tables.stride(1) != 1:
        raise ValueError("out_tables rows must be `width` int32 apart")
    device = out_tables.device
    code = _lib.load().rlt_metadata(
        descriptor.data_ptr(), tables.data_ptr(), slots.data_ptr(), positions.data_ptr(),
        lengths.data_ptr(), blocks.data_ptr(), offsets.data_ptr(), out_tables.data_ptr(),
        _lib.status_word(device).data_ptr(), n, size, width, page, planes, out_width,
        tables.shape[0], _lib.stream_of(device),
    )
    _lib.check(code, "routing metadata")


def gather(pool, slots, out, n, size=None):
    """out[row] = pool[slots[row]] for row < n; zeros for n <= row < size."""
    size = out.shape[0] if size is None else size
    width = pool.shape[1] if pool.ndim > 1 else 1
    code = _lib.load().rlt_gather(
        pool.data_ptr(), slots.data_ptr(), out.data_ptr(), n, size, width, pool.element_size(),
        pool.stride(0), out.stride(0), _lib.stream_of(out.device),
    )
    _lib.check(code, "slot gather")
    return out


def scatter(values, slots, pool, n=None):
    """pool[slots[row]] = values[row] for row < n."""
    n = values.shape[0] if n is None else n
    width = pool.shape[1] if pool.ndim > 1 else 1
    code = _lib.load().rlt_scatter(
        values.data_ptr(), slots.data_ptr(), pool.data_ptr(), n, width, pool.element_size(),
        values.stride(0), pool.stride(0), _lib.stream_of(pool.device),
    )
    _lib.check(code, "slot scatter")
