"""Packed-prefill metadata staging and expansion on sm_100a
(vllm_rlt/kernels/prefill_metadata.py, launched at
vllm_rlt/worker/prefill_metadata.py:53-86)."""

from __future__ import annotations

from .. import _lib


def stage_prefill(source, target, target32, n):
    """target[:n] = source[:n] (int64) and target32[:n] = int32(source[:n])."""
    code = _lib.load().rlt_stage_prefill(source.data_ptr(), target.data_ptr(), target32.data_ptr(),
                                         n, _lib.stream_of(target.device))
    _lib.check(code, "prefill metadata staging")


def expand_prefill(positions, sequences, tables, blocks, offsets, n, width, page):
    """blocks[i] = tables[seq_i * width + pos_i // page], offsets[i] = pos_i % page."""
    device = blocks.device
    code = _lib.load().rlt_expand_prefill(
        positions.data_ptr(), sequences.data_ptr(), tables.data_ptr(), blocks.data_ptr(),
        offsets.data_ptr(), _lib.status_word(device).data_ptr(), n, width, page, tables.numel(),
        _lib.stream_of(device),
    )
    _lib.check(code, "prefill metadata expansion")
