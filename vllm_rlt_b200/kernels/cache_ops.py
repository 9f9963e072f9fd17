"""KV page write and LAST-EXITED exit copy on the sm_100a kernels.

``write_kv`` replaces the reference's index-put page write
``key_cache[write_blocks, layer, write_offsets] = k[:n]`` (and V)
(vllm_rlt/core/kv_cache_manager.py:531-532, vllm_rlt/worker/cuda_graph.py:
16-19). ``finalize`` replaces the exit-copy Triton kernel with the
reference's launch arguments (vllm_rlt/kernels/routing.py:79-109, launched at
vllm_rlt/worker/model_runner.py:543-557). Both are bit-exact copies.
"""

from __future__ import annotations

import torch

from .. import _lib


def _check_pool(key_cache, value_cache):
    if key_cache.ndim != 5 or key_cache.shape != value_cache.shape:
        raise ValueError("KV pools must be [blocks, layers, page, kv_heads, head_dim] and match")
    if key_cache.dtype != value_cache.dtype or key_cache.dtype not in _lib.DTYPE_CODES:
        raise ValueError("KV pools must share a float32, float16 or bfloat16 dtype")
    if key_cache.stride() != value_cache.stride():
        raise ValueError("K and V pools must have identical strides")
    if key_cache.stride(-1) != 1 or key_cache.stride(-2) != key_cache.shape[-1]:
        raise ValueError("each token row of the pool (kv_heads x head_dim) must be contiguous")
    if key_cache.device.type != "cuda":
        raise ValueError("KV pools must live on a CUDA device")


def write_kv(key_cache, value_cache, layer, write_blocks, write_offsets, k, v):
    """key_cache[write_blocks, layer, write_offsets] = k[:n]; same for V."""
    _check_pool(key_cache, value_cache)
    n = int(write_blocks.shape[0])
    blocks_, layers, page, hkv, d = key_cache.shape
    if not 0 <= layer < layers:
        raise ValueError(f"layer must be in [0, {layers})")
    for name, t in (("k", k), ("v", v)):
        if t.ndim != 3 or t.shape[1:] != (hkv, d) or t.shape[0] < n:
            raise ValueError(f"{name} must be [rows >= {n}, {hkv}, {d}]")
        if t.dtype != key_cache.dtype or t.device != key_cache.device:
            raise ValueError(f"{name} must match the pool's dtype and device")
    if n == 0:
        return
    if k.stride(-1) != 1:
        k = k.contiguous()
    if v.stride(-1) != 1:
        v = v.contiguous()
    blocks = write_blocks if write_blocks.dtype == torch.int64 else write_blocks.to(torch.int64)
    offsets = write_offsets if write_offsets.dtype == torch.int64 else write_offsets.to(torch.int64)
    blocks, offsets = blocks.contiguous(), offsets.contiguous()
    device = key_cache.device
    code = _lib.load().rlt_kv_write(
        k.data_ptr(), v.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
        blocks.data_ptr(), offsets.data_ptr(), _lib.status_word(device).data_ptr(),
        _lib.DTYPE_CODES[key_cache.dtype], n, hkv, d, layer, page, blocks_,
        k.stride(0), k.stride(1), v.stride(0), v.stride(1),
        *key_cache.stride()[:4], _lib.stream_of(device),
    )
    _lib.check(code, "KV page write")


def finalize(descriptor, tables, key_cache, value_cache, rows=None):
    """Exit copy for descriptor rows (slot, depth, pos): every layer's K/V of
    the token, plane ``depth`` -> each plane in (depth, planes). ``tables`` is
    the resident ``[slots, planes, width]`` int32 table; ``descriptor`` an
    int64 ``[n, 3]`` tensor on the device or in mapped pinned host memory."""
    _check_pool(key_cache, value_cache)
    if tables.ndim != 3 or tables.dtype != torch.int32 or not tables.is_contiguous():
        raise ValueError("tables must be a contiguous int32 [slots, planes, width] tensor")
    if descriptor.dtype != torch.int64 or not descriptor.is_contiguous():
        raise ValueError("descriptor must be a contiguous int64 [n, 3] tensor")
    n = descriptor.shape[0] if rows is None else int(rows)
    if n == 0:
        return
    slots, planes, width = tables.shape
    blocks_, layers, page, hkv, d = key_cache.shape
    device = key_cache.device
    code = _lib.load().rlt_finalize(
        descriptor.data_ptr(), tables.data_ptr(), key_cache.data_ptr(), value_cache.data_ptr(),
        _lib.status_word(device).data_ptr(), _lib.DTYPE_CODES[key_cache.dtype], n, slots, width,
        planes, page, layers, hkv * d, blocks_, *key_cache.stride()[:3], _lib.stream_of(device),
    )
    _lib.check(code, "exit copy")
