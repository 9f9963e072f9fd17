"""Fused per-layer glue of the Ouro recurrent core on sm_100a: RMSNorm
(+ residual), RoPE fused with the KV page write, SwiGLU. Each rounds where
the reference's torch expressions round (vllm_rlt/models/ouro.py)."""

from __future__ import annotations

import torch

from .. import _lib


def rms_norm(x, weight, eps, residual=None, out=None, weight2=None, out2=None):
    """weight * to_dtype(x * rsqrt(mean(x^2) + eps)) [+ residual].

    With ``weight2`` the same launch also returns the next norm of that
    result, ``(out, rms_norm(out, weight2, eps))``, bit-identical to two calls."""
    if x.stride(-1) != 1:
        x = x.contiguous()
    out = torch.empty_like(x) if out is None else out
    rows, hidden = x.shape
    lib = _lib.load()
    if weight2 is None:
        code = lib.rlt_rms_norm(
            x.data_ptr(), weight.data_ptr(), _lib.ptr(residual), out.data_ptr(),
            _lib.DTYPE_CODES[x.dtype], rows, hidden, float(eps), x.stride(0),
            0 if residual is None else residual.stride(0), out.stride(0),
            _lib.stream_of(x.device))
        _lib.check(code, "rms norm")
        return out
    out2 = torch.empty_like(x) if out2 is None else out2
    code = lib.rlt_rms_norm2(
        x.data_ptr(), weight.data_ptr(), _lib.ptr(residual), out.data_ptr(), weight2.data_ptr(),
        out2.data_ptr(), _lib.DTYPE_CODES[x.dtype], rows, hidden, float(eps), x.stride(0),
        0 if residual is None else residual.stride(0), out.stride(0), out2.stride(0),
        _lib.stream_of(x.device))
    _lib.check(code, "rms norm pair")
    return out, out2


def rope_write_kv(qkv, positions, inv_freq, key_cache, value_cache, layer, write_blocks,
                  write_offsets, heads, kv_heads, head_dim, q_out=None):
    """RoPE on the q and k parts of ``qkv`` [rows, (heads + 2*kv_heads)*D];
    returns q [rows, heads, D]; k (rotated) and v go to the KV pages."""
    rows = qkv.shape[0]
    q_out = torch.empty((rows, heads, head_dim), device=qkv.device, dtype=qkv.dtype) \
        if q_out is None else q_out
    code = _lib.load().rlt_rope_write_kv(
        qkv.data_ptr(), positions.data_ptr(), inv_freq.data_ptr(), q_out.data_ptr(),
        key_cache.data_ptr(), value_cache.data_ptr(), write_blocks.data_ptr(),
        write_offsets.data_ptr(), _lib.status_word(qkv.device).data_ptr(),
        _lib.DTYPE_CODES[qkv.dtype], rows, heads, kv_heads, head_dim, layer, key_cache.shape[2],
        key_cache.shape[0], qkv.stride(0), q_out.stride(0), q_out.stride(1),
        *key_cache.stride()[:4], _lib.stream_of(qkv.device))
    _lib.check(code, "rope + kv write")
    return q_out


def silu_mul(gate_up, intermediate, out=None):
    rows = gate_up.shape[0]
    out = torch.empty((rows, intermediate), device=gate_up.device, dtype=gate_up.dtype) \
        if out is None else out
    code = _lib.load().rlt_silu_mul(gate_up.data_ptr(), out.data_ptr(),
                                    _lib.DTYPE_CODES[gate_up.dtype], rows, intermediate,
                                    gate_up.stride(0), out.stride(0), _lib.stream_of(gate_up.device))
    _lib.check(code, "silu mul")
    return out
