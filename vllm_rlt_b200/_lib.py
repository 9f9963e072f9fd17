"""ctypes binding of the sm_100a C ABI (``include/rlt_b200.h``).

The shared library is built in-tree by ``vllm_rlt_b200._build`` and loaded
from ``vllm_rlt_b200/_lib/librlt_b200.so``. There is no fallback: if the
library is missing every operator raises, so a GPU run can never silently
route through another implementation.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "librlt_b200.so"

F32, F16, BF16 = 0, 1, 2
DTYPE_CODES = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16}

OK = 0
ERRORS = {
    -1: "unsupported dtype",
    -2: "unsupported head_dim",
    -3: "query heads must be a positive multiple of KV heads",
    -4: "workspace missing or too small",
    -5: "invalid shape",
    -6: "misaligned pointer",
    -7: "no suitable CUDA device",
    -8: "launch shape needs more split scratch than the library's static array holds",
}

STATUS_BITS = {
    1: "context length outside [0, table width * page]",
    2: "block id outside the KV pool",
    4: "in-page offset outside [0, page)",
    8: "descriptor slot/depth/position outside the resident tables",
    16: "packed-prefill metadata inconsistent",
    32: "a bounded wait in a kernel timed out (the call's output is void)",
    64: "a tensor-core kernel found its shared memory misaligned",
}

_i32, _i64, _f32, _sz, _p = (
    ctypes.c_int32,
    ctypes.c_int64,
    ctypes.c_float,
    ctypes.c_size_t,
    ctypes.c_void_p,
)

# name -> (restype, argtypes); the order and meaning follow include/rlt_b200.h.
SIGNATURES = {
    "rlt_version": (_i32, []),
    "rlt_paged_decode_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32, _i32]),
    "rlt_paged_decode": (
        _i32,
        [_p, _p, _p, _p, _p, _p, _p, _sz, _p, _i32]
        + [_i32] * 6
        + [_i64] * 12
        + [_f32, _p],
    ),
    "rlt_paged_decode_lse": (
        _i32,
        [_p, _p, _p, _p, _p, _p, _p, _sz, _p, _i32]
        + [_i32] * 6
        + [_i64] * 12
        + [_f32, _p, _p],
    ),
    "rlt_paged_decode_noalloc": (_i32, [_p] * 7 + [_i32] * 7 + [_i64] * 12 + [_f32, _p]),
    "rlt_paged_prefill_workspace_bytes": (_sz, [_i32, _i32, _i32, _i32, _i32]),
    "rlt_paged_prefill": (
        _i32,
        [_p] * 8 + [_sz, _p, _i32] + [_i32] * 8 + [_i64] * 12 + [_f32, _p],
    ),
    "rlt_paged_prefill_uses_tensor_cores": (_i32, [_i32, _i32, _i32]),
    "rlt_prefill_tc_select": (_i32, [_i32]),
    "rlt_paged_decode_shared_workspace_bytes": (_sz, [_i32, _i32, _i32]),
    "rlt_paged_decode_shared": (
        _i32,
        [_p] * 11 + [_sz, _p] + [_i32] * 7 + [_i64] + [_i32] * 3 + [_i64] * 11 + [_f32, _p],
    ),
    "rlt_paged_decode_shared_phases": (
        _i32,
        [_p] * 11 + [_sz, _p] + [_i32] * 7 + [_i64] + [_i32] * 3 + [_i64] * 11
        + [_f32, _i32, _p],
    ),
    "rlt_shared_prefix_suffix": (_i32, [_p] * 6 + [_i32] * 3 + [_i64, _p]),
    "rlt_shared_prefix_select": (_i32, [_i32]),
    "rlt_kv_write": (_i32, [_p] * 7 + [_i32] * 6 + [_i64] * 9 + [_p]),
    "rlt_finalize": (_i32, [_p] * 5 + [_i32] * 8 + [_i64] * 4 + [_p]),
    "rlt_metadata": (_i32, [_p] * 9 + [_i32] * 7 + [_p]),
    "rlt_stage_prefill": (_i32, [_p, _p, _p, _i64, _p]),
    "rlt_expand_prefill": (_i32, [_p] * 6 + [_i64, _i32, _i32, _i64, _p]),
    "rlt_rms_norm": (_i32, [_p] * 4 + [_i32] * 3 + [_f32] + [_i64] * 3 + [_p]),
    "rlt_rms_norm2": (_i32, [_p] * 6 + [_i32] * 3 + [_f32] + [_i64] * 4 + [_p]),
    "rlt_rope_write_kv": (_i32, [_p] * 9 + [_i32] * 7 + [_i64] * 8 + [_p]),
    "rlt_silu_mul": (_i32, [_p, _p, _i32, _i32, _i32, _i64, _i64, _p]),
    "rlt_copy_segments": (_i32, [_p, _i32, _i64, _p, _p]),
    "rlt_enable_peer_access": (_i32, [_i32]),
    "rlt_gather": (_i32, [_p, _p, _p, _i32, _i32, _i32, _i32, _i64, _i64, _p]),
    "rlt_scatter": (_i32, [_p, _p, _p, _i32, _i32, _i32, _i64, _i64, _p]),
}

_lock = threading.Lock()
_handle: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library once; raise if it was not built."""
    global _handle
    if _handle is not None:
        return _handle
    with _lock:
        if _handle is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python -m vllm_rlt_b200._build` "
                    "(there is no fallback implementation)"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (restype, argtypes) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _handle = handle
    return _handle


def check(code: int, what: str) -> None:
    if code == OK:
        return
    if code < 0:
        raise ValueError(f"{what}: {ERRORS.get(code, f'error {code}')}")
    raise RuntimeError(f"{what}: CUDA launch failed with cudaError {code}")


def ptr(tensor: torch.Tensor | None) -> int | None:
    return None if tensor is None else tensor.data_ptr()


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_status: dict[int, torch.Tensor] = {}


def status_word(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the kernels OR metadata-error bits into."""
    index = device.index if device.index is not None else torch.cuda.current_device()
    word = _status.get(index)
    if word is None:
        # a normal tensor even when first requested under torch.inference_mode
        # (the reference's graph runner runs there), so it can be cleared later
        with torch.inference_mode(False):
            word = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
        _status[index] = word
    return word


def read_status(device: torch.device, reset: bool = True) -> list[str]:
    """Synchronise and return (and by default clear) the raised error bits."""
    word = status_word(device)
    value = int(word.item())
    if reset and value:
        word.zero_()
    return [text for bit, text in STATUS_BITS.items() if value & bit]
