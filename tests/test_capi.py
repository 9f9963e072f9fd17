"""The C-ABI library loads without a GPU and exports every entry point that
include/rlt_b200.h declares, with the argument counts the binding uses."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from vllm_rlt_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "rlt_b200.h"


def declared_functions():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    decls = {}
    for match in re.finditer(r"\b(?:int|size_t)\s+(rlt_\w+)\s*\(([^)]*)\)\s*;", text):
        args = [a.strip() for a in match.group(2).split(",") if a.strip() and a.strip() != "void"]
        decls[match.group(1)] = len(args)
    return decls


def test_header_declares_the_path():
    names = set(declared_functions())
    for required in ("rlt_paged_decode", "rlt_paged_prefill", "rlt_kv_write", "rlt_finalize",
                     "rlt_metadata", "rlt_stage_prefill", "rlt_expand_prefill", "rlt_gather",
                     "rlt_scatter"):
        assert required in names


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    for name, nargs in declared_functions().items():
        assert hasattr(lib, name), name
        assert name in _lib.SIGNATURES, f"{name} has no ctypes signature"
        assert len(_lib.SIGNATURES[name][1]) == nargs, name


def test_host_only_entry_points_without_gpu():
    lib = _lib.load()
    assert lib.rlt_version() >= 100
    # no split can be needed when every row fits one split
    assert lib.rlt_paged_decode_workspace_bytes(8, 16, 128, 16, 16) == 0
    # The reference's graph width 4096 x page 16 allows 128 splits per row;
    # split partials (fp32 acc + max + sum per query head) live in a ring of
    # max(2 x 128, 4096) (row, split) slots, not rows x 128. Before them the
    # int metadata: one merge counter per (row, query head), the rows + 1
    # work schedule, the claim counter, the row order, each row's first ring
    # pair, per-row merge counts, one sequence word per ring slot and the
    # wrap flag, rounded to 16 bytes.
    def expected(rows, ring):
        meta = (rows * 16 + 4 * rows + 3 + ring) * 4
        return (meta + 15) // 16 * 16 + ring * 16 * 130 * 4

    assert lib.rlt_paged_decode_workspace_bytes(256, 16, 128, 16, 4096) == expected(256, 4096)
    assert lib.rlt_paged_decode_workspace_bytes(256, 16, 128, 16, 4096) < 35 << 20
    # few rows: one slot per possible (row, split), no ring wrap-around
    assert lib.rlt_paged_decode_workspace_bytes(4, 16, 128, 16, 4096) == expected(4, 4 * 128)
    assert lib.rlt_paged_decode_workspace_bytes(40, 16, 128, 16, 4096) == expected(40, 4096)
    assert lib.rlt_paged_prefill_workspace_bytes(0, 16, 128, 16, 64) == 0


def test_invalid_arguments_are_rejected_before_any_launch():
    lib = _lib.load()
    null = None
    # bad dtype, bad head_dim, bad GQA: the call returns before touching CUDA
    base = [null] * 7 + [0, null]
    shape = [1, 4, 3, 128, 16, 4]
    strides = [0] * 12
    assert lib.rlt_paged_decode(*base, 7, *shape, *strides, 1.0, null) == -1
    assert lib.rlt_paged_decode(*base, 2, 1, 4, 2, 300, 16, 4, *strides, 1.0, null) == -2
    assert lib.rlt_paged_decode(*base, 2, *shape, *strides, 1.0, null) == -3
    # zero rows is a no-op
    assert lib.rlt_paged_decode(*base, 2, 0, 4, 2, 128, 16, 4, *strides, 1.0, null) == 0
    assert lib.rlt_metadata(*([null] * 9), 3, 2, 16, 16, 4, 8, 4, null) == -5
    assert lib.rlt_gather(null, null, null, 1, 1, 4, 3, 4, 4, null) == -1


def test_missing_library_raises(monkeypatch, tmp_path):
    monkeypatch.setattr(_lib, "LIB_PATH", tmp_path / "missing.so")
    monkeypatch.setattr(_lib, "_handle", None)
    with pytest.raises(RuntimeError, match="no fallback"):
        _lib.load()
