"""Shared test utilities: golden-fixture loading and pool replay.

A scenario fixture (tests/golden/make_golden.py) records the reference's
allocation tables, the ordered write/finalize operations and the seed of the
value generator. ``replay_pool`` rebuilds the KV pool by applying the same
operations through a pluggable writer -- the numpy oracle or the CUDA
kernels -- and the caller checks the result against the reference pool's
digest before using it.
"""

from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden"

OP_ALLOC, OP_FREE, OP_WRITE, OP_FINALIZE = 0, 1, 2, 3


def load(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz", allow_pickle=False) as data:
        return {key: data[key] for key in data.files}


def scenario_names() -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob("*.npz") if not p.stem.startswith(("prefill", "routing")))


def value_transform(name: str):
    """The per-write value adjustment a scenario applied (make_golden.py)."""
    if name.startswith("mixed"):
        # request "a" has index 2 (retained=0, hole=1, a=2, b=3)
        return lambda k, v, rid, depth: (k + np.float32(depth * 0.5), v + np.float32(4 if rid == 2 else -4))
    if name.startswith("long"):
        return lambda k, v, rid, depth: (k * np.float32(8), v)
    return None


def digest(array: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(array).tobytes()).hexdigest()


class NumpyWriter:
    """Applies writes/finalizes to numpy pools with the oracle."""

    def __init__(self, shape, dtype: str):
        self.dtype = dtype
        self.key = np.zeros(shape, dtype=oracle.ref_ops.storage_dtype(dtype))
        self.value = np.zeros_like(self.key)

    def write(self, layer, block, offset, k, v):
        oracle.kv_write(self.key, self.value, layer, [block], [offset], k[None], v[None])

    def finalize(self, plane_tables, pos, exit_depth, planes, page):
        oracle.finalize_token(self.key, self.value, plane_tables, pos, exit_depth, planes, page)


def replay_pool(fx: dict, name: str, writer) -> None:
    """Replay a scenario's operations through ``writer``."""
    layers, hkv, hq, d, num_blocks, page, loops, seed = (int(x) for x in fx["dims"])
    dtype = str(fx["dtype"])
    layout = str(fx["layout"])
    planes = loops if layout == "last_exited" else 1
    tables = fx["alloc_tables"]
    transform = value_transform(name)
    rng = np.random.default_rng([seed, 1])
    for kind, a, b, c, e in fx["ops"].tolist():
        if kind == OP_WRITE:
            layer, rid, depth, pos = a, b, c, e
            k = rng.standard_normal((1, hkv, d), dtype=np.float32)
            v = rng.standard_normal((1, hkv, d), dtype=np.float32)
            k = oracle.to_f32(oracle.from_f32(k, dtype), dtype)[0]
            v = oracle.to_f32(oracle.from_f32(v, dtype), dtype)[0]
            if transform is not None:
                k, v = transform(k, v, rid, depth)
            plane = depth if layout == "last_exited" else 0
            block = int(tables[rid, plane, pos // page])
            writer.write(layer, block, pos % page, oracle.from_f32(k, dtype), oracle.from_f32(v, dtype))
        elif kind == OP_FINALIZE:
            rid, pos, exit_depth = a, b, c
            if layout == "last_exited":
                writer.finalize(tables[rid], pos, exit_depth, planes, page)
    return None


def query_inputs(fx: dict, qi: int = 0):
    return dict(
        layer=int(fx[f"q{qi}_layer"]),
        q=fx[f"q{qi}_q"],
        block_tables=fx[f"q{qi}_block_tables"],
        context_lengths=fx[f"q{qi}_context_lengths"],
        out=fx[f"q{qi}_out"],
        triton_out=fx[f"q{qi}_triton_out"],
        rows=fx[f"q{qi}_rows"],
    )


def tolerance(dtype: str) -> dict:
    """Attention tolerance against the reference's torch path: max-abs 1e-5
    for fp32 and 2e-3 for bf16/fp16 inputs with fp32 accumulation. For the
    16-bit dtypes the bound adds one unit in the last place of the output
    dtype at the expected value's magnitude: both sides round an fp32 result
    to bf16/fp16, and two correct fp32 results a few fp32 ulps apart can
    round to neighbouring 16-bit values (the reference's own Triton kernel and
    torch oracle differ by exactly that on its bf16 inputs)."""
    if dtype == "f32":
        return dict(atol=1e-5, ulps=0)
    return dict(atol=2e-3, ulps=1)


def ulp(values: np.ndarray, dtype: str) -> np.ndarray:
    """Spacing of the 16-bit output dtype at |values| (normal range)."""
    mantissa_bits = {"bf16": 7, "f16": 10, "f32": 23}[dtype]
    _, exponent = np.frexp(np.abs(values))
    return np.ldexp(1.0, exponent - 1 - mantissa_bits)


def assert_close(actual, expected, dtype: str, **override):
    tol = tolerance(dtype)
    tol.update(override)
    a = oracle.to_f32(actual, dtype).astype(np.float64)
    b = oracle.to_f32(expected, dtype).astype(np.float64)
    assert a.shape == b.shape, (a.shape, b.shape)
    bound = tol["atol"] + tol.get("ulps", 0) * ulp(b, dtype) + tol.get("rtol", 0.0) * np.abs(b)
    err = np.abs(a - b)
    bad = ~(err <= bound)
    if bad.any():
        idx = np.argwhere(bad)[0]
        raise AssertionError(
            f"{int(bad.sum())} of {a.size} elements exceed {tol}; "
            f"max abs err {err.max():.3e}; first at {tuple(idx)}: {a[tuple(idx)]} vs {b[tuple(idx)]}"
        )
    return float(err.max()) if err.size else 0.0


def prefill_names() -> list[str]:
    return sorted(p.stem for p in GOLDEN.glob("prefill*.npz"))


def prefill_case(name: str, writer_factory):
    """Rebuild a packed-prefill scenario: prefix writes (drawn from the
    recorded seed), then per layer the chunk's k, v, q (stored in the fixture
    or re-drawn in the order make_golden.py drew them). Returns the fixture,
    the writer holding the prefix pool and the per-layer inputs."""
    fx = load(name)
    dtype = str(fx["dtype"])
    d, blocks, _ = (int(x) for x in fx["geometry"]) if "geometry" in fx else (64, 80, 65)
    writer = writer_factory((blocks, 2, 16, 2, d), dtype)
    rng = np.random.default_rng(fx["prefix_seed"].tolist())

    def draw(shape):
        return oracle.from_f32(rng.standard_normal(shape, dtype=np.float32), dtype)

    for rid, depth, prefix, count in fx["spec"].tolist():
        for layer in range(2):
            if prefix:
                kv = draw((prefix, 2, d))
                neg = oracle.from_f32(-oracle.to_f32(kv, dtype), dtype)
                for p in range(prefix):
                    writer.write(layer, int(fx["alloc_tables"][rid, depth, p // 16]), p % 16,
                                 kv[p], neg[p])
    n = int(fx["cu_seqlens_q"][-1])
    inputs = []
    for layer in range(2):
        if f"k{layer}" in fx:
            inputs.append((fx[f"k{layer}"], fx[f"v{layer}"], fx[f"q{layer}"]))
        else:
            k, v, q = draw((n, 2, d)), draw((n, 2, d)), draw((n, 4, d))
            inputs.append((k, v, q))
    return fx, writer, inputs
