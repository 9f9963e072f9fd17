"""Packed chunked prefill at the full configs[3] size against the oracle.

The benchmarked workload itself (``workloads.config4_plan(seed=100)``: 64
prompts of 512..8192 tokens, chunk 2048, prefix pages reused from a donor,
bf16 16x128 heads, page 16) runs as the same four chunk-round launches the
benchmark times. For sampled sequences -- the shortest, the longest, the one
with the largest reused prefix and two more -- sampled query rows of every
chunk (the first and last 32 rows of the chunk, where the causal edge and
the reused prefix meet, and 32 rows between) are recomputed by the oracle's
per-token restatement of the reference's prefill semantics
(oracle.paged_prefill's bottom-right rule, vllm_rlt/kernels/flash_attention.py:
66-96) and compared at the stated bound.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
import vllm_rlt_b200 as rb
from gpu_helpers import to_numpy
from helpers import assert_close, tolerance, ulp
from vllm_rlt_b200 import _lib, workloads

pytestmark = pytest.mark.gpu


def _fill(t, g):
    flat = t.view(-1)
    step = 1 << 28
    for s in range(0, flat.numel(), step):
        n = min(step, flat.numel() - s)
        flat[s : s + n].copy_(torch.randn(n, generator=g, device=t.device))


def config4_case(device="cuda", seed=100):
    """The benchmark's configs[3] inputs: pool, per-round launch inputs."""
    plan = workloads.config4_plan(seed=seed)
    g = torch.Generator(device=device).manual_seed(7)
    key = torch.empty((plan.num_blocks, 16, 16, 128), device=device, dtype=torch.bfloat16)
    value = torch.empty_like(key)
    _fill(key, g)
    _fill(value, g)
    rounds = []
    for active, starts, lengths in plan.rounds():
        cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
        q = torch.empty((int(cu[-1]), 16, 128), device=device, dtype=torch.bfloat16)
        _fill(q, g)
        rounds.append(dict(active=active, starts=starts, chunk=lengths, cu=cu, q=q))
    return plan, key, value, rounds


def run_round(plan, key, value, r, device="cuda"):
    tables = torch.from_numpy(plan.tables[r["active"]]).to(device)
    lengths = torch.from_numpy((r["starts"] + r["chunk"]).astype(np.int32)).to(device)
    return rb.paged_prefill(r["q"], key, value, tables, lengths,
                            torch.from_numpy(r["cu"]).to(device), int(r["chunk"].max()))


def sampled_sequences(plan):
    lengths, reused = plan.prompt_lengths, plan.reused
    picks = [int(np.argmin(lengths)), int(np.argmax(lengths)), int(np.argmax(reused))]
    rng = np.random.default_rng(3)
    for s in rng.permutation(len(lengths)):
        if len(picks) == 5:
            break
        if int(s) not in picks:
            picks.append(int(s))
    return picks


def oracle_rows(plan, key, value, r, out, seq, rng):
    """(got, expected) for sampled query rows of sequence ``seq`` in round
    ``r``; None when the sequence has no chunk in this round."""
    where = np.nonzero(r["active"] == seq)[0]
    if len(where) == 0:
        return None
    i = int(where[0])
    start, chunk = int(r["starts"][i]), int(r["chunk"][i])
    head = np.arange(min(32, chunk))
    tail = np.arange(max(0, chunk - 32), chunk)
    middle = rng.integers(0, chunk, size=32)
    rows = np.unique(np.concatenate([head, tail, middle]))
    pages = int(np.ceil((start + chunk) / plan.page))
    ids = torch.from_numpy(plan.tables[seq, :pages].astype(np.int64)).to(key.device)
    k_seq, v_seq = to_numpy(key[ids]), to_numpy(value[ids])
    base = int(r["cu"][i])
    q_rows = to_numpy(r["q"][torch.from_numpy(base + rows).to(key.device)])
    tables = np.tile(np.arange(pages, dtype=np.int32), (len(rows), 1))
    lengths = (start + rows + 1).astype(np.int64)  # bottom-right causal: prefix + i + 1
    expected = oracle.paged_attention(q_rows, k_seq, v_seq, tables, lengths, "bf16")
    got = to_numpy(out[torch.from_numpy(base + rows).to(out.device)])
    return got, expected


@pytest.fixture(scope="module")
def case():
    return config4_case()


@pytest.mark.parametrize("version", [0, 5, 7, 8])
def test_config4_prefill_matches_oracle_on_sampled_rows(case, version):
    """version 0: the library's default kernel; 5: P rounded to bf16; 7: P
    split into a bf16 hi + lo pair everywhere; 8: 64-key steps with two S
    buffers per query tile."""
    lib = _lib.load()
    previous = lib.rlt_prefill_tc_select(version) if version else None
    try:
        check_config4(case)
    finally:
        if previous is not None:
            lib.rlt_prefill_tc_select(previous)


def check_config4(case):
    plan, key, value, rounds = case
    assert _lib.load().rlt_paged_prefill_uses_tensor_cores(_lib.BF16, 128, 16) == 1
    picks = sampled_sequences(plan)
    rng = np.random.default_rng(11)
    worst, compared = 0.0, 0
    backend = rb.B200PagedAttention("cuda", torch.bfloat16, 128, 16)
    for r in rounds:
        out = run_round(plan, key, value, r)
        torch.cuda.synchronize()
        assert backend.check_errors() == []
        for seq in picks:
            pair = oracle_rows(plan, key, value, r, out, seq, rng)
            if pair is None:
                continue
            got, expected = pair
            a, b = oracle.to_f32(got, "bf16"), oracle.to_f32(expected, "bf16")
            # error beyond the output's own rounding (one bf16 ulp allowed)
            excess = np.abs(a - b) - ulp(b, "bf16") * tolerance("bf16")["ulps"]
            worst = max(worst, float(excess.max()))
            assert_close(got, expected, "bf16")
            compared += got.size
    print(f"configs[3] prefill: {compared} outputs compared, max |err| - 1 ulp = {worst:.3e}")
    assert compared > 100_000
