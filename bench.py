"""Benchmark: depth-aware paged decode attention on B200 (HBM GB/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (configs[1] of the reference's hot-path benchmark set): one layer of
paged decode attention, 256 rows, bf16, 16 query heads = 16 KV heads,
head_dim 128, page 16, context lengths log-normal (median 2048, sigma 0.6)
clipped to [128, 8192], LAST-EXITED layout with 4 depth planes (each row
attends through the table of its own query plane), random page permutation.
Inputs are seeded synthetic data. One step = one decode call over the batch.
Each call reads ~5 GB of K/V, far more than the 126 MB L2, so no flush is
needed between steps.

Multi-GPU (torchrun, one process per GPU): request-sharded replicas with no
collective on the data path -- every rank runs its own 256-row batch (weak
scaling); the step time is the max over ranks of the device-timed region.

--impl reference times the reference's own CPU path, torch_paged_attention
from the unmodified reference installed under baseline/_ref (the numpy
restatement in oracle/ when that install is absent), on all of this box's
host cores, on the whole batch when a call fits the run's time budget and a
stated row sample otherwise; its line also carries the reference's CPU
KVCacheManager.write / finalize_token times.

--impl reference-triton times the reference's own GPU decode, its Triton
kernel behind vllm_rlt.kernels.paged_attention.triton_paged_attention, from
the unmodified reference installed under baseline/_ref, on the same GPU
workload as our arm (rank 0 only; prints an "unavailable" line when that
install or Triton is missing).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "paged decode attn HBM GB/s (% of peak); Ouro-1.4B mixed-depth decode tok/s/GPU"
WORKLOAD = ("configs[1]: single-layer depth-aware paged decode, 256 rows, bf16, 16x128 heads, "
            "page 16, ctx lognormal(median 2048, sigma 0.6) in [128, 8192], LAST-EXITED 4 planes")
FALLBACK_HBM_GBS = 6650.0


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference", "reference-triton"], default="ours")
    p.add_argument("--rows", type=int, default=256)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-extras", action="store_true",
                   help="skip the Ouro, prefill, long-context and shared-prefix sub-measurements")
    p.add_argument("--workload",
                   choices=["decode", "prefill", "longctx", "ouro", "shared", "kernels",
                            "reference-engine"],
                   default="decode",
                   help="decode: the headline line; the others: that workload alone")
    return p.parse_args()


def measured_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def measured_tensor_peak():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["bf16_tflops"]), "measured (burst)"
    return 1590.0, "fallback (burst)"


def committed_traffic():
    """Per-launch DRAM bytes of the decode call from the committed ncu summary."""
    path = ROOT / "profiles" / "decode_config2_traffic.json"
    if path.exists():
        return json.loads(path.read_text())
    return None


# ------------------------------------------------------------------ clocks


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.file, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9 and parts[1].isdigit():
                rows.append(parts)
        os.unlink(self.file.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [int(r[1]) for r in rows]
        loaded = [s for s in sm if s > 300] or sm
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": int(statistics.median(loaded)), "sm_max_mhz": int(rows[0][2]),
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------- reference (CPU)


def decode_config(plan, world):
    """The headline workload's config, shared by both arms' lines."""
    from vllm_rlt_b200.kernels.paged_attention import decode_bytes

    return {
        "workload": WORKLOAD,
        "rows_per_gpu": plan.num_rows,
        "sum_ctx_per_gpu": int(plan.context_lengths.sum()),
        "bytes_per_step_per_gpu": int(decode_bytes(plan.context_lengths, plan.num_q_heads,
                                                   plan.num_kv_heads, plan.head_dim, 2,
                                                   plan.page)),
        "l2": "no flush: each step reads ~5 GB of K/V (> 126 MB L2)",
        "parallelism": f"{world} request-sharded replicas, no data-path collective",
    }


def reference_module(name):
    """Import a module of the unmodified reference installed under
    baseline/_ref; None when that install is missing."""
    import importlib

    path = str(ROOT / "baseline" / "_ref")
    if not (ROOT / "baseline" / "_ref" / "vllm_rlt" / "__init__.py").exists():
        return None
    if path not in sys.path:
        sys.path.insert(0, path)
    try:
        return importlib.import_module(name)
    except Exception:  # an install that cannot be imported counts as absent
        return None


class HostDecode:
    """configs[1] rows on the host, for the reference's own CPU path.

    The selected rows' query-plane pages are laid out in a compact bf16 pool
    (each row's pages consecutive), filled by tiling a bank of 512 seeded
    N(0,1) pages: the reference's torch_paged_attention reads every context
    token of every row once, so its time depends on the shapes only."""

    BANK_PAGES = 512

    def __init__(self, plan, rows, seed=0):
        import torch

        self.rows = list(rows)
        page, hkv, d = plan.page, plan.num_kv_heads, plan.head_dim
        lengths = np.array([int(plan.context_lengths[r]) for r in self.rows], dtype=np.int64)
        pages = (lengths + page - 1) // page
        total = int(pages.sum())
        g = torch.Generator().manual_seed(seed)
        bank_k = torch.randn((self.BANK_PAGES, page, hkv, d), generator=g).to(torch.bfloat16)
        bank_v = torch.randn((self.BANK_PAGES, page, hkv, d), generator=g).to(torch.bfloat16)
        pick = torch.arange(total) % self.BANK_PAGES
        self.key = bank_k[pick]
        self.value = bank_v[pick]
        width = int(pages.max())
        tables = np.full((len(self.rows), width), -1, dtype=np.int32)
        first = np.concatenate([[0], np.cumsum(pages)[:-1]])
        for i, (f, n) in enumerate(zip(first, pages)):
            tables[i, :n] = np.arange(f, f + n)
        self.tables = torch.from_numpy(tables)
        self.lengths = torch.from_numpy(lengths.astype(np.int32))
        self.q = torch.randn((len(self.rows), plan.num_q_heads, d), generator=g).to(torch.bfloat16)
        self.tokens = int(lengths.sum())
        from vllm_rlt_b200.kernels.paged_attention import decode_bytes

        self.bytes = decode_bytes(lengths, plan.num_q_heads, hkv, d, 2, page)

    def run(self, fn):
        return fn(self.q, self.key, self.value, self.tables, self.lengths)


def reference_cpu_path():
    """(callable, kind, label) of the reference's CPU decode: its own
    torch_paged_attention (vllm_rlt/kernels/paged_attention.py:12-36) from the
    unmodified install, else the numpy restatement of it in oracle/."""
    import torch

    module = reference_module("vllm_rlt.kernels.paged_attention")
    if module is not None:
        return module.torch_paged_attention, "reference", \
            "the reference's torch_paged_attention (baseline/_ref), bf16 inputs, fp32 math"
    import oracle

    def bits(t):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)

    def port(q, k, v, tables, lengths):
        return oracle.paged_attention(bits(q), bits(k), bits(v), tables.numpy(),
                                      lengths.numpy(), "bf16")

    return port, "port", "numpy restatement of the reference's torch path (oracle/), " \
        "the reference install being absent"


def reference_cpu_sample(plan, budget_s):
    """Rows per step for the reference's CPU path: the whole batch when one
    call fits ``budget_s`` seconds at the rate of a pilot call, else the
    largest seeded random subset that does. Returns (HostDecode, fn, kind,
    label, threads)."""
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    fn, kind, label = reference_cpu_path()
    order = [int(r) for r in np.random.default_rng(123).permutation(plan.num_rows)]
    pilot = HostDecode(plan, order[:8])
    pilot.run(fn)
    t0 = time.perf_counter()
    pilot.run(fn)
    rate = pilot.tokens / max(time.perf_counter() - t0, 1e-6)  # context tokens per second
    rows, tokens = [], 0
    for r in order:
        n = int(plan.context_lengths[r])
        if rows and (tokens + n) / rate > budget_s:
            break
        rows.append(r)
        tokens += n
    return HostDecode(plan, rows), fn, kind, label, threads


def cpu_model() -> str:
    """The host CPU's model name (Linux /proc/cpuinfo), for the baseline lines."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def single_thread_rate(plan, fn, budget_s=3.0):
    """The reference's CPU path on one host thread (torch.set_num_threads(1)):
    GB/s over a seeded 4-row sample, repeated for about ``budget_s`` seconds."""
    import torch

    before = torch.get_num_threads()
    torch.set_num_threads(1)
    try:
        rows = [int(r) for r in np.random.default_rng(321).permutation(plan.num_rows)[:4]]
        host = HostDecode(plan, rows, seed=1)
        host.run(fn)
        reps, spent = 0, 0.0
        while spent < budget_s and reps < 20:
            t0 = time.perf_counter()
            host.run(fn)
            spent += time.perf_counter() - t0
            reps += 1
        return {"value": round(host.bytes * reps / spent / 1e9, 3), "unit": "GB/s", "cores": 1,
                "sample": f"{len(rows)} rows (sum ctx {host.tokens}) x {reps} calls"}
    finally:
        torch.set_num_threads(before)


def prefill_cpu_baseline(budget_s=5.0, rows_per_seq=32, seqs=4):
    """configs[3] on the host: the reference's CPU attention path
    (torch_paged_attention, vllm_rlt/kernels/paged_attention.py:12-36) over
    per-token query rows, each row attending its bottom-right causal context
    (the flat-table form of tests/test_flash_attention.py:169-186). A seeded
    sample: ``seqs`` prompts of the bench plan, ``rows_per_seq`` query rows of
    each spread over its computed (not reused) tokens; TFLOP/s on the bench's
    count (4 x D x Hq per attended key), repeated for about ``budget_s``
    seconds on all host cores."""
    import torch

    from vllm_rlt_b200 import workloads

    torch.set_num_threads(os.cpu_count() or 1)
    fn, kind, label = reference_cpu_path()
    plan = workloads.config4_plan(seed=100)
    rng = np.random.default_rng(5)
    picks = rng.choice(len(plan.prompt_lengths), size=seqs, replace=False)
    g = torch.Generator().manual_seed(9)
    page, hkv, d, hq = 16, 16, 128, 16
    qs, ks, vs, tabs, lens, firsts = [], [], [], [], [], 0
    for sq in picks:
        length = int(plan.prompt_lengths[sq])
        pages = -(-length // page)
        ks.append(torch.randn((pages, page, hkv, d), generator=g).to(torch.bfloat16))
        vs.append(torch.randn((pages, page, hkv, d), generator=g).to(torch.bfloat16))
        start = int(plan.reused[sq])  # reused prefix rows are not queries
        rows = np.unique(np.linspace(start, length - 1, rows_per_seq).astype(np.int64))
        for r in rows:
            t = np.full(-(-length // page), -1, dtype=np.int32)
            t[:pages] = np.arange(firsts, firsts + pages, dtype=np.int32)
            tabs.append(t)
            lens.append(int(r) + 1)  # query token r of the prompt sees keys 0..r
        firsts += pages
        qs.append(torch.randn((len(rows), hq, d), generator=g).to(torch.bfloat16))
    width = max(len(t) for t in tabs)
    tables = np.full((len(tabs), width), -1, dtype=np.int32)
    for i, t in enumerate(tabs):
        tables[i, : len(t)] = t
    q = torch.cat(qs)
    key, value = torch.cat(ks), torch.cat(vs)
    t_tables = torch.from_numpy(tables)
    t_lengths = torch.tensor(lens, dtype=torch.int32)
    flops = 4 * d * hq * int(sum(lens))
    fn(q, key, value, t_tables, t_lengths)
    reps, spent = 0, 0.0
    while spent < budget_s and reps < 20:
        t0 = time.perf_counter()
        fn(q, key, value, t_tables, t_lengths)
        spent += time.perf_counter() - t0
        reps += 1
    return {"value": round(flops * reps / spent / 1e12, 5), "unit": "TFLOP/s", "kind": kind,
            "cores": torch.get_num_threads(),
            "sample": f"{len(lens)} query rows of {seqs} configs[3] prompts (sum of attended "
                      f"keys {int(sum(lens))}) x {reps} calls; {label}"}


def longctx_cpu_baseline(budget_s=5.0):
    """configs[4] on the host: the reference's CPU decode path on a seeded row
    sample of the one-GPU request set (as the decode line's cpu_baseline)."""
    from vllm_rlt_b200 import workloads

    plan = workloads.config5_plan(seed=0, rows=64)
    host, fn, kind, label, threads = reference_cpu_sample(plan, budget_s / 2)
    host.run(fn)
    reps, spent = 0, 0.0
    while spent < budget_s and reps < 20:
        t0 = time.perf_counter()
        host.run(fn)
        spent += time.perf_counter() - t0
        reps += 1
    return {"value": round(host.bytes * reps / spent / 1e9, 3), "unit": "GB/s", "kind": kind,
            "cores": threads,
            "sample": f"{len(host.rows)} of {plan.num_rows} rows (sum ctx {host.tokens}) x "
                      f"{reps} calls; {label}"}


def reference_kv_cpu(batch=64, reps=20):
    """BASELINE B4: the reference's CPU KVCacheManager.write (one layer, a
    batch of rows) and finalize_token (one token, every layer, into the deeper
    planes) in microseconds per call, Ouro geometry (24 layers, 16 KV heads x
    128, page 16, 4 planes), bf16 (vllm_rlt/core/kv_cache_manager.py:498-614)."""
    import torch

    module = reference_module("vllm_rlt.core.kv_cache_manager")
    if module is None:
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    torch.set_num_threads(os.cpu_count() or 1)
    cache = module.KVCacheManager(num_layers=24, num_kv_heads=16, head_dim=128,
                                  num_blocks=4 * batch, block_size=16, max_loops=4,
                                  dtype=torch.bfloat16)
    ids = [f"r{i}" for i in range(batch)]
    for rid in ids:
        cache.allocate(rid, 16)
    k = torch.randn(batch, 16, 128).to(torch.bfloat16)
    for layer in range(24):  # position 0 at depth 0 of every layer: finalize may then run
        cache.write(layer, ids, [0] * batch, [0] * batch, k, k)
    t0 = time.perf_counter()
    for i in range(reps):
        cache.write(i % 24, ids, [0] * batch, [0] * batch, k, k)
    write_us = (time.perf_counter() - t0) / reps * 1e6
    t0 = time.perf_counter()
    for i in range(reps):
        cache.finalize_token(ids[i % batch], 0, 0)
    finalize_us = (time.perf_counter() - t0) / reps * 1e6
    return {"write_us": round(write_us, 1), "write_rows": batch,
            "finalize_token_us": round(finalize_us, 1),
            "finalize": "one token: 24 layers x K,V copied from plane 0 into planes 1-3",
            "threads": torch.get_num_threads(), "kind": "reference"}


def reference_engine_cpu(requests=4, prompt=16, new_tokens=8):
    """BASELINE B5: the reference's own engine end to end on the host cores --
    LLMEngine with its torch attention backend (vllm_rlt/engine/llm_engine.py,
    vllm_rlt/kernels/paged_attention.py:12-36) serving a random-init
    Ouro-1.4B-shaped model (24 layers x 4 loops, 2048 hidden, 16x128 heads,
    SwiGLU 5632, vocab 49152, RoPE 1e4) in fp32, a reduced batch, exit depth
    per token from a seeded trace in {1..4}. Plumbing only: no GPU."""
    import torch

    config_mod = reference_module("vllm_rlt.models")
    engine_mod = reference_module("vllm_rlt.engine.llm_engine")
    root = reference_module("vllm_rlt")
    if config_mod is None or engine_mod is None or root is None:
        return {"unavailable": "the reference is not installed under baseline/_ref"}
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    t0 = time.perf_counter()
    model = config_mod.OuroForCausalLM(config_mod.OuroConfig(rope_theta=10000.0)).eval()
    build_s = time.perf_counter() - t0
    rng = np.random.default_rng(8)
    # the first output follows the prompt's prefill (all 4 loops); later ones exit at 1..4
    traces = {str(i): [4] + [int(x) for x in rng.integers(1, 5, size=new_tokens + 3)]
              for i in range(requests)}
    engine = engine_mod.LLMEngine(
        model, cache_config=root.CacheConfig(num_blocks=requests * 8, block_size=16),
        exit_config=root.ExitConfig("trace", depths_by_request=traces),
        attention_backend="torch")
    for i in range(requests):
        engine.add_request(str(i), [int(x) for x in rng.integers(0, 49152, size=prompt)],
                           root.SamplingParams(max_tokens=new_tokens, min_loops=1, ignore_eos=True))
    t0 = time.perf_counter()
    generated = 0
    while engine.has_unfinished_requests():
        for out in engine.step():
            if out.finished:
                generated += len(out.token_ids)
    run_s = time.perf_counter() - t0
    return {"tok_s": round(generated / run_s, 3), "tokens": generated, "seconds": round(run_s, 2),
            "model_init_s": round(build_s, 1), "threads": threads,
            "batch": f"{requests} requests x {prompt}-token prompts, {new_tokens} new tokens each",
            "kind": "reference", "dtype": "fp32 (the reference's CPU default)"}


def run_reference(args):
    from vllm_rlt_b200 import workloads

    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    plan = workloads.config2_plan(0, rows=args.rows)
    # the whole run (warm-up and timed steps) within about three minutes
    budget = max(1.0, 150.0 / max(args.steps + args.warmup, 1))
    host, fn, kind, label, threads = reference_cpu_sample(plan, budget)
    for _ in range(args.warmup):
        host.run(fn)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        host.run(fn)
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = host.bytes * args.steps / total / 1e9
    sample = (f"{len(host.rows)} of {plan.num_rows} rows per step (sum ctx {host.tokens}); "
              f"{label}; {threads} threads")
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": (decode_config(plan, 1) if len(host.rows) == plan.num_rows else
                   {"workload": WORKLOAD, "rows_per_gpu": len(host.rows),
                    "sum_ctx_per_gpu": host.tokens, "bytes_per_step_per_gpu": int(host.bytes),
                    "sample": sample}),
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads,
                         "kind": kind, "sample": sample, "cpu_model": cpu_model(),
                         "single_thread": single_thread_rate(plan, fn)},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "reference_kv_cpu": reference_kv_cpu(),
    }
    print(json.dumps(line), flush=True)


def run_reference_triton(args):
    import torch

    from vllm_rlt_b200 import workloads
    from vllm_rlt_b200.kernels.paged_attention import decode_bytes

    if int(os.environ.get("RANK", "0")) != 0:
        return
    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    try:
        from vllm_rlt.kernels.paged_attention import triton_paged_attention
    except Exception as exc:  # the install is optional
        print(json.dumps({"impl": "reference-triton",
                          "unavailable": f"reference not importable from baseline/_ref: {exc}"}))
        return
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    plan = workloads.config2_plan(seed=0, rows=args.rows)
    g = torch.Generator(device=device).manual_seed(1000)
    shape = (plan.num_blocks, 1, plan.page, plan.num_kv_heads, plan.head_dim)
    kpool = torch.empty(shape, device=device, dtype=torch.bfloat16)
    vpool = torch.empty_like(kpool)
    fill_random(kpool, g)
    fill_random(vpool, g)
    k_layer, v_layer = kpool[:, 0], vpool[:, 0]
    tables = torch.from_numpy(plan.block_tables()).to(device)
    lengths = torch.from_numpy(plan.context_lengths).to(device)
    q = torch.randn((plan.num_rows, 16, 128), generator=g, device=device).to(torch.bfloat16)
    step_bytes = decode_bytes(plan.context_lengths, 16, 16, 128, 2, plan.page)

    def step():
        return triton_paged_attention(q, k_layer, v_layer, tables, lengths)

    for _ in range(max(args.warmup, 1)):
        out = step()
    torch.cuda.synchronize(device)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        t0.record()
        for _ in range(args.steps):
            out = step()
        t1.record()
        torch.cuda.synchronize(device)
    ms = t0.elapsed_time(t1) / args.steps
    value = step_bytes / (ms / 1e3) / 1e9
    peak, kind = measured_peak()
    import vllm_rlt_b200 as rb

    ours = rb.B200PagedAttention(device, torch.bfloat16, 128, plan.page)(q, k_layer, v_layer,
                                                                          tables, lengths)
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "impl": "reference-triton",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": WORKLOAD, "rows": plan.num_rows,
                   "kernel": "reference _paged_attention_kernel (Triton), one program per "
                             "(row, query head), 32-token tiles, no split-KV"},
        "roofline": {"bound": "hbm", "achieved": round(value, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(value / peak, 4), "peak_kind": kind},
        "max_abs_vs_ours": float((out.float() - ours.float()).abs().max()),
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ extras


def fill_random(t, g):
    """Fill a (large) tensor with N(0,1) in chunks, bounding the fp32 temporary."""
    import torch

    flat = t.view(-1)
    step = 1 << 28
    for s in range(0, flat.numel(), step):
        n = min(step, flat.numel() - s)
        flat[s : s + n].copy_(torch.randn(n, generator=g, device=t.device))


def time_region(fn, steps, warmup, device):
    """Device time of `steps` calls of fn() after `warmup` calls (CUDA events)."""
    import torch

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(device)
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(steps):
        fn()
    b.record()
    torch.cuda.synchronize(device)
    return a.elapsed_time(b) / steps


def prefill_extra(device, steps, warmup, rank):
    """chunked prefill of 64 prompts (uniform 512..8192, chunk
    2048, shared leading pages up to 50%) on the tensor-core kernel."""
    import torch

    import vllm_rlt_b200 as rb
    from vllm_rlt_b200 import workloads

    plan = workloads.config4_plan(seed=100)  # same shape on every rank (weak scaling)
    g = torch.Generator(device=device).manual_seed(7 + rank)
    key = torch.empty((plan.num_blocks, 1, 16, 16, 128), device=device, dtype=torch.bfloat16)
    value = torch.empty_like(key)
    fill_random(key, g)
    fill_random(value, g)
    tables_all = torch.from_numpy(plan.tables).to(device)
    rounds = []
    for active, starts, lengths in plan.rounds():
        cu = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
        q = torch.empty((int(cu[-1]), 16, 128), device=device, dtype=torch.bfloat16)
        fill_random(q, g)
        rounds.append(dict(
            q=q, tables=tables_all[torch.from_numpy(active).to(device)].contiguous(),
            lengths=torch.from_numpy((starts + lengths).astype(np.int32)).to(device),
            cu=torch.from_numpy(cu).to(device), max_q=int(lengths.max())))
    backend = rb.B200PagedAttention(device, torch.bfloat16, 128, 16)

    def step():
        for r in rounds:
            backend.prefill(r["q"], key[:, 0], value[:, 0], r["tables"], r["lengths"], r["cu"],
                            r["max_q"])

    ms = time_region(step, steps, warmup, device)
    errors = backend.check_errors()
    peak, kind = measured_tensor_peak()
    tflops = plan.flops() / (ms / 1e3) / 1e12
    tc = rb._lib.load().rlt_paged_prefill_uses_tensor_cores(rb._lib.BF16, 128, 16)
    return {
        "workload": "configs[3]: 64 prompts U[512,8192], chunk 2048, prefix pages U[0,50%], "
                    "bf16 16x128, page 16",
        "ms_per_step": round(ms, 3), "chunk_rounds": len(rounds),
        "tokens_per_step": int((plan.prompt_lengths - plan.reused).sum()),
        "value": round(tflops, 1), "unit": "TFLOP/s (causal pairs x 4 x D x Hq)",
        "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak,
                     "unit": "TFLOP/s", "frac": round(tflops / peak, 4), "peak_kind": kind},
        "path": "tcgen05" if tc else "cuda-core", "errors": errors,
    }


def longctx_extra(device, steps, warmup, rank, world):
    """long-context skewed decode, SHARED layout, 64 rows per GPU,
    Pareto(1.5) contexts in [1024, 32768], split-KV; the 64 x world requests
    are assigned to ranks by greedy LPT on KV bytes."""
    import torch

    import vllm_rlt_b200 as rb
    from vllm_rlt_b200 import workloads
    from vllm_rlt_b200.kernels.paged_attention import decode_bytes

    full = workloads.config5_plan(seed=0, rows=64 * world)
    kv = full.context_lengths.astype(np.int64) * 16 * 128 * 2 * 2
    parts = workloads.lpt_assign(kv, world)
    mine = np.array(sorted(parts[rank]), dtype=np.int64)
    loads = [int(kv[p].sum()) for p in parts]
    lengths = full.context_lengths[mine]
    pages = [int(math.ceil(int(n) / 16)) for n in lengths]
    num_blocks = sum(pages)
    width = max(pages)
    tables = np.full((len(mine), width), -1, dtype=np.int32)
    perm = np.random.default_rng(1 + rank).permutation(num_blocks)
    c = 0
    for i, n in enumerate(pages):
        tables[i, :n] = perm[c : c + n]
        c += n
    g = torch.Generator(device=device).manual_seed(11 + rank)
    key = torch.empty((num_blocks, 1, 16, 16, 128), device=device, dtype=torch.bfloat16)
    value = torch.empty_like(key)
    fill_random(key, g)
    fill_random(value, g)
    q = torch.empty((len(mine), 16, 128), device=device, dtype=torch.bfloat16)
    fill_random(q, g)
    t_tables = torch.from_numpy(tables).to(device)
    t_lengths = torch.from_numpy(lengths.astype(np.int32)).to(device)
    backend = rb.B200PagedAttention(device, torch.bfloat16, 128, 16)
    ms = time_region(lambda: backend(q, key[:, 0], value[:, 0], t_tables, t_lengths), steps,
                     warmup, device)
    step_bytes = decode_bytes(lengths, 16, 16, 128, 2)
    peak, kind = measured_peak()
    gbs = step_bytes / (ms / 1e3) / 1e9
    return {
        "workload": "configs[4]: SHARED layout, Pareto(1.5) ctx in [1024, 32768], 64 rows/GPU, "
                    "split-KV, LPT by KV bytes across ranks",
        "rows": int(len(mine)), "sum_ctx": int(lengths.sum()), "max_ctx": int(lengths.max()),
        "ms_per_step": round(ms, 4), "value": round(gbs, 1), "unit": "GB/s",
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "peak_kind": kind},
        "rank_kv_bytes_max_over_mean": round(max(loads) / (sum(loads) / len(loads)), 4),
        "errors": backend.check_errors(),
    }


def shared_extra(device, steps, warmup, rank):
    """Prefix-cached decode (configs[1] geometry): 256 rows in 16 groups of 16
    that share a system prompt of U[1024, 4096] tokens (the same physical
    pages, as prefix caching hands out), each row then its own
    lognormal(median 512, sigma 0.6) suffix in [16, 4096]. Times the
    shared-prefix path against the plain decode kernel on the same inputs."""
    import torch

    import vllm_rlt_b200 as rb
    from vllm_rlt_b200.kernels.paged_attention import decode_bytes

    page, hkv, d = 16, 16, 128
    rng = np.random.default_rng(21)
    groups, per_group = 16, 16
    prompt = (rng.integers(1024, 4097, size=groups) // page) * page
    suffix = np.clip(np.exp(rng.normal(np.log(512), 0.6, size=groups * per_group)), 16, 4096)
    suffix = suffix.astype(np.int64)
    lengths = np.repeat(prompt, per_group) + suffix
    shared_pages = prompt // page
    own_pages = [int(math.ceil(int(n) / page)) for n in suffix]
    num_blocks = int(shared_pages.sum() + sum(own_pages) + groups * per_group)
    width = int(max(int(math.ceil(int(n) / page)) for n in lengths))
    perm = rng.permutation(num_blocks)
    tables = np.full((groups * per_group, width), -1, dtype=np.int32)
    c = 0
    group_pages = []
    for gi in range(groups):
        group_pages.append(perm[c : c + shared_pages[gi]])
        c += shared_pages[gi]
    for r in range(groups * per_group):
        gi = r // per_group
        n_total = int(math.ceil(int(lengths[r]) / page))
        tables[r, : shared_pages[gi]] = group_pages[gi]
        extra = n_total - shared_pages[gi]
        tables[r, shared_pages[gi] : n_total] = perm[c : c + extra]
        c += extra
    g = torch.Generator(device=device).manual_seed(31 + rank)
    key = torch.empty((num_blocks, 1, page, hkv, d), device=device, dtype=torch.bfloat16)
    value = torch.empty_like(key)
    fill_random(key, g)
    fill_random(value, g)
    q = torch.empty((len(lengths), hkv, d), device=device, dtype=torch.bfloat16)
    fill_random(q, g)
    t_tables = torch.from_numpy(tables).to(device)
    t_lengths = torch.from_numpy(lengths.astype(np.int32)).to(device)
    import time as _time
    t0 = _time.perf_counter()
    plan = rb.plan_shared_prefix(tables, lengths, page, hkv, hkv, device)
    plan_ms = (_time.perf_counter() - t0) * 1e3
    backend = rb.B200PagedAttention(device, torch.bfloat16, d, page)
    ms_shared = time_region(
        lambda: rb.paged_attention_shared(q, key[:, 0], value[:, 0], t_tables, plan), steps,
        warmup, device)
    ms_plain = time_region(lambda: backend(q, key[:, 0], value[:, 0], t_tables, t_lengths), steps,
                           warmup, device)
    logical = decode_bytes(lengths, page, hkv, d, 2)
    read = plan.read_tokens * hkv * d * 2 * 2
    peak, kind = measured_peak()
    return {
        "workload": "configs[1] geometry with prefix caching: 256 rows = 16 groups x 16 sharing a "
                    "U[1024,4096]-token prompt, own suffix lognormal(512, 0.6) in [16, 4096]",
        "rows": int(len(lengths)), "sum_ctx": int(lengths.sum()),
        "kv_rows_read_over_logical": round(plan.read_tokens / plan.logical_tokens, 4),
        "ms_per_step": round(ms_shared, 4), "ms_per_step_plain_decode": round(ms_plain, 4),
        "speedup_vs_plain_decode": round(ms_plain / ms_shared, 3),
        "value": round(logical / (ms_shared / 1e3) / 1e9, 1),
        "unit": "GB/s (logical: every row's K/V counted, as a per-row decode reads it)",
        "hbm": {"achieved": round(read / (ms_shared / 1e3) / 1e9, 1), "peak": peak,
                "unit": "GB/s", "frac": round(read / (ms_shared / 1e3) / 1e9 / peak, 4),
                "peak_kind": kind, "bytes": "K/V token rows the plan reads, once per group"},
        "plan_ms_host": round(plan_ms, 2), "chunk_tokens": plan.chunk_tokens,
        "errors": backend.check_errors(),
    }


def ouro_extra(device, steps, warmup, rank, world=1, requests=64):
    """random-init Ouro-1.4B-shaped mixed-depth decode. 64 resident
    requests per GPU (LAST-EXITED needs ~1.6 GB of KV per request at 4 planes
    x 24 layers, so 512 requests are reached at 8 GPUs), contexts uniform in
    [256, 4096], per-token exit depth uniform in {1..4}; one step = one
    CUDA-graph replay of the recurrent core at every request's own depth.

    With several GPUs every rank is one request-sharded replica, and each step
    also runs the single front-end's exchange: an NCCL all-gather over NVLink
    of every rank's sampled tokens and exit flags, copied to pinned host
    memory without a sync (the front-end reads step t's tokens while step
    t + 1 runs). The job's rate is the tokens of all ranks over the slowest
    rank's device time."""
    import torch
    import torch.distributed as dist

    from vllm_rlt_b200.ouro import (DecodeScheduler, OuroDecoder, OuroShape, OuroWeights,
                                    decode_bytes_per_pass)
    from vllm_rlt_b200.replicas import gather_step_outputs, max_over_ranks

    rng = np.random.default_rng(50)  # same request mix on every rank (weak scaling)
    shape = OuroShape()
    ctx = rng.integers(256, 4097, size=requests).astype(np.int64)
    exits = rng.integers(0, 4, size=(requests, 4 * (steps + warmup) + 8))
    weights = OuroWeights(shape, device, torch.bfloat16, seed=rank)
    dec = OuroDecoder(shape, weights, ctx + steps + warmup + 8, device, torch.bfloat16,
                      seed=rank)
    g = torch.Generator(device=device).manual_seed(60 + rank)
    for pool in (dec.key_cache, dec.value_cache):  # synthetic history for every plane
        flat = pool.view(-1)
        for s0 in range(0, flat.numel(), 1 << 30):
            flat[s0 : s0 + (1 << 30)].normal_(generator=g)
    sched = DecodeScheduler(dec, ctx, lambda slot, i: int(exits[slot, i]))
    front = world > 1 and dist.is_initialized()
    seen = [torch.empty((world, requests), dtype=torch.int64, pin_memory=True) for _ in range(2)]

    def step(i):
        exiting = sched.prepare()
        dec.run()
        if front:
            tokens, _flags = gather_step_outputs(dec.tokens, dec.exit_mask)
            seen[i & 1].copy_(tokens, non_blocking=True)
        sched.advance(exiting)

    exiting = sched.prepare()
    dec.capture()
    dec.run()
    sched.advance(exiting)
    for i in range(warmup):
        step(i)
    torch.cuda.synchronize(device)
    if front:
        dist.barrier(device_ids=[device.index])
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    generated0 = sched.generated
    step_bytes = 0
    a.record()
    for i in range(steps):
        step_bytes += decode_bytes_per_pass(shape, sched.pos + 1)
        step(i)
    b.record()
    torch.cuda.synchronize(device)
    ms = a.elapsed_time(b)
    tokens = sched.generated - generated0
    (job_ms,), job_tokens = max_over_ranks([ms], float(tokens), device=device)
    errors = dec.attention.check_errors()
    peak, kind = measured_peak()
    gbs = step_bytes / (ms / 1e3) / 1e9
    kv_gb = (dec.key_cache.numel() + dec.value_cache.numel()) * 2 / 1e9
    del dec, weights
    torch.cuda.empty_cache()
    job_tok_s = job_tokens / (job_ms / 1e3)
    return {
        "workload": "configs[2]: Ouro-1.4B-shaped (24 layers x 4 loops, 2048 hidden, 16x128 "
                    "heads, SwiGLU 5632, vocab 49152, RoPE 1e4, bf16, random init), 64 requests "
                    "per GPU, ctx U[256,4096], exit depth U{1..4}, LAST-EXITED, graph-captured step",
        "n_gpus": world,
        "job_tok_s": round(job_tok_s, 1),
        "tok_s_per_gpu": round(job_tok_s / world, 1),
        "tok_s_rank0": round(tokens / (ms / 1e3), 1),
        "tokens": int(job_tokens), "steps": steps, "ms_per_step": round(job_ms / steps, 3),
        "timing": "CUDA events per rank, max over ranks; tokens summed over ranks",
        "front_end_gather": ("NCCL all-gather of sampled tokens + exit flags every step, "
                             "async copy to pinned host") if front else None,
        "kv_pool_gb": round(kv_gb, 1),
        "hbm": {"achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                "frac": round(gbs / peak, 4), "peak_kind": kind,
                "bytes": "per pass: every layer's K/V of every row's context + core weights"},
        "errors": errors,
    }


def kernels_extra(device, steps, warmup):
    """Every auxiliary kernel of the path once at a representative size, timed
    with CUDA events (median of ``steps`` launches after ``warmup``): the
    algorithmic bytes each moves, and GB/s against the copy peak. Sizes: Ouro
    geometry (24 layers, 16 KV heads x 128, page 16, 4 planes, hidden 2048,
    SwiGLU 5632), bf16; a 2048-token prefill chunk for the page write and the
    per-row glue, 512 exiting tokens for the exit copy, a 512-row routing
    bank, 256 Ouro-shaped blocks for the PD page transport (same GPU)."""
    import torch

    import vllm_rlt_b200 as rb
    from vllm_rlt_b200.kernels import ouro_ops
    from vllm_rlt_b200.pd import PageTransport

    g = torch.Generator(device=device).manual_seed(5)
    bf = torch.bfloat16
    layers, hkv, d, page, planes, hidden, inter = 24, 16, 128, 16, 4, 2048, 5632
    rng = np.random.default_rng(5)
    results = {}
    peak, kind = measured_peak()

    reps = 20

    def timed(name, fn, nbytes, note, graph=True):
        # `reps` launches back to back -- captured in one CUDA graph, so the
        # events see device time, not the host's launch rate -- per timing
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(device)
        if graph:
            side = torch.cuda.Stream(device)
            side.wait_stream(torch.cuda.current_stream(device))
            with torch.cuda.stream(side):
                fn()
            torch.cuda.current_stream(device).wait_stream(side)
            torch.cuda.synchronize(device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for _ in range(reps):
                    fn()

            def run():
                g.replay()
        else:
            def run():
                for _ in range(reps):
                    fn()
        run()
        torch.cuda.synchronize(device)
        times = []
        for _ in range(max(steps, 1)):
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            run()
            b.record()
            b.synchronize()
            times.append(a.elapsed_time(b) / reps)
        us = statistics.median(times) * 1e3
        gbs = nbytes / (us / 1e6) / 1e9
        results[name] = {"us": round(us, 2), "bytes": int(nbytes), "gb_s": round(gbs, 1),
                         "frac_of_peak": round(gbs / peak, 4), "what": note}

    # pool: 1,200 blocks of 24 layers (K and V: 3.5 GB)
    blocks = 1200
    kc = torch.empty((blocks, layers, page, hkv, d), device=device, dtype=bf)
    vc = torch.empty_like(kc)
    fill_random(kc, g)
    fill_random(vc, g)
    row_bytes = hkv * d * 2

    # KV page write: a 2048-token chunk into one layer
    n = 2048
    slots = torch.from_numpy(rng.permutation(blocks * page)[:n]).to(device)
    wb, wo = slots // page, slots % page
    k = torch.randn((n, hkv, d), generator=g, device=device).to(bf)
    v = torch.randn_like(k)
    timed("kv_write_kernel", lambda: rb.write_kv(kc, vc, 3, wb, wo, k, v), 2 * 2 * n * row_bytes,
          "2048 rows x (K, V) of 16x128 bf16 into one layer: read + write")

    # exit copy: 512 tokens leaving at depth 0 -> planes 1..3, all 24 layers;
    # slot s owns one page per plane, tokens at distinct (page, offset)
    exiting = 512
    tables = np.zeros((exiting, planes, 1), dtype=np.int32)
    for s_ in range(exiting):
        for pl in range(planes):
            tables[s_, pl, 0] = (s_ // page) * planes + pl
    tables_t = torch.from_numpy(tables).to(device)
    desc = torch.zeros((exiting, 3), dtype=torch.int64)
    desc[:, 0] = torch.arange(exiting)
    desc[:, 2] = torch.arange(exiting) % page
    desc_t = desc.to(device)
    timed("finalize_kernel", lambda: rb.finalize(desc_t, tables_t, kc, vc),
          exiting * 2 * layers * row_bytes * (1 + (planes - 1)),
          "512 exiting tokens, depth 0 -> 3 deeper planes, 24 layers, K and V: "
          "each source row read once, written 3 times")

    # routing metadata: a 512-row bank over resident tables [512, 4, 256]
    rows, width = 512, 256
    res_tables = torch.from_numpy(rng.integers(0, blocks, size=(rows, planes, width),
                                               dtype=np.int32)).to(device)
    mdesc = torch.zeros((rows, 3), dtype=torch.int64)
    mdesc[:, 0] = torch.arange(rows)
    mdesc[:, 1] = torch.from_numpy(rng.integers(0, planes, size=rows))
    mdesc[:, 2] = torch.from_numpy(rng.integers(0, width * page, size=rows))
    mdesc_t = mdesc.to(device)
    i64 = dict(device=device, dtype=torch.int64)
    outs = [torch.empty(rows, **i64) for _ in range(2)]
    lens = torch.empty(rows, device=device, dtype=torch.int32)
    ob, oo = torch.empty(rows, **i64), torch.empty(rows, **i64)
    out_tables = torch.empty((rows, width), device=device, dtype=torch.int32)
    timed("metadata_kernel",
          lambda: rb.metadata(mdesc_t, res_tables, outs[0], outs[1], lens, ob, oo, out_tables,
                              rows, rows, page, planes, width),
          rows * (24 + 4 * width + 4 * width + 8 * 4 + 4),
          "512-row bank: descriptor, the row's plane table read and copied, 4 int64 + 1 int32 "
          "outputs per row")

    # resident hidden-state gather / scatter: 512 rows x 2048 bf16
    pool = torch.randn((rows, hidden), generator=g, device=device).to(bf)
    perm_slots = torch.from_numpy(rng.permutation(rows)).to(device)
    hid = torch.empty((rows, hidden), device=device, dtype=bf)
    timed("gather_kernel", lambda: rb.gather(pool, perm_slots, hid, rows, rows),
          2 * rows * hidden * 2, "512 rows x 2048 bf16: read + write")
    timed("scatter_kernel", lambda: rb.scatter(hid, perm_slots, pool, rows),
          2 * rows * hidden * 2, "512 rows x 2048 bf16: read + write")

    # packed-prefill metadata: stage 64K int64 values, expand 2048 tokens
    vals = 1 << 16
    src = torch.from_numpy(rng.integers(0, 1000, size=vals)).pin_memory()
    t64 = torch.empty(vals, **i64)
    t32 = torch.empty(vals, device=device, dtype=torch.int32)
    timed("stage_kernel", lambda: rb.stage_prefill(src, t64, t32, vals),
          vals * (8 + 8 + 4), "65,536 int64 from mapped pinned host memory -> int64 + int32")
    pos = torch.from_numpy(rng.integers(0, width * page, size=n)).to(device)
    seqs = torch.from_numpy(rng.integers(0, 16, size=n)).to(device)
    ptab = torch.from_numpy(rng.integers(0, blocks, size=(16, width), dtype=np.int32)).to(device)
    eb, eo = torch.empty(n, **i64), torch.empty(n, **i64)
    timed("expand_kernel", lambda: rb.expand_prefill(pos, seqs, ptab, eb, eo, n, width, page),
          n * (8 + 8 + 4 + 8 + 8), "2048 tokens: position, sequence, table entry in; block, "
                                   "offset out")

    # RoPE + page write: 2048 rows of fused qkv [2048, (16 + 32) x 128]
    qkv = torch.randn((n, 48 * d), generator=g, device=device).to(bf)
    rpos = torch.from_numpy(rng.integers(0, 4096, size=n)).to(device)
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, d, 2, device=device, dtype=torch.float32) / d))
    timed("rope_write_kernel",
          lambda: ouro_ops.rope_write_kv(qkv, rpos, inv_freq, kc, vc, 5, wb, wo, 16, 16, d),
          n * (48 * d * 2 + 16 * d * 2 + 2 * row_bytes + 8 * 3),
          "2048 rows: qkv read, rotated q written, rotated k and v written into the pages")

    # paired RMSNorm with residual, SwiGLU
    x = torch.randn((n, hidden), generator=g, device=device).to(bf)
    res = torch.randn_like(x)
    w1 = torch.ones(hidden, device=device, dtype=bf)
    timed("rms_norm_vec_kernel",
          lambda: ouro_ops.rms_norm(x, w1, 1e-6, residual=res, weight2=w1),
          n * hidden * 2 * 4, "2048 x 2048 bf16: x and residual read, two normed outputs written")
    gu = torch.randn((n, 2 * inter), generator=g, device=device).to(bf)
    timed("silu_mul_vec_kernel", lambda: ouro_ops.silu_mul(gu, inter),
          n * inter * 2 * 3, "2048 x 11264 bf16 read, 2048 x 5632 written")

    # PD page transport on one GPU: 256 whole Ouro-shaped blocks, 4 planes
    del k, v, qkv, gu, x, res
    src_k, src_v = kc[:512], vc[:512]
    dst_k, dst_v = kc[512:1024], vc[512:1024]
    transport = PageTransport(src_k, src_v, page, transfer_chunk_bytes=1 << 30,
                              max_inflight_bytes=1 << 36)
    transport.connect("peer", dst_k, dst_v)
    local = [list(map(int, rng.permutation(512)[:64])) for _ in range(planes)]
    remote = [list(map(int, rng.permutation(512)[:64])) for _ in range(planes)]

    def transfer():
        transport.poll()  # retire the previous (completed) transfer from the budget
        transport.stream.wait_stream(torch.cuda.current_stream(device))
        if not transport.submit("t", 0, "peer", local, remote, 0, 64 * page):
            raise RuntimeError("the PD transfer was refused by the in-flight budget")
        torch.cuda.current_stream(device).wait_stream(transport.stream)

    timed("copy_segments_kernel", transfer,
          2 * planes * 64 * 2 * layers * page * row_bytes,
          "256 whole blocks (4 planes x 64 pages, 24 layers, K and V): read + write",
          graph=False)
    torch.cuda.synchronize(device)
    transport.poll()
    errors = rb.B200PagedAttention(device, bf, d, page).check_errors()
    del kc, vc
    torch.cuda.empty_cache()
    return {"kernels": results, "peak": peak, "peak_kind": kind, "errors": errors,
            "timing": f"CUDA events around {reps} back-to-back launches (one captured CUDA "
                      "graph; the PD transfer, which stages host descriptors, eagerly), "
                      "per launch, median over steps; inputs under 126 MB stay in L2"}


# ------------------------------------------------------------------ ours


def run_ours(args):
    import torch
    import torch.distributed as dist

    import vllm_rlt_b200 as rb
    from vllm_rlt_b200 import workloads
    from vllm_rlt_b200.kernels.paged_attention import decode_bytes

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=device)

    if args.workload != "decode":
        if args.workload == "prefill":
            res = prefill_extra(device, args.steps, args.warmup, rank)
        elif args.workload == "ouro":
            res = ouro_extra(device, args.steps, args.warmup, rank, world)
        elif args.workload == "shared":
            res = shared_extra(device, args.steps, args.warmup, rank)
        elif args.workload == "kernels":
            res = kernels_extra(device, args.steps, args.warmup)
        else:
            res = longctx_extra(device, args.steps, args.warmup, rank, world)
        if world > 1:
            dist.barrier(device_ids=[local])
            dist.destroy_process_group()
        if rank == 0:
            print(json.dumps({"workload_line": args.workload, "n_gpus": world, **res}), flush=True)
        return

    # Weak scaling: every rank serves a shard of the same shape (same context
    # lengths and tables); only the synthetic K/V contents differ per rank.
    plan = workloads.config2_plan(seed=0, rows=args.rows)
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    shape = (plan.num_blocks, 1, plan.page, plan.num_kv_heads, plan.head_dim)
    kpool = torch.empty(shape, device=device, dtype=torch.bfloat16)
    vpool = torch.empty_like(kpool)
    fill_random(kpool, g)
    fill_random(vpool, g)
    k_layer, v_layer = kpool[:, 0], vpool[:, 0]
    tables_np = plan.block_tables()
    tables = torch.from_numpy(tables_np).to(device)
    lengths = torch.from_numpy(plan.context_lengths).to(device)
    q = torch.randn((plan.num_rows, 16, 128), generator=g, device=device).to(torch.bfloat16)
    backend = rb.B200PagedAttention(device, torch.bfloat16, 128, plan.page)
    step_bytes = decode_bytes(plan.context_lengths, 16, 16, 128, 2, plan.page)
    # two kernels per call: the one-CTA work schedule (which also clears the
    # split counters) and the decode kernel, into which the split merge is fused
    launches_per_step = 2

    stream = torch.cuda.current_stream(device)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # ---- device-resident timing (value) + per-launch events (roofline)
    for _ in range(args.warmup):
        backend(q, k_layer, v_layer, tables, lengths)
    torch.cuda.synchronize(device)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize(device)
        t0.record(stream)
        for i in range(args.steps):
            starts[i].record(stream)
            out = backend(q, k_layer, v_layer, tables, lengths)
            ends[i].record(stream)
        t1.record(stream)
        torch.cuda.synchronize(device)
        barrier()
    elapsed_ms = t0.elapsed_time(t1)
    launch_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    errors = backend.check_errors()
    if errors:
        raise RuntimeError(f"kernel reported metadata errors: {errors}")

    # ---- end to end through the public API with host buffers. Every step
    # copies its own inputs from pinned host memory and reads its result
    # back; as a serving loop would, the copies run on the copy engines (one
    # stream per direction, double-buffered device inputs) while the previous
    # or next step's kernel runs.
    pin = dict(
        q=q.cpu().pin_memory(), tables=tables.cpu().pin_memory(),
        lengths=lengths.cpu().pin_memory(),
    )
    out_host = [torch.empty(out.shape, dtype=out.dtype, pin_memory=True) for _ in range(2)]
    h2d = sum(t.numel() * t.element_size() for t in pin.values())
    d2h = out_host[0].numel() * out_host[0].element_size()
    dev_in = [{k: torch.empty_like(v, device=device) for k, v in pin.items()} for _ in range(2)]
    h2d_stream = torch.cuda.Stream(device)
    d2h_stream = torch.cuda.Stream(device)
    landed = [torch.cuda.Event() for _ in range(2)]    # inputs of buffer b copied
    consumed = [torch.cuda.Event() for _ in range(2)]  # the kernel that read buffer b is done
    for e in consumed:
        e.record(stream)

    def e2e_step(i):
        b = i & 1
        with torch.cuda.stream(h2d_stream):
            h2d_stream.wait_event(consumed[b])
            for k, v in pin.items():
                dev_in[b][k].copy_(v, non_blocking=True)
            landed[b].record(h2d_stream)
        stream.wait_event(landed[b])
        o = backend(dev_in[b]["q"], k_layer, v_layer, dev_in[b]["tables"], dev_in[b]["lengths"])
        consumed[b].record(stream)
        with torch.cuda.stream(d2h_stream):
            d2h_stream.wait_event(consumed[b])
            out_host[b].copy_(o, non_blocking=True)
        o.record_stream(d2h_stream)

    for i in range(args.warmup):
        e2e_step(i)
    torch.cuda.synchronize(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(device)
    e0.record(stream)
    h2d_stream.wait_event(e0)
    d2h_stream.wait_event(e0)
    for i in range(args.steps):
        e2e_step(i)
    stream.wait_stream(d2h_stream)  # the last result is on the host
    e1.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms = e0.elapsed_time(e1)
    if not torch.equal(out_host[(args.steps - 1) & 1], out.cpu()):
        raise RuntimeError("end-to-end result differs from the device-resident one")

    # the same steps with every copy in series with the kernel, one stream
    def serial_step():
        for k, v in pin.items():
            dev_in[0][k].copy_(v, non_blocking=True)
        o = backend(dev_in[0]["q"], k_layer, v_layer, dev_in[0]["tables"], dev_in[0]["lengths"])
        out_host[0].copy_(o, non_blocking=True)

    serial_step()
    torch.cuda.synchronize(device)
    barrier()
    torch.cuda.synchronize(device)
    e0.record(stream)
    for _ in range(args.steps):
        serial_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    serial_ms = e0.elapsed_time(e1)

    # ---- max over ranks; bytes summed over ranks
    from vllm_rlt_b200.replicas import max_over_ranks

    (elapsed_ms, e2e_ms, serial_ms), job_bytes = max_over_ranks(
        [elapsed_ms, e2e_ms, serial_ms], float(step_bytes), device=device)
    value = job_bytes * args.steps / (elapsed_ms / 1e3) / 1e9
    e2e_value = job_bytes * args.steps / (e2e_ms / 1e3) / 1e9
    serial_value = job_bytes * args.steps / (serial_ms / 1e3) / 1e9
    peak, peak_kind = measured_peak()
    kernel_ms = statistics.mean(launch_ms)
    achieved = step_bytes / (kernel_ms / 1e3) / 1e9
    traffic = committed_traffic()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        host, fn, kind, label, threads = reference_cpu_sample(plan, 5.0)
        host.run(fn)
        reps, spent = 0, 0.0
        while spent < 12.0 and reps < 20:
            t_start = time.perf_counter()
            host.run(fn)
            spent += time.perf_counter() - t_start
            reps += 1
        cpu = {
            "value": round(host.bytes * reps / spent / 1e9, 3), "unit": "GB/s",
            "cores": threads, "kind": kind,
            "sample": (f"{len(host.rows)} of {plan.num_rows} rows (sum ctx {host.tokens}) x "
                       f"{reps} calls; {label}"),
            "cpu_model": cpu_model(), "host_threads": os.cpu_count(),
            "single_thread": single_thread_rate(plan, fn),
            "reference_kv_cpu": reference_kv_cpu(),
        }
        del host

    extras = {}
    if not args.no_extras:
        # free the decode pool first: the extras allocate their own pools
        del kpool, vpool, k_layer, v_layer
        torch.cuda.empty_cache()
        for name, fn in (("ouro", lambda: ouro_extra(device, 30, 3, rank, world)),
                         ("prefill", lambda: prefill_extra(device, 10, 3, rank)),
                         ("longctx", lambda: longctx_extra(device, 20, 5, rank, world)),
                         ("shared_prefix", lambda: shared_extra(device, 20, 5, rank))):
            try:
                extras[name] = fn()
            except Exception as error:  # reported, never silently dropped
                extras[name] = {"error": f"{type(error).__name__}: {error}"}
            torch.cuda.empty_cache()
        if rank == 0 and world == 1 and not args.no_cpu_baseline:
            # the reference's CPU path on samples of the prefill and long-context workloads
            for name, fn in (("prefill", prefill_cpu_baseline), ("longctx", longctx_cpu_baseline)):
                if "value" not in extras[name]:
                    continue
                try:
                    extras[name]["cpu_baseline"] = fn()
                except Exception as error:
                    extras[name]["cpu_baseline"] = {"error": f"{type(error).__name__}: {error}"}

    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(elapsed_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic",
        "pct_of_peak": round(100.0 * value / world / peak, 2),
        "config": decode_config(plan, world),
        "roofline": {
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "peak_kind": peak_kind,
            "kernel": "paged_decode_kernel (split merge fused) with its one-CTA work "
                      "schedule, CUDA events per call",
            "traffic": None if traffic is None else traffic.get("bytes_per_launch"),
        },
        "e2e": {
            "value": round(serial_value, 2),
            "unit": "GB/s",
            "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h),
            "copies": "each step's inputs H2D from pinned memory, the call, its result D2H, "
                      "in series on one stream, inside the timed region",
            "overlapped_value": round(e2e_value, 2),
            "overlapped": "the same steps with the copies on one stream per direction "
                          "overlapping the neighbouring steps' kernels; varies between runs "
                          "(host enqueue across three streams)",
        },
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if extras:
        line["extras"] = extras
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.workload == "reference-engine":  # host only
        print(json.dumps({"workload_line": "reference-engine", **reference_engine_cpu()}),
              flush=True)
        return
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "reference-triton":
        run_reference_triton(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
