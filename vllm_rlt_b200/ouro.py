"""Ouro-shaped looped-transformer decode on the B200 kernels (calling context).

This is the caller of the attention path, restated compactly so the path can
be measured end to end: the reference's Ouro model (vllm_rlt/models/ouro.py:
27-217) -- RMSNorm in fp32 (:33-36), RoPE with fp32 angles cast to the
activation dtype (:61-70, :73-75), attention = page write then paged attend
(:96-112), SwiGLU MLP (:115-123), the doubled residual norms of a decoder
layer (:136-147), the recurrent core of all layers + final norm + exit gate
(:209-217) -- and the runner's mixed-depth decode step with the CUDA-graph-
captured core (vllm_rlt/worker/model_runner.py:386-431,
vllm_rlt/worker/cuda_graph.py:43-122).

GEMMs stay on cuBLAS (torch.matmul); the page write, the depth/page
resolution, the decode attention and the LAST-EXITED exit copy run on the
sm_100a kernels of this package. Weights are random (normal, std 0.02, as the
reference's initialiser at models/ouro.py:183-191); no checkpoint is loaded.

One decode step advances every resident request by one recurrent pass at its
own depth: rows at depth 0 start a new token from its embedding, other rows
continue from their previous pass's hidden state; rows whose pass reaches
their exit depth copy their K/V into the deeper planes, go through the LM
head and sample (greedy) the next token. The step is one CUDA graph.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .kernels import ouro_ops
from .kernels.cache_ops import finalize, write_kv
from .kernels.paged_attention import B200PagedAttention
from .kernels.routing import metadata


@dataclass(frozen=True)
class OuroShape:
    """Ouro-1.4B geometry (vllm_rlt/models/config.py:14-40); the benchmark
    configuration uses rope_theta 10000."""

    vocab: int = 49152
    hidden: int = 2048
    intermediate: int = 5632
    layers: int = 24
    heads: int = 16
    kv_heads: int = 16
    head_dim: int = 128
    loops: int = 4
    rope_theta: float = 10000.0
    eps: float = 1e-6

    @classmethod
    def tiny(cls):
        return cls(vocab=97, hidden=128, intermediate=192, layers=2, heads=2, kv_heads=2,
                   head_dim=64, loops=4)


class OuroWeights:
    """Random-initialised weights with the reference's parameter roles; the
    q/k/v and gate/up projections are stored concatenated for one GEMM each."""

    def __init__(self, shape: OuroShape, device, dtype, seed: int = 0):
        g = torch.Generator(device=device).manual_seed(seed)
        std = 0.02

        def normal(*size):
            t = torch.empty(size, device=device, dtype=dtype)
            t.normal_(0.0, std, generator=g)
            return t

        def linear(out_features, in_features):
            # [out, in] like torch.nn.Linear.weight, held as the transposed view
            # of a contiguous [in, out] tensor: `x @ w.t()` then reads the
            # weights in the layout cuBLAS streams fastest at decode batch
            # sizes (24 layers' projections at 64 rows in one graph: 3.28 TB/s
            # against 3.00 TB/s for contiguous [out, in] weights)
            return normal(in_features, out_features).t()

        h, d = shape.hidden, shape.head_dim
        qkv = (shape.heads + 2 * shape.kv_heads) * d
        self.embed = normal(shape.vocab, h)
        self.wqkv = [linear(qkv, h) for _ in range(shape.layers)]
        self.wo = [linear(h, shape.heads * d) for _ in range(shape.layers)]
        self.wgu = [linear(2 * shape.intermediate, h) for _ in range(shape.layers)]
        self.wdown = [linear(h, shape.intermediate) for _ in range(shape.layers)]
        ones = torch.ones(h, device=device, dtype=dtype)
        # input, input_2, post_attention, post_attention_2 norms per layer
        self.norms = [[ones.clone() for _ in range(4)] for _ in range(shape.layers)]
        self.final_norm = ones.clone()
        self.gate_w = normal(1, h)
        self.gate_b = torch.zeros(1, device=device, dtype=dtype)
        self.lm_head = linear(shape.vocab, h)
        self.inv_freq = self.frequencies(shape, device)

    @staticmethod
    def frequencies(shape: OuroShape, device):
        """fp32 RoPE inverse frequencies (vllm_rlt/models/ouro.py:44-52)."""
        d = shape.head_dim
        return 1.0 / (shape.rope_theta ** (
            torch.arange(0, d, 2, dtype=torch.float32, device=device) / d))

    @classmethod
    def from_state_dict(cls, shape: OuroShape, state, device, dtype):
        """Weights of a reference ``OuroForCausalLM`` (its ``state_dict()``
        names, vllm_rlt/models/ouro.py:79-217), in this decoder's layout: q/k/v
        and gate/up concatenated, every projection held as the transposed view
        of a contiguous [in, out] tensor."""
        self = cls.__new__(cls)

        def get(name):
            return state[name].to(device=device, dtype=dtype)

        def linear(*names):
            weight = torch.cat([get(n) for n in names], dim=0)  # [out, in]
            return weight.t().contiguous().t()

        self.embed = get("model.embed_tokens.weight").contiguous()
        self.wqkv, self.wo, self.wgu, self.wdown, self.norms = [], [], [], [], []
        for i in range(shape.layers):
            p = f"model.layers.{i}."
            self.wqkv.append(linear(p + "self_attn.q_proj.weight", p + "self_attn.k_proj.weight",
                                    p + "self_attn.v_proj.weight"))
            self.wo.append(linear(p + "self_attn.o_proj.weight"))
            self.wgu.append(linear(p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight"))
            self.wdown.append(linear(p + "mlp.down_proj.weight"))
            self.norms.append([get(p + n + ".weight").contiguous() for n in (
                "input_layernorm", "input_layernorm_2", "post_attention_layernorm",
                "post_attention_layernorm_2")])
        self.final_norm = get("model.norm.weight").contiguous()
        self.gate_w = get("model.early_exit_gate.weight").reshape(1, shape.hidden).contiguous()
        self.gate_b = get("model.early_exit_gate.bias").reshape(1).contiguous()
        self.lm_head = linear("lm_head.weight")
        self.inv_freq = self.frequencies(shape, device)
        return self


def rms_norm(x, weight, eps):
    value = x.float()
    value = value * torch.rsqrt(value.square().mean(-1, keepdim=True) + eps)
    return weight * value.to(x.dtype)


def rotate_half(x):
    first, second = x.chunk(2, dim=-1)
    return torch.cat((-second, first), dim=-1)


class OuroDecoder:
    """Resident-slot mixed-depth decoder over a LAST-EXITED (or SHARED) pool.

    ``capacity[s]`` tokens are reserved per slot; pages for every plane are
    claimed up front (vllm_rlt/core/kv_cache_manager.py:253-293 without
    incremental growth) from a seeded permutation of the pool.
    """

    def __init__(self, shape: OuroShape, weights: OuroWeights, capacity, device, dtype,
                 layout: str = "last_exited", page: int = 16, seed: int = 0, fused: bool = True):
        self.shape, self.w = shape, weights
        self.fused = fused  # fused sm_100a glue kernels, or the plain torch expressions
        self.device, self.dtype, self.page = torch.device(device), dtype, page
        self.layout = layout
        self.planes = shape.loops if layout == "last_exited" else 1
        self.slots = len(capacity)
        self.capacity = np.asarray(capacity, dtype=np.int64)
        pages = (self.capacity + page - 1) // page
        self.width = int(pages.max())
        self.num_blocks = int(pages.sum()) * self.planes
        order = np.random.default_rng(seed).permutation(self.num_blocks)
        tables = np.zeros((self.slots, self.planes, self.width), dtype=np.int32)
        cursor = 0
        for s in range(self.slots):
            n = int(pages[s])
            for d in range(self.planes):
                tables[s, d, :n] = order[cursor : cursor + n]
                cursor += n
        self.tables_host = tables
        self.tables = torch.from_numpy(tables).to(self.device)
        pool = (self.num_blocks, shape.layers, page, shape.kv_heads, shape.head_dim)
        self.key_cache = torch.zeros(pool, device=self.device, dtype=dtype)
        self.value_cache = torch.zeros(pool, device=self.device, dtype=dtype)
        self.attention = B200PagedAttention(self.device, dtype, shape.head_dim, page)
        n = self.slots
        i64 = dict(device=self.device, dtype=torch.int64)
        # step inputs (written by the host each step) and per-slot state
        self.desc_core = torch.zeros((n, 3), **i64)
        self.desc_exit = torch.zeros((n, 3), **i64)
        self.exit_mask = torch.zeros(n, device=self.device, dtype=torch.bool)
        self.start_mask = torch.zeros(n, device=self.device, dtype=torch.bool)
        self.tokens = torch.zeros(n, **i64)
        self.hidden_state = torch.zeros((n, shape.hidden), device=self.device, dtype=dtype)
        # metadata produced on device by the routing kernel each step
        self.slot_ids = torch.zeros(n, **i64)
        self.positions = torch.zeros(n, **i64)
        self.lengths = torch.zeros(n, device=self.device, dtype=torch.int32)
        self.write_blocks = torch.zeros(n, **i64)
        self.write_offsets = torch.zeros(n, **i64)
        self.row_tables = torch.zeros((n, self.width), device=self.device, dtype=torch.int32)
        self.graph = None
        self.gate = None

    # ------------------------------------------------------------ the model

    def rope(self, positions):
        angles = positions.float().unsqueeze(-1) * self.w.inv_freq
        angles = torch.cat((angles, angles), dim=-1)
        return angles.cos().to(self.dtype).unsqueeze(1), angles.sin().to(self.dtype).unsqueeze(1)

    def layer(self, index, hidden, cos, sin):
        s, w = self.shape, self.w
        norms = w.norms[index]
        x = rms_norm(hidden, norms[0], s.eps)
        qkv = x @ w.wqkv[index].t()
        n = hidden.shape[0]
        q = qkv[:, : s.heads * s.head_dim].view(n, s.heads, s.head_dim)
        k = qkv[:, s.heads * s.head_dim : (s.heads + s.kv_heads) * s.head_dim].view(
            n, s.kv_heads, s.head_dim)
        v = qkv[:, (s.heads + s.kv_heads) * s.head_dim :].view(n, s.kv_heads, s.head_dim)
        q = q * cos + rotate_half(q) * sin
        k = k * cos + rotate_half(k) * sin
        write_kv(self.key_cache, self.value_cache, index, self.write_blocks, self.write_offsets,
                 k, v)
        attn = self.attention(q, self.key_cache[:, index], self.value_cache[:, index],
                              self.row_tables, self.lengths)
        out = attn.reshape(n, -1) @ w.wo[index].t()
        hidden = hidden + rms_norm(out, norms[1], s.eps)
        gu = rms_norm(hidden, norms[2], s.eps) @ w.wgu[index].t()
        gate, up = gu[:, : s.intermediate], gu[:, s.intermediate :]
        mlp = (torch.nn.functional.silu(gate) * up) @ w.wdown[index].t()
        return hidden + rms_norm(mlp, norms[3], s.eps)

    def layer_fused(self, index, hidden, x, next_norm):
        """The same layer with the glue on fused kernels: the residual add folded
        into the norm before it, and each norm of the residual stream paired in
        one launch with the norm that reads its output (post-attention -> MLP
        input; post-MLP -> ``next_norm``, the next layer's input norm or the
        final norm); RoPE fused with the page write; one SwiGLU kernel. ``x`` is
        this layer's normed input; returns (hidden, next_norm(hidden))."""
        s, w = self.shape, self.w
        norms = w.norms[index]
        qkv = x @ w.wqkv[index].t()
        q = ouro_ops.rope_write_kv(qkv, self.positions, w.inv_freq, self.key_cache,
                                   self.value_cache, index, self.write_blocks,
                                   self.write_offsets, s.heads, s.kv_heads, s.head_dim)
        attn = self.attention(q, self.key_cache[:, index], self.value_cache[:, index],
                              self.row_tables, self.lengths)
        out = attn.reshape(hidden.shape[0], -1) @ w.wo[index].t()
        hidden, x2 = ouro_ops.rms_norm(out, norms[1], s.eps, residual=hidden, weight2=norms[2])
        mlp = ouro_ops.silu_mul(x2 @ w.wgu[index].t(), s.intermediate) @ w.wdown[index].t()
        return ouro_ops.rms_norm(mlp, norms[3], s.eps, residual=hidden, weight2=next_norm)

    def core(self, hidden):
        """One recurrent pass: all layers, final norm, exit gate
        (vllm_rlt/models/ouro.py:209-217)."""
        layers = self.shape.layers
        if self.fused:
            x = ouro_ops.rms_norm(hidden, self.w.norms[0][0], self.shape.eps)
            for index in range(layers):
                nxt = self.w.norms[index + 1][0] if index + 1 < layers else self.w.final_norm
                hidden, x = self.layer_fused(index, hidden, x, nxt)
            hidden = x  # the final norm of the last layer's output
        else:
            cos, sin = self.rope(self.positions)
            for index in range(layers):
                hidden = self.layer(index, hidden, cos, sin)
            hidden = rms_norm(hidden, self.w.final_norm, self.shape.eps)
        gate = torch.sigmoid(hidden @ self.w.gate_w.t() + self.w.gate_b).squeeze(-1)
        return hidden, gate

    # ------------------------------------------------------------- the step

    def step_body(self):
        """Device work of one decode step (captured as one graph)."""
        n = self.slots
        metadata(self.desc_core, self.tables, self.slot_ids, self.positions, self.lengths,
                 self.write_blocks, self.write_offsets, self.row_tables, n, n, self.page,
                 self.planes, self.width)
        start = torch.nn.functional.embedding(self.tokens, self.w.embed)
        hidden = torch.where(self.start_mask.unsqueeze(-1), start, self.hidden_state)
        hidden, gate = self.core(hidden)
        if self.planes > 1:
            finalize(self.desc_exit, self.tables, self.key_cache, self.value_cache)
        logits = hidden @ self.w.lm_head.t()
        sampled = torch.argmax(logits, dim=-1)
        self.tokens.copy_(torch.where(self.exit_mask, sampled, self.tokens))
        self.hidden_state.copy_(hidden)
        self.gate = gate

    def capture(self, warmup: int = 2):
        """Capture step_body into a CUDA graph (warm-up on a side stream first,
        as vllm_rlt/worker/cuda_graph.py:95-112)."""
        # Warm-up passes rewrite the same KV slots the first real step writes,
        # but they also advance the sampled tokens and hidden states: restore.
        saved = (self.tokens.clone(), self.hidden_state.clone())
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                self.step_body()
        torch.cuda.current_stream(self.device).wait_stream(stream)
        torch.cuda.synchronize(self.device)
        self.tokens.copy_(saved[0])
        self.hidden_state.copy_(saved[1])
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.step_body()

    def run(self, graphed: bool = True):
        if graphed:
            if self.graph is None:
                raise RuntimeError("capture() before run(graphed=True)")
            self.graph.replay()
        else:
            self.step_body()


class DecodeScheduler:
    """Host side of the mixed-depth loop: per slot the current position,
    depth and the exit depth of the current token (a trace, like the
    reference's ExitConfig("trace"), vllm_rlt/config.py:82-97)."""

    def __init__(self, decoder: OuroDecoder, context_lengths, exit_trace):
        self.dec = decoder
        self.pos = np.asarray(context_lengths, dtype=np.int64).copy()  # next token's position
        self.depth = np.zeros(decoder.slots, dtype=np.int64)
        self.trace = exit_trace  # callable (slot, token_index) -> exit depth 0..loops-1
        self.count = np.zeros(decoder.slots, dtype=np.int64)
        self.exit_depth = np.array([self.trace(s, 0) for s in range(decoder.slots)], dtype=np.int64)
        n = decoder.slots
        # A ring of pinned descriptor banks: the host fills bank i while the
        # GPU may still be copying bank i-1; a bank is reused only after the
        # event recorded behind its copies has completed.
        self.banks = [
            dict(core=torch.zeros((n, 3), dtype=torch.int64).pin_memory(),
                 exit=torch.zeros((n, 3), dtype=torch.int64).pin_memory(),
                 emask=torch.zeros(n, dtype=torch.bool).pin_memory(),
                 smask=torch.zeros(n, dtype=torch.bool).pin_memory(),
                 event=None)
            for _ in range(3)
        ]
        self.bank = 0
        self.generated = 0

    def prepare(self):
        """Write this step's descriptors (non-blocking H2D); returns the
        number of tokens the step completes."""
        dec, n = self.dec, self.dec.slots
        slots = np.arange(n, dtype=np.int64)
        exiting = self.depth == self.exit_depth
        if (self.pos >= dec.capacity).any():
            raise RuntimeError("a request outgrew its reserved capacity")
        core = np.stack([slots, self.depth, self.pos], axis=1)
        exit_desc = np.stack([slots, np.where(exiting, self.depth, dec.planes - 1), self.pos], axis=1)
        bank = self.banks[self.bank]
        self.bank = (self.bank + 1) % len(self.banks)
        if bank["event"] is not None:
            bank["event"].synchronize()
        bank["core"].numpy()[:] = core
        bank["exit"].numpy()[:] = exit_desc
        bank["emask"].numpy()[:] = exiting
        bank["smask"].numpy()[:] = self.depth == 0
        dec.desc_core.copy_(bank["core"], non_blocking=True)
        dec.desc_exit.copy_(bank["exit"], non_blocking=True)
        dec.exit_mask.copy_(bank["emask"], non_blocking=True)
        dec.start_mask.copy_(bank["smask"], non_blocking=True)
        bank["event"] = torch.cuda.Event()
        bank["event"].record(torch.cuda.current_stream(dec.device))
        return exiting

    def advance(self, exiting):
        self.count[exiting] += 1
        self.generated += int(exiting.sum())
        self.pos[exiting] += 1
        self.depth[~exiting] += 1
        self.depth[exiting] = 0
        for s in np.nonzero(exiting)[0]:
            self.exit_depth[s] = self.trace(int(s), int(self.count[s]))


def decode_bytes_per_pass(shape: OuroShape, lengths, elem_bytes: int = 2) -> int:
    """HBM bytes of one recurrent pass: every layer's K/V of every row's
    context read once, plus all core weights read once."""
    kv = int(np.asarray(lengths, dtype=np.int64).sum()) * shape.kv_heads * shape.head_dim * 2
    layer_params = ((shape.heads + 2 * shape.kv_heads) * shape.head_dim * shape.hidden
                    + shape.hidden * shape.heads * shape.head_dim
                    + 3 * shape.hidden * shape.intermediate)
    return (kv * shape.layers + layer_params * shape.layers) * elem_bytes


__all__ = ["OuroShape", "OuroWeights", "OuroDecoder", "DecodeScheduler", "decode_bytes_per_pass",
           "rms_norm", "rotate_half"]
