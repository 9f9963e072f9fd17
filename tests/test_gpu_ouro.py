"""End-to-end mixed-depth decode of an Ouro-shaped model on the B200 kernels.

An independent dense reference (torch, fp32) keeps every (slot, plane,
layer) K/V history as a dense tensor, attends with an explicit softmax over
positions 0..pos of the row's plane, and copies an exiting token's K/V into
the deeper planes (LAST-EXITED, vllm_rlt/core/kv_cache_manager.py:588-614;
the dense-model check of the reference is tests/test_ouro.py:34-96). Both run
the same schedule of mixed depths from the same initial pool.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from vllm_rlt_b200.ouro import (DecodeScheduler, OuroDecoder, OuroShape, OuroWeights, rms_norm,
                                rotate_half)

pytestmark = pytest.mark.gpu


class DenseOuro:
    def __init__(self, dec: OuroDecoder):
        self.dec, self.s, self.w = dec, dec.shape, dec.w
        page = dec.page
        self.k, self.v = {}, {}
        for slot in range(dec.slots):
            for plane in range(dec.planes):
                ids = torch.from_numpy(dec.tables_host[slot, plane].astype(np.int64)).cuda()
                # [pages, L, page, Hkv, D] -> [L, pages*page, Hkv, D]
                k = dec.key_cache[ids].permute(1, 0, 2, 3, 4).reshape(self.s.layers, -1, self.s.kv_heads, self.s.head_dim)
                v = dec.value_cache[ids].permute(1, 0, 2, 3, 4).reshape(self.s.layers, -1, self.s.kv_heads, self.s.head_dim)
                self.k[slot, plane] = k.float().clone()
                self.v[slot, plane] = v.float().clone()
        self.tokens = torch.zeros(dec.slots, dtype=torch.int64, device="cuda")
        self.hidden_state = torch.zeros((dec.slots, self.s.hidden), device="cuda")
        del page

    def plane(self, depth):
        return depth if self.dec.layout == "last_exited" else 0

    def step(self, depth, pos, exiting):
        s, w = self.s, self.w
        n = self.dec.slots
        start = torch.nn.functional.embedding(self.tokens, w.embed.float())
        mask = torch.from_numpy(depth == 0).cuda().unsqueeze(-1)
        hidden = torch.where(mask, start, self.hidden_state)
        positions = torch.from_numpy(pos).cuda()
        angles = positions.float().unsqueeze(-1) * w.inv_freq
        angles = torch.cat((angles, angles), dim=-1)
        cos, sin = angles.cos().unsqueeze(1), angles.sin().unsqueeze(1)
        for layer in range(s.layers):
            norms = [x.float() for x in w.norms[layer]]
            x = rms_norm(hidden, norms[0], s.eps)
            qkv = x @ w.wqkv[layer].float().t()
            q = qkv[:, : s.heads * s.head_dim].view(n, s.heads, s.head_dim)
            k = qkv[:, s.heads * s.head_dim : (s.heads + s.kv_heads) * s.head_dim].view(n, s.kv_heads, s.head_dim)
            v = qkv[:, (s.heads + s.kv_heads) * s.head_dim :].view(n, s.kv_heads, s.head_dim)
            q = q * cos + rotate_half(q) * sin
            k = k * cos + rotate_half(k) * sin
            outs = []
            for r in range(n):
                plane = self.plane(int(depth[r]))
                p = int(pos[r])
                self.k[r, plane][layer, p] = k[r]
                self.v[r, plane][layer, p] = v[r]
                keys = self.k[r, plane][layer, : p + 1]  # [T, Hkv, D]
                vals = self.v[r, plane][layer, : p + 1]
                group = s.heads // s.kv_heads
                keys = keys.repeat_interleave(group, dim=1)
                vals = vals.repeat_interleave(group, dim=1)
                scores = torch.einsum("hd,thd->ht", q[r], keys) / s.head_dim ** 0.5
                outs.append(torch.einsum("ht,thd->hd", scores.softmax(-1), vals))
            attn = torch.stack(outs)
            out = attn.reshape(n, -1) @ w.wo[layer].float().t()
            hidden = hidden + rms_norm(out, norms[1], s.eps)
            gu = rms_norm(hidden, norms[2], s.eps) @ w.wgu[layer].float().t()
            gate, up = gu[:, : s.intermediate], gu[:, s.intermediate :]
            mlp = (torch.nn.functional.silu(gate) * up) @ w.wdown[layer].float().t()
            hidden = hidden + rms_norm(mlp, norms[3], s.eps)
        hidden = rms_norm(hidden, w.final_norm.float(), s.eps)
        if self.dec.layout == "last_exited":
            for r in np.nonzero(exiting)[0]:
                e, p = int(depth[r]), int(pos[r])
                for target in range(e + 1, self.dec.planes):
                    self.k[r, target][:, p] = self.k[r, e][:, p]
                    self.v[r, target][:, p] = self.v[r, e][:, p]
        sampled = torch.argmax(hidden @ w.lm_head.float().t(), dim=-1)
        ex = torch.from_numpy(exiting).cuda()
        self.tokens = torch.where(ex, sampled, self.tokens)
        self.hidden_state = hidden
        return hidden


def make_decoder(dtype, layout="last_exited", seed=0):
    shape = OuroShape.tiny()
    weights = OuroWeights(shape, "cuda", dtype, seed=seed)
    ctx = np.array([5, 17, 33, 1, 40, 16], dtype=np.int64)
    dec = OuroDecoder(shape, weights, ctx + 24, "cuda", dtype, layout=layout, seed=seed)
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    dec.key_cache.normal_(generator=g)
    dec.value_cache.normal_(generator=g)
    rng = np.random.default_rng(seed + 2)
    exits = rng.integers(0, 4, size=(dec.slots, 64))
    sched = DecodeScheduler(dec, ctx, lambda slot, i: int(exits[slot, i]))
    return dec, sched


@pytest.mark.parametrize("layout", ["last_exited", "shared"])
def test_mixed_depth_decode_matches_dense_reference(layout):
    dec, sched = make_decoder(torch.float32, layout)
    dense = DenseOuro(dec)
    for _ in range(14):
        depth, pos = sched.depth.copy(), sched.pos.copy()
        exiting = sched.prepare()
        dec.run(graphed=False)
        expected = dense.step(depth, pos, exiting)
        torch.cuda.synchronize()
        torch.testing.assert_close(dec.hidden_state, expected, atol=2e-4, rtol=2e-4)
        assert torch.equal(dec.tokens, dense.tokens)
        sched.advance(exiting)
    assert sched.generated > 0
    assert dec.attention.check_errors() == []


def test_graph_replay_matches_eager_steps():
    eager, s1 = make_decoder(torch.bfloat16, seed=3)
    graphed, s2 = make_decoder(torch.bfloat16, seed=3)
    exiting = s2.prepare()
    graphed.capture()
    first = True
    for _ in range(10):
        e1 = s1.prepare()
        eager.run(graphed=False)
        if not first:
            exiting = s2.prepare()
        graphed.run(graphed=True)
        first = False
        torch.cuda.synchronize()
        assert torch.equal(eager.hidden_state, graphed.hidden_state)
        assert torch.equal(eager.tokens, graphed.tokens)
        s1.advance(e1)
        s2.advance(exiting)
    assert torch.equal(eager.key_cache, graphed.key_cache)
    assert torch.equal(eager.value_cache, graphed.value_cache)


@pytest.mark.parametrize("d", [128, 24])  # 16-byte vector path; element path
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_fused_rope_kv_write_is_bit_identical_to_torch(dtype, d):
    from vllm_rlt_b200 import write_kv
    from vllm_rlt_b200.kernels import ouro_ops

    torch.manual_seed(0)
    heads, kv_heads, n = 16, 4, 37
    qkv = torch.randn(n, (heads + 2 * kv_heads) * d, device="cuda").to(dtype) * 3
    positions = torch.randint(0, 70000, (n,), device="cuda")
    inv_freq = 1.0 / (10000.0 ** (torch.arange(0, d, 2, device="cuda", dtype=torch.float32) / d))
    pool = torch.zeros(40, 3, 16, kv_heads, d, device="cuda", dtype=dtype)
    vpool = torch.zeros_like(pool)
    blocks = torch.randperm(40, device="cuda")[:n].sort().values
    offsets = torch.randint(0, 16, (n,), device="cuda")
    q = ouro_ops.rope_write_kv(qkv, positions, inv_freq, pool, vpool, 1, blocks, offsets, heads,
                               kv_heads, d)
    # the unfused expression of vllm_rlt/models/ouro.py:61-75, :104-110
    angles = positions.float().unsqueeze(-1) * inv_freq
    angles = torch.cat((angles, angles), dim=-1)
    cos, sin = angles.cos().to(dtype).unsqueeze(1), angles.sin().to(dtype).unsqueeze(1)
    q_ref = qkv[:, : heads * d].view(n, heads, d)
    k_ref = qkv[:, heads * d : (heads + kv_heads) * d].view(n, kv_heads, d)
    v_ref = qkv[:, (heads + kv_heads) * d :].view(n, kv_heads, d)
    q_ref = q_ref * cos + rotate_half(q_ref) * sin
    k_ref = k_ref * cos + rotate_half(k_ref) * sin
    pool_ref, vpool_ref = torch.zeros_like(pool), torch.zeros_like(vpool)
    write_kv(pool_ref, vpool_ref, 1, blocks, offsets, k_ref, v_ref)
    torch.cuda.synchronize()
    assert torch.equal(q, q_ref)
    assert torch.equal(pool, pool_ref) and torch.equal(vpool, vpool_ref)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_norm_and_swiglu_match_torch(dtype):
    from vllm_rlt_b200.kernels import ouro_ops

    torch.manual_seed(1)
    x = torch.randn(19, 2048, device="cuda").to(dtype)
    res = torch.randn(19, 2048, device="cuda").to(dtype)
    w = (1 + 0.1 * torch.randn(2048, device="cuda")).to(dtype)
    got = ouro_ops.rms_norm(x, w, 1e-6, residual=res)
    want = res + rms_norm(x, w, 1e-6)
    tol = dict(atol=0, rtol=2**-7) if dtype == torch.bfloat16 else dict(atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(got, want, **tol)
    gu = torch.randn(19, 2 * 5632, device="cuda").to(dtype) * 4
    got = ouro_ops.silu_mul(gu, 5632)
    want = torch.nn.functional.silu(gu[:, :5632]) * gu[:, 5632:]
    torch.testing.assert_close(got, want, **tol)


@pytest.mark.parametrize("residual", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_norm_pair_is_bit_identical_to_two_norms(dtype, residual):
    """rlt_rms_norm2 (norm [+ residual], then the next norm of that output,
    one launch) equals two rlt_rms_norm calls bit for bit."""
    from vllm_rlt_b200.kernels import ouro_ops

    torch.manual_seed(2)
    x = torch.randn(23, 2048, device="cuda").to(dtype) * 2
    res = torch.randn(23, 2048, device="cuda").to(dtype) if residual else None
    w = (1 + 0.1 * torch.randn(2048, device="cuda")).to(dtype)
    w2 = (1 + 0.1 * torch.randn(2048, device="cuda")).to(dtype)
    out, out2 = ouro_ops.rms_norm(x, w, 1e-6, residual=res, weight2=w2)
    first = ouro_ops.rms_norm(x, w, 1e-6, residual=res)
    second = ouro_ops.rms_norm(first, w2, 1e-6)
    assert torch.equal(out, first) and torch.equal(out2, second)
    want = (res if residual else 0) + rms_norm(x, w, 1e-6)
    tol = dict(atol=0, rtol=2**-7) if dtype == torch.bfloat16 else dict(atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(out, want.to(dtype), **tol)


def test_fused_decoder_matches_unfused_decoder():
    fused, s1 = make_decoder(torch.float32, seed=5)
    plain, s2 = make_decoder(torch.float32, seed=5)
    plain.fused = False
    for _ in range(8):
        e1, e2 = s1.prepare(), s2.prepare()
        fused.run(graphed=False)
        plain.run(graphed=False)
        torch.cuda.synchronize()
        torch.testing.assert_close(fused.hidden_state, plain.hidden_state, atol=1e-5, rtol=1e-5)
        assert torch.equal(fused.tokens, plain.tokens)
        s1.advance(e1)
        s2.advance(e2)
