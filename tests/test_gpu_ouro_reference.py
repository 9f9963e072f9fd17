"""The Ouro decoder on the B200 kernels, pinned to the reference's own model.

One random-initialised reference ``OuroForCausalLM`` (vllm_rlt/models/
ouro.py:150-220, from baseline/_ref) provides the weights; ``OuroWeights.
from_state_dict`` loads them into this package's decoder. The decoder runs a
mixed-depth schedule -- several requests in one batch, each token of a
request leaving the recurrent core at that request's exit depth -- through
its captured CUDA-graph step, and every pass's hidden state, exit-gate value
and sampled token is compared with the reference's dense oracle
``dense_reference`` (vllm_rlt/models/reference.py:7-82) run on the same
token sequence, the way the reference pins its own model
(tests/test_ouro.py:34-96: every depth of every position, and a mixed-depth
batch against separate dense runs).
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from vllm_rlt_b200.ouro import DecodeScheduler, OuroDecoder, OuroShape, OuroWeights

pytestmark = pytest.mark.gpu

REF = Path(__file__).resolve().parents[1] / "baseline" / "_ref"


def _reference():
    if not (REF / "vllm_rlt" / "__init__.py").exists():
        pytest.skip("the unmodified reference is not installed under baseline/_ref")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from vllm_rlt.models import OuroConfig, OuroForCausalLM
    from vllm_rlt.models.reference import dense_reference

    return OuroConfig, OuroForCausalLM, dense_reference


def _shape(config):
    return OuroShape(vocab=config.vocab_size, hidden=config.hidden_size,
                     intermediate=config.intermediate_size, layers=config.num_hidden_layers,
                     heads=config.num_attention_heads, kv_heads=config.num_key_value_heads,
                     head_dim=config.head_dim, loops=config.total_ut_steps,
                     rope_theta=float(config.rope_theta), eps=float(config.rms_norm_eps))


def _run_decoder(model, shape, dtype, exits, first_tokens, steps, fused):
    """Run ``steps`` graph-captured decode steps; slot s exits every token at
    depth ``exits[s]``. Returns per slot the token sequence and, per
    (position, depth), the pass's hidden state and gate."""
    device = torch.device("cuda")
    weights = OuroWeights.from_state_dict(shape, model.state_dict(), device, dtype)
    capacity = [steps + 1] * len(exits)
    dec = OuroDecoder(shape, weights, capacity, device, dtype, page=16, seed=5, fused=fused)
    dec.tokens.copy_(torch.tensor(first_tokens, dtype=torch.int64))
    sched = DecodeScheduler(dec, [0] * len(exits), lambda slot, index: exits[slot])
    exiting = sched.prepare()
    dec.capture()
    tokens = [[t] for t in first_tokens]
    passes = [dict() for _ in exits]
    for step in range(steps):
        if step:
            exiting = sched.prepare()
        depth, pos = sched.depth.copy(), sched.pos.copy()
        dec.run(graphed=True)
        torch.cuda.synchronize()
        hidden = dec.hidden_state.float().cpu()
        gate = dec.gate.float().cpu()
        sampled = dec.tokens.cpu().tolist()
        for s in range(len(exits)):
            passes[s][int(pos[s]), int(depth[s])] = (hidden[s], float(gate[s]))
            if exiting[s]:
                tokens[s].append(int(sampled[s]))
        sched.advance(exiting)
    assert dec.attention.check_errors() == []
    return tokens, passes


@pytest.mark.parametrize("head_dim", [64, 128])
@pytest.mark.parametrize("fused", [True, False])
def test_mixed_depth_decoder_matches_dense_reference_fp32(head_dim, fused):
    OuroConfig, OuroForCausalLM, dense_reference = _reference()
    torch.manual_seed(71)
    config = OuroConfig.tiny(vocab_size=97, hidden_size=128, intermediate_size=192,
                             num_attention_heads=4, num_key_value_heads=2, head_dim=head_dim)
    model = OuroForCausalLM(config).float()
    shape = _shape(config)
    exits = [3, 1, 2, 0]  # a different exit depth per request: a mixed-depth batch
    tokens, passes = _run_decoder(model, shape, torch.float32, exits, [5, 7, 11, 13], 16, fused)
    checked = 0
    for s, exit_depth in enumerate(exits):
        seq = torch.tensor(tokens[s])
        expected = dense_reference(model, seq, exit_depth + 1)
        for (pos, depth), (hidden, gate) in passes[s].items():
            want_hidden, want_gate, want_logits = expected[depth]
            torch.testing.assert_close(hidden, want_hidden[pos].float(), atol=2e-4, rtol=1e-3)
            want = float(torch.sigmoid(want_gate[pos].float()))
            assert abs(gate - want) < 1e-4, (s, pos, depth)
            if depth == exit_depth:
                assert tokens[s][pos + 1] == int(want_logits[pos].argmax()), (s, pos)
            checked += 1
    assert checked >= 40


def test_mixed_depth_decoder_tracks_dense_reference_bf16():
    """bf16 weights and activations on both sides (the reference's dense
    oracle on the GPU in bf16): the two agree to bf16 rounding -- relative
    L2 error of every pass's hidden state under 3 %, and the same greedy
    token wherever the reference's top-2 logit gap exceeds its rounding."""
    OuroConfig, OuroForCausalLM, dense_reference = _reference()
    torch.manual_seed(72)
    config = OuroConfig.tiny(vocab_size=97, hidden_size=256, intermediate_size=384,
                             num_attention_heads=4, num_key_value_heads=4, head_dim=128)
    model = OuroForCausalLM(config).float()
    shape = _shape(config)
    exits = [3, 2, 1, 3]
    tokens, passes = _run_decoder(model, shape, torch.bfloat16, exits, [3, 9, 27, 81], 16, True)
    gpu_model = OuroForCausalLM(config).to("cuda", torch.bfloat16)
    gpu_model.load_state_dict({k: v.to(torch.bfloat16) for k, v in model.state_dict().items()})
    worst, agreed, decided = 0.0, 0, 0
    for s, exit_depth in enumerate(exits):
        seq = torch.tensor(tokens[s], device="cuda")
        expected = dense_reference(gpu_model, seq, exit_depth + 1)
        for (pos, depth), (hidden, _gate) in passes[s].items():
            want = expected[depth][0][pos].float().cpu()
            worst = max(worst, float((hidden - want).norm() / want.norm()))
            if depth == exit_depth:
                logits = expected[depth][2][pos].float()
                top = torch.topk(logits, 2).values
                if float(top[0] - top[1]) > 0.05 * float(logits.abs().max()):
                    decided += 1
                    agreed += tokens[s][pos + 1] == int(logits.argmax())
    assert worst < 0.03, worst
    assert decided >= 8 and agreed == decided


def test_weights_load_every_reference_parameter():
    OuroConfig, OuroForCausalLM, _ = _reference()
    torch.manual_seed(1)
    config = OuroConfig.tiny(hidden_size=64, intermediate_size=96, head_dim=32)
    model = OuroForCausalLM(config)
    shape = _shape(config)
    w = OuroWeights.from_state_dict(shape, model.state_dict(), torch.device("cuda"),
                                    torch.float32)
    state = model.state_dict()
    layer = model.model.layers[1]
    q, k, v = (layer.self_attn.q_proj.weight, layer.self_attn.k_proj.weight,
               layer.self_attn.v_proj.weight)
    assert torch.equal(w.wqkv[1].cpu(), torch.cat([q, k, v]).detach())
    assert torch.equal(w.lm_head.cpu(), state["lm_head.weight"])
    assert torch.equal(w.gate_b.cpu(), state["model.early_exit_gate.bias"])
    assert np.allclose(w.inv_freq.cpu().numpy(), model.model.rotary_emb.inv_freq.numpy(), 0, 0)
