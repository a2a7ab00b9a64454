"""Greedy token streams at the full depth of the two BASELINE model shapes, random weights.

The engine's CUDA-graph runner (every projection as a weight stream, the fused prologue, the
split-KV decode) against the reference's runner restated in ``oracle/runner.py`` -- with its
literal attention (``cuda_graph_executor.py:124-130,180-184,261-263``) and with the fp32-softmax
parity oracle at the same sites -- over 96 greedy steps after a 64-token prompt, on the 36-layer
Qwen3-4B shape and the 28-layer Qwen3-0.6B shape (vocab 151936, tied embeddings).

What is asserted (``stream_parity``): at every step whose top-2 oracle margin exceeds twice the
reference's own noise band, the engine's argmax equals the oracle's; the free-running engine
stream equals the oracle's up to the first step that is not decided that way; and the engine's
logit noise is within 1.25x of the reference's. Each test prints the full comparison (decided
steps, undecided steps and their margins, exact bf16 ties, the first divergence of the engine's
and of the reference's own free-running stream from the oracle's).
"""

from __future__ import annotations

import json

import pytest
import torch

from stream_parity import assert_stream_parity, compare, teacher_forced

pytestmark = pytest.mark.gpu

SHAPES = {"qwen3-4b": (36, 2560, 9728, 32, 8), "qwen3-0.6b": (28, 1024, 3072, 16, 8)}
STEPS, PROMPT, MAX_LEN = 96, 64, 512


def _model(shape: str, seed: int):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    layers, hidden, inter, nh, nkv = SHAPES[shape]
    cfg = Qwen3Config(vocab_size=151936, hidden_size=hidden, intermediate_size=inter,
                      num_hidden_layers=layers, num_attention_heads=nh, num_key_value_heads=nkv,
                      head_dim=128, max_position_embeddings=40960, rms_norm_eps=1e-6,
                      tie_word_embeddings=True)
    cfg.rope_parameters = {"rope_type": "default", "rope_theta": 1e6}
    cfg.rope_theta = 1e6
    torch.manual_seed(seed)
    with torch.device("cuda"):
        return Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()


@pytest.mark.parametrize("shape", list(SHAPES))
def test_full_depth_greedy_stream(shape):
    from oracle.runner import ReferenceQwen3Runner
    from solort_b200.runner import GraphQwen3Runner

    model = _model(shape, seed=0)
    prompt = torch.randint(0, 151936, (PROMPT,), generator=torch.Generator().manual_seed(5)).cuda()
    with torch.no_grad():
        oracle_stream = ReferenceQwen3Runner(model, MAX_LEN, attention="fp32").greedy(prompt, STEPS)
        lf = teacher_forced(ReferenceQwen3Runner(model, MAX_LEN, attention="fp32"), prompt, oracle_stream)
        lr = teacher_forced(ReferenceQwen3Runner(model, MAX_LEN, graphs=True), prompt, oracle_stream)
        ref_stream = ReferenceQwen3Runner(model, MAX_LEN, graphs=True).greedy(prompt, STEPS)
        ours_stream = GraphQwen3Runner(model, MAX_LEN).greedy(prompt, STEPS)
        lo = teacher_forced(GraphQwen3Runner(model, MAX_LEN), prompt, oracle_stream)
    res = compare(oracle_stream, lf, lr, lo, ours_stream, ref_stream)
    print(json.dumps({"shape": shape, **res}))
    assert_stream_parity(res)
