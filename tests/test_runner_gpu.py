"""End-to-end: the engine's CUDA-graph runner vs the reference runner's math (oracle/runner.py)
on the same random-weight Qwen3 on the GPU. Greedy token streams must be identical."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _model(layers, nh, nkv, hidden, inter, vocab, seed):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    torch.manual_seed(seed)
    cfg = Qwen3Config(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter,
                      num_hidden_layers=layers, num_attention_heads=nh, num_key_value_heads=nkv,
                      head_dim=128, max_position_embeddings=8192, rms_norm_eps=1e-6)
    cfg.rope_parameters = {"rope_type": "default", "rope_theta": 1e6}
    cfg.rope_theta = 1e6
    return Qwen3ForCausalLM(cfg).to(device="cuda", dtype=torch.bfloat16).eval()


def _first_divergence(a, b):
    for i, (x, y) in enumerate(zip(a, b)):
        if x != y:
            return i
    return None


@pytest.mark.parametrize("shape", [(4, 32, 8, 1024, 2048, 4096), (4, 16, 8, 1024, 3072, 4096)])
def test_greedy_stream_identical_to_reference_runner(shape):
    from oracle.runner import ReferenceQwen3Runner
    from solort_b200.runner import GraphQwen3Runner

    layers, nh, nkv, hidden, inter, vocab = shape
    model = _model(layers, nh, nkv, hidden, inter, vocab, seed=11)
    g = torch.Generator().manual_seed(5)
    prompt = torch.randint(0, vocab, (37,), generator=g).cuda()
    with torch.no_grad():
        ref = ReferenceQwen3Runner(model, 512).greedy(prompt, 40)
        ours = GraphQwen3Runner(model, 512).greedy(prompt, 40)
    assert ours == ref, f"first divergence at {_first_divergence(ours, ref)}: {ours} vs {ref}"


def test_verify_and_chunked_decode_match_reference_runner():
    from oracle.runner import ReferenceQwen3Runner
    from solort_b200.runner import GraphQwen3Runner

    model = _model(3, 32, 8, 1024, 2048, 4096, seed=3)
    prompt = torch.randint(0, 4096, (60,), generator=torch.Generator().manual_seed(8)).cuda()
    with torch.no_grad():
        ref = ReferenceQwen3Runner(model, 256)
        ours = GraphQwen3Runner(model, 256)
        r_toks = ref.greedy(prompt, 12)
        o_toks = ours.greedy(prompt, 12)
        assert o_toks == r_toks
        # chunked greedy through decode_gpu_argmax (the executor's K=4 loop)
        cur = torch.tensor([o_toks[-1]], device="cuda")
        pos = 60 + 12
        chunk = []
        for i in range(4):
            cur = ours.decode_gpu_argmax(cur, pos + i)
            chunk.append(int(cur.item()))
        ref_chunk = []
        t = r_toks[-1]
        for i in range(4):
            t = int(ref.decode(t, pos + i).argmax(-1))
            ref_chunk.append(t)
        assert chunk == ref_chunk
        # speculative verify of 5 tokens at the next position
        drafts = torch.tensor([chunk[-1]] + chunk[:4], device="cuda")
        vr = ref.verify(drafts, pos + 4).argmax(-1).tolist()
        vo = ours.verify(drafts, pos + 4).argmax(-1).tolist()
        assert vo == vr
