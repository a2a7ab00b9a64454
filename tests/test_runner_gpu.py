"""End-to-end: the engine's CUDA-graph runner against the reference runner's math
(oracle/runner.py) on the same random-weight Qwen3 on the GPU.

* Greedy streams (``stream_parity``): teacher-forced along the fp32 parity oracle's stream, the
  engine's argmax equals the oracle's at every step whose margin exceeds twice the reference's own
  noise band (literal bf16-score attention vs the oracle); the free-running streams agree up to
  the first step that is not decided that way; the engine's logit noise is within 1.25x of the
  reference's. The comparison is printed.
* The chunked greedy loop and verify agree with the reference runner token for token.
* The speculative loop: the engine's ``spec_round`` and the reference's ``_spec_round`` restated
  (``oracle.runner.reference_spec_round``) driven over identical engine runners give the same
  tokens and the same accepted counts, round by round.
"""

from __future__ import annotations

import json

import pytest
import torch

from stream_parity import assert_stream_parity, compare, first_divergence, teacher_forced

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


SHAPES = [(4, 32, 8, 1024, 2048, 4096), (4, 16, 8, 1024, 3072, 4096)]


@pytest.mark.parametrize("shape", SHAPES)
def test_greedy_stream_matches_parity_oracle_and_reference(shape):
    from oracle.runner import ReferenceQwen3Runner
    from solort_b200.runner import GraphQwen3Runner

    layers, nh, nkv, hidden, inter, vocab = shape
    model = _model(layers, nh, nkv, hidden, inter, vocab, seed=11)
    prompt = torch.randint(0, vocab, (37,), generator=torch.Generator().manual_seed(5)).cuda()
    n = 64
    with torch.no_grad():
        stream_f = ReferenceQwen3Runner(model, 512, attention="fp32").greedy(prompt, n)
        stream_r = ReferenceQwen3Runner(model, 512, graphs=True).greedy(prompt, n)
        stream_o = GraphQwen3Runner(model, 512).greedy(prompt, n)
        lf = teacher_forced(ReferenceQwen3Runner(model, 512, attention="fp32"), prompt, stream_f)
        lo = teacher_forced(GraphQwen3Runner(model, 512), prompt, stream_f)
        lr = teacher_forced(ReferenceQwen3Runner(model, 512, graphs=True), prompt, stream_f)
    res = compare(stream_f, lf, lr, lo, stream_o, stream_r)
    print(json.dumps({"shape": list(shape), **res}))
    assert_stream_parity(res)


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
        cur = torch.tensor([o_toks[-1]], device="cuda")
        pos = 60 + 12
        chunk = []
        for i in range(4):  # the executor's chunked greedy loop (decode_gpu_argmax, K = 4)
            cur = ours.decode_gpu_argmax(cur, pos + i)
            chunk.append(int(cur.item()))
        ref_chunk, t = [], r_toks[-1]
        for i in range(4):
            t = int(ref.decode(t, pos + i).argmax(-1))
            ref_chunk.append(t)
        assert chunk == ref_chunk
        drafts = torch.tensor([chunk[-1]] + chunk[:4], device="cuda")
        vr = ref.verify(drafts, pos + 4).argmax(-1).tolist()
        vo = ours.verify(drafts, pos + 4).argmax(-1).tolist()
        assert vo == vr


def test_single_decode_graph_gives_the_bucketed_stream():
    """One decode graph for every position (the engine reads the live length from pos_buf) gives
    the logits of one graph per bucket: teacher-forced along the bucketed stream across the 128
    bucket, within 2e-2, argmax equal except at near-ties (the split plans differ, so the fp32
    merge order does)."""
    from solort_b200.runner import GraphQwen3Runner

    model = _model(2, 32, 8, 1024, 2048, 4096, seed=4)
    prompt = torch.randint(0, 4096, (100,), generator=torch.Generator().manual_seed(2)).cuda()
    with torch.no_grad():
        bucketed = GraphQwen3Runner(model, 512)
        single = GraphQwen3Runner(model, 512, single_decode_graph=True)
        assert single.buckets == [512]
        stream = bucketed.greedy(prompt, 40)
        la = teacher_forced(GraphQwen3Runner(model, 512), prompt, stream)
        lb = teacher_forced(single, prompt, stream)
    for step, (a, b) in enumerate(zip(la, lb)):
        assert (a - b).abs().max().item() <= 2e-2, step
        if a.argmax().item() != b.argmax().item():
            top2 = a.flatten().topk(2).values
            assert (top2[0] - top2[1]).item() <= 4e-2, step


def test_speculative_round_is_the_reference_round():
    """The engine's speculative loop and the reference's ``_spec_round`` (restated in the oracle)
    over identical engine runners: same tokens, same accepted count in every round, with a draft on
    the target's weights (whole rounds accepted, the draft's continuity decode taken) and an
    unrelated draft (early rejections). Also: greedy speculative decoding reproduces the target's
    own greedy stream up to the first step whose teacher-forced margin is a near-tie between the
    verify (multi-row projections) and decode (weight-stream) roundings."""
    from oracle.runner import reference_speculative_greedy
    from solort_b200.runner import GraphQwen3Runner, speculative_greedy

    model = _model(3, 32, 8, 1024, 2048, 4096, seed=3)
    other = _model(2, 32, 8, 1024, 2048, 4096, seed=11)
    prompt = torch.randint(0, 4096, (60,), generator=torch.Generator().manual_seed(8)).cuda()
    steps, k = 32, 4
    with torch.no_grad():
        greedy = GraphQwen3Runner(model, 256).greedy(prompt, steps)
        forced = teacher_forced(GraphQwen3Runner(model, 256), prompt, greedy)
        for draft_model, full_rounds in ((model, True), (other, False)):
            ours, acc_ours = speculative_greedy(GraphQwen3Runner(model, 256),
                                                GraphQwen3Runner(draft_model, 256), prompt, steps, k)
            ref, acc_ref = reference_speculative_greedy(GraphQwen3Runner(model, 256),
                                                        GraphQwen3Runner(draft_model, 256), prompt,
                                                        steps, k)
            assert ours == ref and acc_ours == acc_ref, (ours, ref, acc_ours, acc_ref)
            assert len(ours) == steps + 1
            assert any(a == k for a in acc_ours) if full_rounds else any(a < k for a in acc_ours)
            i = first_divergence(ours, greedy)
            if i is not None:
                top2 = forced[i].flatten().topk(2)
                print(json.dumps({"spec_vs_greedy_first_divergence": i,
                                  "margin": (top2.values[0] - top2.values[1]).item()}))
                assert (top2.values[0] - top2.values[1]).item() <= 4e-2, (i, acc_ours)
                assert ours[i] in top2.indices.tolist(), i
