"""The engine bound into the reference's runner (``solort_b200.reference_binding``) on the GPU.

``EngineAttention`` overrides ``_prefill_forward`` / ``_decode_forward`` / ``_verify_forward`` of
a ``_GraphQwen3Runner``-shaped class and nothing else. It is bound here to the oracle's restatement
of ``_GraphQwen3Runner`` with graph capture on (``graphs=True``: the reference's own capture and
replay code path), and, where the reference package itself is importable, to the reference's
class. Checked: every attention call of the captured graphs goes through
``torch.ops.solort_attn``; teacher-forced along the fp32 oracle's stream the bound runner is
within the reference's own noise band (``stream_parity``); the chunked greedy loop, verify and the
reference's speculative round run unchanged on top of it.
"""

from __future__ import annotations

import json
import os
import sys

import pytest
import torch

from stream_parity import assert_stream_parity, compare, teacher_forced

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


def _graphed_reference():
    from oracle.runner import ReferenceQwen3Runner

    class GraphedReference(ReferenceQwen3Runner):
        """The restated runner with the reference's graph capture and literal attention."""

        def __init__(self, model, max_len: int) -> None:
            super().__init__(model, max_len, attention="reference", graphs=True)

    return GraphedReference


@pytest.fixture
def op_calls(monkeypatch):
    """Count the engine ops' C-ABI calls (the registered kernels look these up per call)."""
    from solort_b200 import _calls

    counts = {"decode": 0, "prefill": 0}

    def wrap(fn, key):
        def inner(*a, **k):
            counts[key] += 1
            return fn(*a, **k)
        return inner

    monkeypatch.setattr(_calls, "decode_static_into", wrap(_calls.decode_static_into, "decode"))
    monkeypatch.setattr(_calls, "prefill_into", wrap(_calls.prefill_into, "prefill"))
    return counts


def test_binding_on_the_restated_reference_runner(op_calls):
    from oracle.runner import ReferenceQwen3Runner, reference_speculative_greedy
    from solort_b200.reference_binding import EngineAttention, engine_runner_class

    base = _graphed_reference()
    bound_cls = engine_runner_class(base)
    assert issubclass(bound_cls, EngineAttention) and issubclass(bound_cls, base)
    layers = 4
    model = _model(layers, 32, 8, 1024, 2048, 4096, seed=11)
    prompt = torch.randint(0, 4096, (37,), generator=torch.Generator().manual_seed(5)).cuda()
    n = 48
    with torch.no_grad():
        stream_f = ReferenceQwen3Runner(model, 512, attention="fp32").greedy(prompt, n)
        bound = bound_cls(model, 512)
        stream_b = bound.greedy(prompt, n)
        # the prefill graph (bucket 64) and the decode graphs (buckets 128, 512) were captured with
        # the engine's ops inside: one call per layer per capture and per warm-up forward
        assert op_calls["prefill"] == layers * 3, op_calls  # 2 warm-up forwards + 1 capture
        assert op_calls["decode"] == layers * 4, op_calls  # 3 warm-up + 1 capture, bucket 128
        stream_r = base(model, 512).greedy(prompt, n)
        lf = teacher_forced(ReferenceQwen3Runner(model, 512, attention="fp32"), prompt, stream_f)
        lb = teacher_forced(bound_cls(model, 512), prompt, stream_f)
        lr = teacher_forced(base(model, 512), prompt, stream_f)
    res = compare(stream_f, lf, lr, lb, stream_b, stream_r)
    print(json.dumps({"binding": "restated _GraphQwen3Runner", **res}))
    assert_stream_parity(res)

    # chunked greedy (decode_gpu_argmax x 4) and verify run unchanged on the bound runner
    with torch.no_grad():
        pos = 37 + n
        cur = torch.tensor([stream_b[-1]], device="cuda")
        chunk = []
        for i in range(4):
            cur = bound.decode_gpu_argmax(cur, pos + i)
            chunk.append(int(cur.item()))
        drafts = torch.tensor([stream_b[-1]] + chunk[:3], device="cuda")
        v = bound.verify(drafts, pos)
        assert v.shape == (4, 4096) and torch.isfinite(v).all()
        # each verify row predicts the token the decode graphs produced after the same prefix, or
        # its top-2 margin is within the verify/decode rounding difference (multi-row GEMMs)
        for i in range(3):
            t2 = v[i].topk(2)
            assert int(t2.indices[0]) == chunk[i] or (t2.values[0] - t2.values[1]).item() <= 4e-2, i

    # the reference's speculative loop over bound runners: exact greedy acceptance bookkeeping
    with torch.no_grad():
        spec, accepted = reference_speculative_greedy(bound_cls(model, 256), bound_cls(model, 256),
                                                      prompt, 24, 4)
    assert len(spec) == 25 and any(a == 4 for a in accepted), accepted


def test_binding_on_the_reference_package():
    """The same binding on the reference's own ``_GraphQwen3Runner`` where the package imports
    (it is not installed on every machine this suite runs on)."""
    src = os.environ.get("SOLORT_REFERENCE_SRC")
    if src and src not in sys.path:
        sys.path.insert(0, src)
    try:
        from solort.model import cuda_graph_executor as cge
    except Exception as exc:
        pytest.skip(f"the reference package is not importable here ({type(exc).__name__})")
    from oracle.runner import ReferenceQwen3Runner
    from solort_b200.reference_binding import engine_runner_class

    model = _model(3, 32, 8, 1024, 2048, 4096, seed=3)
    prompt = torch.randint(0, 4096, (40,), generator=torch.Generator().manual_seed(8)).cuda()
    n = 32
    with torch.no_grad():
        stream_f = ReferenceQwen3Runner(model, 256, attention="fp32").greedy(prompt, n)
        bound_cls = engine_runner_class(cge._GraphQwen3Runner)

        def greedy(r):
            toks = [int(r.prefill(prompt).argmax(-1).item())]
            for i in range(n):
                toks.append(r.decode_argmax(toks[-1], 40 + i))
            return toks

        stream_b = greedy(bound_cls(model, 256))
        stream_r = greedy(cge._GraphQwen3Runner(model, 256))
        lf = teacher_forced(ReferenceQwen3Runner(model, 256, attention="fp32"), prompt, stream_f)
        lb = teacher_forced(bound_cls(model, 256), prompt, stream_f)
        lr = teacher_forced(cge._GraphQwen3Runner(model, 256), prompt, stream_f)
    res = compare(stream_f, lf, lr, lb, stream_b, stream_r)
    print(json.dumps({"binding": "reference _GraphQwen3Runner", **res}))
    assert_stream_parity(res)
