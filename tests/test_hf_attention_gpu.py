"""The HF AttentionInterface callable (paged-bridge drop-in) on the GPU: the reference bridge's own
fallback cases (tests/golden/fallback.npz) and a whole random-weight Qwen3 forward (prefill +
cached decode) against transformers' eager attention."""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _close(got, ref, what, max_abs=2e-2, mean_abs=2e-3):
    d = (got.float().cpu() - ref.float().cpu()).abs()
    assert d.max().item() <= max_abs, f"{what}: max {d.max().item():.4g}"
    assert d.mean().item() <= mean_abs, f"{what}: mean {d.mean().item():.4g}"


@pytest.mark.parametrize("name", ["gqa_bottom_right", "gqa_decode", "gqa_square"])
def test_callable_matches_reference_fallback(name):
    from solort_b200.hf_attention import solort_b200_attention_forward

    f = np.load("tests/golden/fallback.npz")
    q, k, v = (torch.from_numpy(f[name + s]).to(torch.bfloat16).cuda()
               for s in (".query", ".key", ".value"))
    out, w = solort_b200_attention_forward(None, q, k, v, None, float(f[name + ".scale"]))
    assert w is None and out.shape == (1, q.shape[2], q.shape[1], 128)
    _close(out, torch.from_numpy(f[name + ".out"]), name)


def test_callable_rejects_unsupported_inputs():
    from solort_b200.hf_attention import solort_b200_attention_forward

    q = torch.zeros(2, 8, 1, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(2, 2, 4, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="batch_size=1"):
        solort_b200_attention_forward(None, q, k, k, None, 0.1)
    with pytest.raises(RuntimeError, match="sliding"):
        solort_b200_attention_forward(None, q[:1], k[:1], k[:1], None, 0.1, sliding_window=8)


def test_qwen3_forward_with_registered_attention():
    from transformers import Qwen3Config, Qwen3ForCausalLM

    from solort_b200 import hf_attention as H

    H.register_solort_b200_attention()
    torch.manual_seed(0)
    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=8, num_key_value_heads=2, head_dim=128)
    model = Qwen3ForCausalLM(cfg).to(device="cuda", dtype=torch.bfloat16).eval()
    ids = torch.randint(0, 512, (1, 150), device="cuda")
    with torch.no_grad():
        model.set_attn_implementation("eager")
        ref = model(ids, use_cache=True)
        ref_next = model(ids[:, -1:] * 0 + 7, past_key_values=ref.past_key_values).logits
        model.set_attn_implementation(H.ATTENTION_NAME)
        before = H.attention_snapshot()
        got = model(ids, use_cache=True)
        got_next = model(ids[:, -1:] * 0 + 7, past_key_values=got.past_key_values).logits
        after = H.attention_snapshot()
    assert after["prefill_calls"] - before["prefill_calls"] == 2
    assert after["decode_calls"] - before["decode_calls"] == 2
    scale = ref.logits.float().abs().max().item()
    _close(got.logits, ref.logits, "prefill logits", max_abs=2e-2 * max(1.0, scale), mean_abs=2e-3 * max(1.0, scale))
    _close(got_next, ref_next, "decode logits", max_abs=2e-2 * max(1.0, scale), mean_abs=2e-3 * max(1.0, scale))
