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


def test_paged_bridge_mirrors_into_and_reads_from_solort_paged_kv():
    """The paged bridge end to end: a 2-layer Qwen3 runs through HF with the engine's callable
    inside ``solort_kv_write_context`` for every forward (a 150-token prefill, three decode steps,
    one 4-token verify), with a SoloRT arena ``[layers, pages, 2, P, nkv, 128]`` whose unwritten
    slots hold random values and a block table drawn from a seeded permutation of the pages.
    Checked: the arena equals the reference's ``store_layer_tokens`` applied to HF's K / V
    (bit-exact, every other slot untouched); decode and verify were read from the arena through
    the block table (``paged_calls``); logits match transformers' eager attention."""
    from types import SimpleNamespace

    from transformers import Qwen3Config, Qwen3ForCausalLM

    from oracle import paged as OP
    from solort_b200 import hf_attention as H

    H.register_solort_b200_attention()
    torch.manual_seed(1)
    layers, nkv, P, pages = 2, 2, 16, 64
    cfg = Qwen3Config(vocab_size=512, hidden_size=256, intermediate_size=512,
                      num_hidden_layers=layers, num_attention_heads=8, num_key_value_heads=nkv,
                      head_dim=128)
    model = Qwen3ForCausalLM(cfg).to(device="cuda", dtype=torch.bfloat16).eval()
    g = torch.Generator().manual_seed(4)
    arena0 = torch.randn(layers, pages, 2, P, nkv, 128, generator=g).to(torch.bfloat16)
    cache = SimpleNamespace(kv_cache=arena0.cuda(), mirrored_tokens=0, mirror_skipped=0)
    table = torch.randperm(pages, generator=g)[:12].tolist()
    prompt = torch.randint(0, 512, (1, 150), generator=g).cuda()
    steps = [torch.tensor([[t]], device="cuda") for t in (7, 99, 311)]
    verify = torch.tensor([[5, 6, 7, 8]], device="cuda")

    def run(impl, with_context):
        model.set_attn_implementation(impl)
        logits, pos = [], 0

        def fwd(ids, past):
            nonlocal pos
            slots = OP.slot_mapping(table, list(range(pos, pos + ids.shape[1])), P)
            if with_context:
                with H.solort_kv_write_context(cache, slots, block_table=table):
                    o = model(ids, past_key_values=past, use_cache=True)
            else:
                o = model(ids, past_key_values=past, use_cache=True)
            pos += ids.shape[1]
            logits.append(o.logits.float())
            return o.past_key_values

        past = fwd(prompt, None)
        for s in steps:
            past = fwd(s, past)
        past = fwd(verify, past)
        return logits, past

    with torch.no_grad():
        ref_logits, _ = run("eager", False)
        before = H.attention_snapshot()
        got_logits, past = run(H.ATTENTION_NAME, True)
        after = H.attention_snapshot()
    n_tok = 150 + len(steps) + verify.shape[1]
    assert after["paged_calls"] - before["paged_calls"] == (len(steps) + 1) * layers
    assert after["prefill_calls"] - before["prefill_calls"] == layers  # 150 rows: the tcgen05 kernel
    assert after["mirrored_tokens"] - before["mirrored_tokens"] == n_tok * layers
    assert cache.mirrored_tokens == n_tok * layers and cache.mirror_skipped == 0
    # arena == the reference's slot-mapped store of HF's own K / V into the initial arena
    expect = arena0.clone()
    slots = OP.slot_mapping(table, list(range(n_tok)), P)
    for li in range(layers):
        k = past.layers[li].keys[0].transpose(0, 1).cpu()
        v = past.layers[li].values[0].transpose(0, 1).cpu()
        OP.store_layer_tokens(expect[li], slots, k, v)
    assert torch.equal(cache.kv_cache.cpu(), expect)
    scale = max(1.0, ref_logits[0].abs().max().item())
    for i, (a, b) in enumerate(zip(got_logits, ref_logits)):
        _close(a, b, f"forward {i}", max_abs=2e-2 * scale, mean_abs=2e-3 * scale)
    assert ops_status() == 0


def ops_status():
    from solort_b200 import ops

    return ops.device_status()
