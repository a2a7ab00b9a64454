"""Pin the CPU oracle to the reference's own outputs (fixtures made by tests/golden/make_golden.py
from the unmodified reference). Runs on CPU."""

from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from oracle import attention as A
from oracle import paged as OP

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
BF = torch.bfloat16


def _load(name):
    return np.load(os.path.join(GOLDEN, name))


@pytest.fixture(scope="module")
def runner():
    return _load("runner_attention.npz")


@pytest.mark.parametrize("name", ["ref_test", "gqa_bottom_right", "gqa_decode", "gqa_square"])
def test_sdpa_bottom_right_matches_reference_fallback(name):
    """transformers_flashinfer.py:153-202, incl. the reference test's own case
    (tests/test_transformers_flashinfer.py:20-48)."""
    f = _load("fallback.npz")
    dt = BF if bool(f[name + ".bf16"]) else torch.float32
    q, k, v = (torch.from_numpy(f[name + s]).to(dt) for s in (".query", ".key", ".value"))
    got = A.sdpa_bottom_right(q, k, v, float(f[name + ".scale"]), causal=bool(f[name + ".causal"]))
    assert torch.equal(got.float(), torch.from_numpy(f[name + ".out"]))


@pytest.mark.parametrize("name", ["ref_test", "gqa_bottom_right", "gqa_decode", "gqa_square"])
def test_fp32_oracle_matches_reference_fallback(name):
    """The parity oracle (absolute-position causal) agrees with the bridge's bottom-right mask."""
    f = _load("fallback.npz")
    q = torch.from_numpy(f[name + ".query"])[0].transpose(0, 1)  # [q, h, d]
    k = torch.from_numpy(f[name + ".key"])[0].transpose(0, 1)
    v = torch.from_numpy(f[name + ".value"])[0].transpose(0, 1)
    causal = bool(f[name + ".causal"])
    if not causal:
        assert q.shape[0] == 1
    q_pos0 = k.shape[0] - q.shape[0] if causal else k.shape[0] - 1
    got, _ = A.attention_fp32(q, k, v, float(f[name + ".scale"]), q_pos0)
    ref = torch.from_numpy(f[name + ".out"])[0]
    tol = 1e-5 if not bool(f[name + ".bf16"]) else 2e-2
    assert (got - ref).abs().max().item() <= tol


def test_reference_test_case_independent_check():
    """The reference test's independent bottom-right formula (test_transformers_flashinfer.py:34-42)
    and its assertion that top-left is_causal differs (:44-48)."""
    f = _load("fallback.npz")
    q, k, v = (torch.from_numpy(f["ref_test" + s]) for s in (".query", ".key", ".value"))
    scale = float(f["ref_test.scale"])
    got = A.sdpa_bottom_right(q, k, v, scale, causal=True)
    q_len, kv_len = q.shape[2], k.shape[2]
    scores = torch.matmul(q, k.transpose(-1, -2)) * scale
    mask = torch.arange(kv_len)[None, :] <= (torch.arange(q_len)[:, None] + kv_len - q_len)
    ref = torch.matmul(torch.softmax(scores.masked_fill(~mask, float("-inf")), -1), v)
    assert torch.allclose(got, ref.transpose(1, 2), atol=1e-5)
    top_left = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, scale=scale)
    assert not torch.allclose(got, top_left.transpose(1, 2), atol=1e-3)


def test_decode_literal_is_bit_exact(runner):
    """cuda_graph_executor.py:168,180-184 on the reference runner's own tensors."""
    for li in range(2):
        qg = torch.from_numpy(runner[f"decode.l{li}.qg"]).to(BF)
        kc = torch.from_numpy(runner[f"decode.l{li}.kt"]).to(BF).permute(2, 0, 1).contiguous()
        vc = torch.from_numpy(runner[f"decode.l{li}.vb"]).to(BF).permute(1, 0, 2).contiguous()
        nkv, g, hd = qg.shape
        got = A.decode_reference_grouped(qg.reshape(nkv * g, hd), kc, vc, int(runner["decode.pos"]),
                                         int(runner["decode.bound"]), hd**-0.5)
        assert torch.equal(got.float(), torch.from_numpy(runner[f"decode.l{li}.ctx"]).reshape(1, -1))


def test_decode_fp32_oracle_within_tolerance(runner):
    for li in range(2):
        qg = torch.from_numpy(runner[f"decode.l{li}.qg"]).to(BF)
        kc = torch.from_numpy(runner[f"decode.l{li}.kt"]).to(BF).permute(2, 0, 1).contiguous()
        vc = torch.from_numpy(runner[f"decode.l{li}.vb"]).to(BF).permute(1, 0, 2).contiguous()
        nkv, g, hd = qg.shape
        got, _ = A.attention_fp32(qg.reshape(1, nkv * g, hd), kc, vc, hd**-0.5,
                                  int(runner["decode.pos"]))
        ref = torch.from_numpy(runner[f"decode.l{li}.ctx"]).reshape(1, nkv * g, hd)
        d = (got - ref).abs()
        assert d.max().item() <= 2e-2 and d.mean().item() <= 2e-3


def test_prefill_literal_and_fp32(runner):
    """cuda_graph_executor.py:117-130 (repeat_interleave + causal SDPA)."""
    for li in range(2):
        q = torch.from_numpy(runner[f"prefill.l{li}.q"]).to(BF).transpose(0, 1)
        k = torch.from_numpy(runner[f"prefill.l{li}.k"]).to(BF).transpose(0, 1)
        v = torch.from_numpy(runner[f"prefill.l{li}.v"]).to(BF).transpose(0, 1)
        ref = torch.from_numpy(runner[f"prefill.l{li}.out"]).transpose(0, 1)
        t = q.shape[0]
        lit = A.prefill_reference(q, k, v, 128**-0.5)
        assert torch.equal(lit.float(), ref.reshape(t, -1))
        got, _ = A.attention_fp32(q, k, v, 128**-0.5, 0)
        d = (got - ref).abs()
        assert d.max().item() <= 2e-2 and d.mean().item() <= 2e-3


def test_verify_literal_and_fp32(runner):
    """cuda_graph_executor.py:245-263 (absolute-position mask over the whole max_len)."""
    pos0 = int(runner["verify.pos0"])
    for li in range(2):
        q = torch.from_numpy(runner[f"verify.l{li}.q"]).to(BF).transpose(0, 1)
        k = torch.from_numpy(runner[f"verify.l{li}.k"]).to(BF).transpose(0, 1)
        v = torch.from_numpy(runner[f"verify.l{li}.v"]).to(BF).transpose(0, 1)
        ref = torch.from_numpy(runner[f"verify.l{li}.out"]).transpose(0, 1)
        mask = runner[f"verify.l{li}.mask"][0]
        expect = np.arange(mask.shape[1])[None, :] <= (pos0 + np.arange(mask.shape[0]))[:, None]
        assert (mask == expect).all()
        lit = A.verify_reference(q, k, v, pos0, 128**-0.5)
        assert torch.equal(lit.float(), ref.reshape(q.shape[0], -1))
        got, _ = A.attention_fp32(q, k, v, 128**-0.5, pos0)
        d = (got - ref).abs()
        assert d.max().item() <= 2e-2 and d.mean().item() <= 2e-3


def test_input_pipeline_matches_reference_helpers():
    """rmsnorm / cos_sin / rope follow cuda_graph_executor.py:25-28,95-102."""
    q, k, v = A.make_attention_inputs(0, 4, 2, 128, 3, 5, 2)
    assert q.dtype == BF and q.shape == (3, 4, 128) and k.shape == (5, 2, 128)
    n = q.float().norm(dim=-1)  # RMSNorm then a rotation: per-head norm ~ sqrt(hd)
    assert ((n - 128**0.5).abs() < 0.5).all()
    x = torch.randn(7, 128).to(BF)
    w = torch.randn(128).to(BF)
    d = x.float()
    ref = (d * torch.rsqrt(d.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()).to(BF)
    assert torch.equal(A.rmsnorm(x, w, 1e-6), ref)


def test_lse_merge_algebra():
    q, k, v = A.make_attention_inputs(3, 8, 2, 128, 2, 300, 298)
    full, full_lse = A.attention_fp32(q, k, v, 128**-0.5, 298)
    os_, ls_ = [], []
    for a, b in [(0, 100), (100, 200), (200, 300)]:
        o, l = A.attention_fp32(q, k[a:b], v[a:b], 128**-0.5, 298, kv_pos0=a)
        os_.append(o), ls_.append(l)
    o, l = A.lse_merge(torch.stack(os_), torch.stack(ls_))
    assert torch.allclose(o, full, atol=1e-5) and torch.allclose(l, full_lse, atol=1e-4)


def test_kv_cache_metadata_golden():
    """kv_cache.py:116-149 against the reference's values (tests/test_kv_cache.py:8-19 + a
    permuted page-size-16 table)."""
    with open(os.path.join(GOLDEN, "kv_cache.json")) as fh:
        g = json.load(fh)
    for case in ("ref_test", "perm16"):
        c = g[case]
        md = OP.metadata_for(c["block_table"], token_count=c["token_count"],
                             page_size=c["page_size"], positions=c["positions"])
        for key in ("page_indptr", "page_indices", "last_page_len", "slot_mapping"):
            assert md[key] == c[key], key
    assert g["ref_test"]["slot_mapping"] == [0, 3, 4, 5]
    with pytest.raises(IndexError):
        OP.slot_mapping([0], [4], 4)


def test_shared_prefix_block_tables_golden():
    """PageAllocator + incref sharing (page_allocator.py:31-66): two block tables share pages."""
    with open(os.path.join(GOLDEN, "kv_cache.json")) as fh:
        g = json.load(fh)["shared_prefix"]
    assert g["a"][:2] == g["b"][:2]
    assert all(g["ref_count"][p] == 2 for p in g["a"][:2])
    assert len(set(g["a"]) | set(g["b"])) == 8


def test_store_gather_round_trip_golden():
    """kv_cache.py:191-256 on the reference's tensor-backed cache."""
    d = _load("kv_cache.npz")
    arena = torch.zeros(6, 2, 4, 2, 8)
    key = torch.from_numpy(d["key"])
    value = torch.from_numpy(d["value"])
    slots = d["slots"].tolist()
    OP.store_layer_tokens(arena, slots, key[0].transpose(0, 1), value[0].transpose(0, 1))
    assert torch.equal(arena, torch.from_numpy(d["kv_cache"])[1])
    k_out, v_out = OP.gather_layer_tokens(arena, slots)
    assert torch.equal(k_out, torch.from_numpy(d["k_out"]))
    assert torch.equal(v_out, torch.from_numpy(d["v_out"]))


def _tiny_model():
    from transformers import Qwen3Config, Qwen3ForCausalLM

    meta = json.load(open(os.path.join(GOLDEN, "runner_config.json")))
    keys = ["vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers",
            "num_attention_heads", "num_key_value_heads", "head_dim", "max_position_embeddings",
            "rms_norm_eps"]
    torch.manual_seed(meta["seed"])
    cfg = Qwen3Config(**{k: meta[k] for k in keys})
    cfg.rope_parameters = {"rope_type": "default", "rope_theta": 1e6}
    cfg.rope_theta = 1e6
    return Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval(), meta


def test_oracle_runner_reproduces_reference_runner_stream(runner):
    """The restated runner (oracle/runner.py) reproduces the reference runner's prefill logits,
    first decode logits, greedy stream and verify argmax bit-exactly on CPU."""
    from oracle.runner import ReferenceQwen3Runner

    model, meta = _tiny_model()
    r = ReferenceQwen3Runner(model, meta["max_len"])
    prompt = torch.from_numpy(runner["prompt"])
    with torch.no_grad():
        lg = r.prefill(prompt)
        assert torch.equal(lg, torch.from_numpy(runner["prefill.logits"]))
        toks = [int(lg.argmax(-1))]
        for step in range(meta["decode_steps"]):
            dl = r.decode(toks[-1], meta["prompt_len"] + step)
            if step == 0:
                assert torch.equal(dl, torch.from_numpy(runner["decode.logits"]))
            toks.append(int(dl.argmax(-1)))
        assert toks == runner["tokens"].tolist()
        vl = r.verify(torch.from_numpy(runner["verify.tokens"]), meta["verify_pos0"])
        assert vl.argmax(-1).tolist() == runner["verify.argmax"].tolist()
