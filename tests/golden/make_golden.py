"""Generate golden fixtures by running the unmodified reference (owen920831/SoloRT) on the CPU.

Run in a container where the reference source tree is available:

    python tests/golden/make_golden.py --reference-src <reference>/src

It imports the reference's own modules and records what they compute; nothing of the reference is
copied. The fixtures pin the CPU oracle (``oracle/``) and are the known-answer inputs of the GPU
parity tests. Outputs (all small, committed):

* ``fallback.npz`` -- ``_torch_attention_fallback`` (``transformers_flashinfer.py:153-202``) on
  the reference test's own case (``tests/test_transformers_flashinfer.py:20-48``) and three GQA
  cases at head_dim 128 (bottom-right causal, decode, square causal).
* ``runner_attention.npz`` -- the attention inputs and outputs of ``_GraphQwen3Runner``
  (``cuda_graph_executor.py:104-268``) on a tiny random-weight Qwen3, intercepted with a
  ``TorchFunctionMode`` while the reference's own ``_prefill_forward`` / ``_decode_forward`` /
  ``_verify_forward`` run: prefill SDPA, grouped decode matmuls, verify masked SDPA, per layer;
  plus the greedy token stream of the eager runner (prefill + 8 decode steps).
* ``kv_cache.json`` / ``kv_cache.npz`` -- ``PagedKVCache`` metadata and slot mappings
  (``kv_cache.py:116-149``), block tables produced by ``PageAllocator`` with a shared prefix
  (``page_allocator.py:31-66``), and a store/gather round trip (``kv_cache.py:191-256``).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as F
from torch.overrides import TorchFunctionMode

HERE = os.path.dirname(os.path.abspath(__file__))

# Tiny random-weight Qwen3 used for the runner fixtures (attention shapes at head_dim 128, g=4).
TINY = dict(
    vocab_size=512,
    hidden_size=256,
    intermediate_size=512,
    num_hidden_layers=2,
    num_attention_heads=8,
    num_key_value_heads=2,
    head_dim=128,
    max_position_embeddings=4096,
    rms_norm_eps=1e-6,
)
TINY_SEED = 1234
TINY_MAX_LEN = 64
TINY_PROMPT_LEN = 13
TINY_PREFILL_BOUND = 16
TINY_DECODE_STEPS = 8
VERIFY_K1 = 5
VERIFY_POS0 = 20


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


class _Recorder(TorchFunctionMode):
    """Record the attention calls the reference makes (matmul and SDPA), untouched."""

    def __init__(self):
        super().__init__()
        self.calls = []

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        out = func(*args, **kwargs)
        if func is torch.matmul or func is F.scaled_dot_product_attention:
            self.calls.append((func, [a for a in args], dict(kwargs), out))
        return out


def make_fallback(ref) -> dict:
    fb = ref["fallback"]
    cases = {}
    torch.manual_seed(0)
    b, h, d = 1, 2, 8
    q_len, kv_len = 3, 7
    query = torch.randn(b, h, q_len, d)
    key = torch.randn(b, h, kv_len, d)
    value = torch.randn(b, h, kv_len, d)
    scale = 1.0 / (d**0.5)
    cases["ref_test"] = (query, key, value, scale, True)
    g = torch.Generator().manual_seed(7)
    for name, (hq, hkv, ql, kl, causal) in {
        "gqa_bottom_right": (8, 2, 5, 40, True),
        "gqa_decode": (8, 2, 1, 33, False),
        "gqa_square": (8, 2, 24, 24, True),
    }.items():
        qq = torch.randn(1, hq, ql, 128, generator=g).to(torch.bfloat16)
        kk = torch.randn(1, hkv, kl, 128, generator=g).to(torch.bfloat16)
        vv = torch.randn(1, hkv, kl, 128, generator=g).to(torch.bfloat16)
        cases[name] = (qq, kk, vv, 128**-0.5, causal)
    arrays = {}
    for name, (qq, kk, vv, sc, causal) in cases.items():
        out = fb(qq, kk, vv, sc, causal=causal)
        arrays[f"{name}.query"] = f32(qq)
        arrays[f"{name}.key"] = f32(kk)
        arrays[f"{name}.value"] = f32(vv)
        arrays[f"{name}.out"] = f32(out)
        arrays[f"{name}.scale"] = np.float64(sc)
        arrays[f"{name}.causal"] = np.bool_(causal)
        arrays[f"{name}.bf16"] = np.bool_(qq.dtype == torch.bfloat16)
    np.savez_compressed(os.path.join(HERE, "fallback.npz"), **arrays)
    return arrays


def make_runner(ref) -> dict:
    from transformers import Qwen3Config, Qwen3ForCausalLM

    Runner = ref["runner"]
    torch.manual_seed(TINY_SEED)
    cfg = Qwen3Config(**TINY)
    # transformers 5.x keeps theta in rope_parameters; the reference reads cfg.rope_theta
    # (cuda_graph_executor.py:65), so both are set to the Qwen3 value.
    cfg.rope_parameters = {"rope_type": "default", "rope_theta": 1e6}
    cfg.rope_theta = 1e6
    model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
    runner = Runner(model, TINY_MAX_LEN)
    g = torch.Generator().manual_seed(TINY_SEED + 1)
    prompt = torch.randint(0, TINY["vocab_size"], (TINY_PROMPT_LEN,), generator=g)
    arrays = {"prompt": prompt.numpy()}

    with torch.no_grad():
        # Prefill: the runner pads the prompt into pre_tok[:bound] (cuda_graph_executor.py:156-157).
        runner.pre_tok[:TINY_PROMPT_LEN].copy_(prompt)
        runner.pre_tok[TINY_PROMPT_LEN:TINY_PREFILL_BOUND].zero_()
        rec = _Recorder()
        with rec:
            hid = runner._prefill_forward(TINY_PREFILL_BOUND)
        sdpa = [c for c in rec.calls if c[0] is F.scaled_dot_product_attention]
        assert len(sdpa) == TINY["num_hidden_layers"]
        groups = TINY["num_attention_heads"] // TINY["num_key_value_heads"]
        for li, (_, args, kwargs, out) in enumerate(sdpa):
            q, kk, vv = args[:3]
            arrays[f"prefill.l{li}.q"] = f32(q)  # [nh, t, hd]
            arrays[f"prefill.l{li}.k"] = f32(kk[::groups])  # un-expanded [nkv, t, hd]
            arrays[f"prefill.l{li}.v"] = f32(vv[::groups])
            arrays[f"prefill.l{li}.out"] = f32(out)  # [nh, t, hd]
        logits = (hid[TINY_PROMPT_LEN - 1 : TINY_PROMPT_LEN] @ runner.lm_head.T).float()
        tokens = [int(logits.argmax(-1).item())]
        arrays["prefill.logits"] = f32(logits)

        # Greedy eager decode through the reference's own _decode_forward (bucket = max_len).
        bound = TINY_MAX_LEN
        for step in range(TINY_DECODE_STEPS):
            pos = TINY_PROMPT_LEN + step
            runner.tok_buf.fill_(tokens[-1])
            runner.pos_buf.fill_(pos)
            rec = _Recorder()
            with rec:
                lg = runner._decode_forward(bound)
            tokens.append(int(lg.argmax(-1).item()))
            if step == 0:
                mm = [c for c in rec.calls if c[0] is torch.matmul]
                assert len(mm) == 2 * TINY["num_hidden_layers"]
                for li in range(TINY["num_hidden_layers"]):
                    _, a1, _, _ = mm[2 * li]
                    _, a2, _, o2 = mm[2 * li + 1]
                    arrays[f"decode.l{li}.qg"] = f32(a1[0])  # [nkv, g, hd]
                    arrays[f"decode.l{li}.kt"] = f32(a1[1])  # [nkv, hd, bound]
                    arrays[f"decode.l{li}.vb"] = f32(a2[1])  # [nkv, bound, hd]
                    arrays[f"decode.l{li}.ctx"] = f32(o2)  # [nkv, g, hd]
                arrays["decode.pos"] = np.int64(pos)
                arrays["decode.bound"] = np.int64(bound)
                arrays["decode.logits"] = f32(lg)
        arrays["tokens"] = np.array(tokens, dtype=np.int64)

        # Verify: K+1 tokens at VERIFY_POS0.. over the whole static buffer (:245-268).
        runner.vtok = torch.tensor(tokens[1 : 1 + VERIFY_K1], dtype=torch.long)
        runner.vpos0 = torch.tensor([VERIFY_POS0], dtype=torch.long)
        rec = _Recorder()
        with rec:
            vlog = runner._verify_forward()
        sdpa = [c for c in rec.calls if c[0] is F.scaled_dot_product_attention]
        for li, (_, args, kwargs, out) in enumerate(sdpa):
            q, kk, vv = args[:3]
            arrays[f"verify.l{li}.q"] = f32(q)  # [nh, k1, hd]
            arrays[f"verify.l{li}.k"] = f32(kk[::groups])  # [nkv, max_len, hd]
            arrays[f"verify.l{li}.v"] = f32(vv[::groups])
            arrays[f"verify.l{li}.mask"] = kwargs["attn_mask"].numpy()
            arrays[f"verify.l{li}.out"] = f32(out)
        arrays["verify.pos0"] = np.int64(VERIFY_POS0)
        arrays["verify.tokens"] = runner.vtok.numpy()
        arrays["verify.argmax"] = vlog.argmax(-1).numpy()
    np.savez_compressed(os.path.join(HERE, "runner_attention.npz"), **arrays)
    meta = dict(TINY, seed=TINY_SEED, max_len=TINY_MAX_LEN, prompt_len=TINY_PROMPT_LEN,
                prefill_bound=TINY_PREFILL_BOUND, decode_steps=TINY_DECODE_STEPS,
                verify_k1=VERIFY_K1, verify_pos0=VERIFY_POS0, rope_theta=1e6)
    with open(os.path.join(HERE, "runner_config.json"), "w") as fh:
        json.dump(meta, fh, indent=1)
    return arrays


def make_kv_cache(ref) -> None:
    KVCacheConfig, PagedKVCache = ref["kvcfg"], ref["kv"]
    PageAllocator = ref["alloc"]
    out: dict = {}
    # The reference test's case (tests/test_kv_cache.py:8-19).
    cache = PagedKVCache(KVCacheConfig(num_pages=8, page_size=4))
    bt: list[int] = []
    cache.ensure_capacity(bt, 6)
    md = cache.metadata_for(bt, token_count=6, positions=[0, 3, 4, 5])
    out["ref_test"] = dict(block_table=bt, token_count=6, page_size=4, positions=[0, 3, 4, 5],
                           page_indptr=md.page_indptr, page_indices=md.page_indices,
                           last_page_len=md.last_page_len, slot_mapping=md.slot_mapping)
    # A permuted block table at page size 16 (the paged decode's addressing).
    g = torch.Generator().manual_seed(99)
    perm = torch.randperm(64, generator=g).tolist()
    cache16 = PagedKVCache(KVCacheConfig(num_pages=64, page_size=16))
    positions = list(range(80, 101))
    md = cache16.metadata_for(perm[:7], token_count=101, positions=positions)
    out["perm16"] = dict(block_table=perm[:7], token_count=101, page_size=16, positions=positions,
                         page_indptr=md.page_indptr, page_indices=md.page_indices,
                         last_page_len=md.last_page_len, slot_mapping=md.slot_mapping)
    # Shared prefix: sequence B reuses sequence A's first two pages (incref), as a prefix-cache
    # hit does, then allocates its own tail pages.
    alloc = PageAllocator(num_pages=16, page_size=16)
    a_pages = alloc.alloc(5)
    for p in a_pages[:2]:
        alloc.incref(p)
    b_pages = a_pages[:2] + alloc.alloc(3)
    out["shared_prefix"] = dict(a=a_pages, b=b_pages, ref_count=list(alloc.ref_count),
                                snapshot=alloc.snapshot())
    with open(os.path.join(HERE, "kv_cache.json"), "w") as fh:
        json.dump(out, fh, indent=1)
    # Store / gather round trip on a tensor-backed cache (kv_cache.py:191-256).
    cache_t = PagedKVCache(KVCacheConfig(num_layers=2, num_pages=6, page_size=4, num_kv_heads=2,
                                         head_dim=8, dtype="fp32", device="cpu",
                                         allocate_tensors=True))
    cache_t.kv_cache.zero_()
    key = torch.randn(1, 2, 5, 8, generator=g)
    value = torch.randn(1, 2, 5, 8, generator=g)
    slots = [13, 2, 3, 20, 7]
    cache_t.store_layer_tokens(layer_idx=1, slot_mapping=slots, key=key, value=value)
    k_out, v_out = cache_t.gather_layer_tokens(layer_idx=1, slot_mapping=slots)
    np.savez_compressed(os.path.join(HERE, "kv_cache.npz"), key=f32(key), value=f32(value),
                        slots=np.array(slots), kv_cache=f32(cache_t.kv_cache),
                        k_out=f32(k_out), v_out=f32(v_out))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.reference_src)
    from solort.backends.transformers_flashinfer import _torch_attention_fallback
    from solort.cache.kv_cache import KVCacheConfig, PagedKVCache
    from solort.cache.page_allocator import PageAllocator
    from solort.model.cuda_graph_executor import _GraphQwen3Runner

    ref = dict(fallback=_torch_attention_fallback, runner=_GraphQwen3Runner, kvcfg=KVCacheConfig,
               kv=PagedKVCache, alloc=PageAllocator)
    torch.set_num_threads(1)
    make_fallback(ref)
    make_runner(ref)
    make_kv_cache(ref)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
