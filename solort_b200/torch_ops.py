"""The engine's attention ops registered with torch as ``torch.ops.solort_attn.*``.

This is the torch custom-op layer between SoloRT's Python host code and the C ABI
(``include/solort_attn.h``). Each op writes into caller-provided tensors (``out``, ``workspace``,
the paged arena) and returns nothing, so it allocates nothing and can sit inside the reference's
CUDA-graph captures (``src/solort/model/cuda_graph_executor.py:137-147,195-207,272-285``): a
captured call replays with the positions it reads from device memory. Each op has a fake (meta)
implementation that checks shapes and dtypes without touching data, so it also traces under
``FakeTensorMode``. Only a CUDA implementation is registered: CPU tensors raise, there is no
fallback.

Ops (schemas below):
* ``gqa_decode``: decode (``q_len == 1``, ``cuda_graph_executor.py:168,180-184``) and K-token
  verify (``q_len == K + 1``, ``:250,261-263``) over one layer's static K/V buffer.
* ``gqa_decode_paged``: the same over one layer of SoloRT's paged arena and a block table
  (``src/solort/cache/kv_cache.py:86-100,136-149``).
* ``gqa_prefill``: causal prefill (``cuda_graph_executor.py:124-130``), bottom-right aligned when
  the keys outnumber the queries (``src/solort/backends/transformers_flashinfer.py:182-193``).
* ``gqa_decode_partial`` and ``lse_merge``: the per-shard partial ``(O, LSE)`` of a
  sequence-sharded decode and the merge of several partials (no reference counterpart).
* ``kv_store``: the slot-mapped K/V store of ``PagedKVCache.store_layer_tokens``
  (``kv_cache.py:191-235``).

Registration uses ``torch.library.Library`` directly (a C++ dispatcher entry with a Python
kernel, ~3 us per call) rather than ``torch.library.custom_op`` (~18 us per call).
"""

from __future__ import annotations

import torch

from solort_b200 import _calls

NAMESPACE = "solort_attn"

SCHEMAS = {
    "gqa_decode": (
        "gqa_decode(Tensor q, Tensor k_cache, Tensor v_cache, Tensor q_pos, Tensor(a!) out, "
        "Tensor(b!) workspace, str kv_layout=\"NHD\", float? scale=None, int max_kv_len=0, "
        "Tensor? q_lens=None, int num_splits=0, bool stable_prefix=False) -> ()"),
    "gqa_decode_paged": (
        "gqa_decode_paged(Tensor q, Tensor kv_pages, Tensor block_table, Tensor q_pos, "
        "Tensor(a!) out, Tensor(b!) workspace, int max_kv_len, float? scale=None, "
        "Tensor? q_lens=None, int num_splits=0, bool stable_prefix=False) -> ()"),
    "gqa_prefill": (
        "gqa_prefill(Tensor q, Tensor k, Tensor v, Tensor(a!) out, bool causal=True, "
        "float? scale=None) -> ()"),
    "gqa_decode_partial": (
        "gqa_decode_partial(Tensor q, Tensor k_cache, Tensor v_cache, Tensor q_pos, "
        "Tensor(a!) out_f32, Tensor(b!) lse_out, Tensor(c!) workspace, int kv_pos_offset=0, "
        "str kv_layout=\"NHD\", float? scale=None, int max_kv_len=0, int num_splits=0) -> ()"),
    "lse_merge": "lse_merge(Tensor o_parts, Tensor lse_parts, Tensor(a!) out) -> ()",
    "kv_store": "kv_store(Tensor key, Tensor value, Tensor slots, Tensor(a!) kv_pages) -> ()",
}

_LIB = torch.library.Library(NAMESPACE, "DEF")
for _schema in SCHEMAS.values():
    _LIB.define(_schema)


# ---- CUDA implementations: one C-ABI call each ----

def _gqa_decode(q, k_cache, v_cache, q_pos, out, workspace, kv_layout="NHD", scale=None,
                max_kv_len=0, q_lens=None, num_splits=0, stable_prefix=False):
    _calls.decode_static_into(q, k_cache, v_cache, q_pos, out, workspace, kv_layout, scale,
                              max_kv_len, q_lens, num_splits, stable_prefix)


def _gqa_decode_paged(q, kv_pages, block_table, q_pos, out, workspace, max_kv_len, scale=None,
                      q_lens=None, num_splits=0, stable_prefix=False):
    _calls.decode_paged_into(q, kv_pages, block_table, q_pos, out, workspace, max_kv_len, scale,
                             q_lens, num_splits, stable_prefix)


def _gqa_prefill(q, k, v, out, causal=True, scale=None):
    _calls.prefill_into(q, k, v, out, causal, scale)


def _gqa_decode_partial(q, k_cache, v_cache, q_pos, out_f32, lse_out, workspace,
                        kv_pos_offset=0, kv_layout="NHD", scale=None, max_kv_len=0, num_splits=0):
    _calls.decode_partial_into(q, k_cache, v_cache, q_pos, out_f32, lse_out, workspace,
                               kv_pos_offset, kv_layout, scale, max_kv_len, num_splits)


def _lse_merge(o_parts, lse_parts, out):
    _calls.lse_merge_into(o_parts, lse_parts, out)


def _kv_store(key, value, slots, kv_pages):
    _calls.kv_store_into(key, value, slots, kv_pages)


for _name, _fn in (("gqa_decode", _gqa_decode), ("gqa_decode_paged", _gqa_decode_paged),
                   ("gqa_prefill", _gqa_prefill), ("gqa_decode_partial", _gqa_decode_partial),
                   ("lse_merge", _lse_merge), ("kv_store", _kv_store)):
    _LIB.impl(_name, _fn, "CUDA")


# ---- fake (meta) implementations: the same shape / dtype rules, no data access ----

def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(msg)


def _check_q(q) -> tuple[int, int, int, int]:
    _need(q.dtype == torch.bfloat16, "q must be bf16")
    _need(q.dim() == 4 and q.shape[-1] == _calls.HEAD_DIM,
          "q must be [batch, q_len, num_qo_heads, 128]")
    return tuple(q.shape)


def _fake_decode(q, k_cache, v_cache, q_pos, out, workspace, kv_layout="NHD", scale=None,
                 max_kv_len=0, q_lens=None, num_splits=0, stable_prefix=False):
    B, T, H, _ = _check_q(q)
    _need(out.shape == q.shape and out.dtype == torch.bfloat16, "out must match q (bf16)")
    _need(k_cache.dim() == 3 and k_cache.shape == v_cache.shape and
          k_cache.dtype == torch.bfloat16, "k_cache / v_cache must be equal 3-D bf16 tensors")
    _need(kv_layout in ("NHD", "HND"), "kv_layout must be 'NHD' or 'HND'")
    nkv = k_cache.shape[1] if kv_layout == "NHD" else k_cache.shape[0]
    _need(H % nkv == 0, "num_qo_heads must be a multiple of num_kv_heads")
    _need(q_pos.dtype == torch.int64 and q_pos.numel() == B, "q_pos must be int64 [batch]")


def _fake_decode_paged(q, kv_pages, block_table, q_pos, out, workspace, max_kv_len, scale=None,
                       q_lens=None, num_splits=0, stable_prefix=False):
    B, T, H, _ = _check_q(q)
    _need(out.shape == q.shape and out.dtype == torch.bfloat16, "out must match q (bf16)")
    _need(kv_pages.dim() == 5 and kv_pages.shape[1] == 2 and kv_pages.shape[-1] == 128,
          "kv_pages must be [num_pages, 2, page_size, nkv, 128]")
    _need(block_table.dtype == torch.int32 and block_table.dim() == 2 and
          block_table.shape[0] == B, "block_table must be int32 [batch, max_pages]")
    _need(max_kv_len <= block_table.shape[1] * kv_pages.shape[2],
          "max_kv_len exceeds the pages a block-table row can hold")
    _need(q_pos.dtype == torch.int64 and q_pos.numel() == B, "q_pos must be int64 [batch]")


def _fake_prefill(q, k, v, out, causal=True, scale=None):
    _need(q.dim() == 3 and k.dim() == 3 and k.shape == v.shape, "q [T, nh, 128], k / v [S, nkv, 128]")
    _need(out.shape == q.shape and out.dtype == torch.bfloat16, "out must match q (bf16)")
    _need(q.shape[1] % k.shape[1] == 0, "num_qo_heads must be a multiple of num_kv_heads")
    _need(not causal or q.shape[0] <= k.shape[0], "causal prefill needs q_len <= kv_len")


def _fake_decode_partial(q, k_cache, v_cache, q_pos, out_f32, lse_out, workspace,
                         kv_pos_offset=0, kv_layout="NHD", scale=None, max_kv_len=0, num_splits=0):
    B, T, H, D = _check_q(q)
    _need(tuple(out_f32.shape) == (B, T, H, D) and out_f32.dtype == torch.float32,
          "out_f32 must be fp32 [batch, q_len, num_qo_heads, 128]")
    _need(tuple(lse_out.shape) == (B, T, H) and lse_out.dtype == torch.float32,
          "lse_out must be fp32 [batch, q_len, num_qo_heads]")


def _fake_lse_merge(o_parts, lse_parts, out):
    _need(o_parts.dim() == 5 and o_parts.dtype == torch.float32, "o_parts must be fp32 5-D")
    _need(tuple(lse_parts.shape) == tuple(o_parts.shape[:4]), "lse_parts must be [R, B, T, H]")
    _need(tuple(out.shape) == tuple(o_parts.shape[1:]) and out.dtype == torch.bfloat16,
          "out must be bf16 [batch, q_len, num_qo_heads, 128]")


def _fake_kv_store(key, value, slots, kv_pages):
    _need(key.dim() == 3 and key.shape == value.shape, "key / value must be [tokens, nkv, 128]")
    _need(slots.dtype == torch.int64 and slots.numel() == key.shape[0],
          "slots must be int64 [tokens]")
    _need(kv_pages.dim() == 5 and kv_pages.shape[1] == 2 and kv_pages.shape[3] == key.shape[1],
          "kv_pages must be [num_pages, 2, page_size, nkv, 128]")


for _name, _fn in (("gqa_decode", _fake_decode), ("gqa_decode_paged", _fake_decode_paged),
                   ("gqa_prefill", _fake_prefill), ("gqa_decode_partial", _fake_decode_partial),
                   ("lse_merge", _fake_lse_merge), ("kv_store", _fake_kv_store)):
    torch.library.register_fake(f"{NAMESPACE}::{_name}", _fn, lib=_LIB)

OPS = tuple(SCHEMAS)
