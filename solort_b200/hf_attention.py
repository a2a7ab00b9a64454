"""Hugging Face ``AttentionInterface`` callable backed by the engine (the paged bridge's hook).

Drop-in for ``solort_flashinfer_attention_forward`` (``src/solort/backends/
transformers_flashinfer.py:68-129``): same signature, same layouts in and out, same semantics --
``q_len == 1`` is decode over every cached key, ``q_len > 1`` is causal prefill with bottom-right
alignment when the cache already holds keys (``:182-193``). Registration mirrors
``register_solort_flashinfer_attention`` (``:37-56``): call ``register_solort_b200_attention()``
and load the model with ``attn_implementation=ATTENTION_NAME``.

SoloRT's paged KV (``src/solort/cache/kv_cache.py``): inside ``solort_kv_write_context(kv_cache,
slot_mapping)`` -- the context manager the paged executor wraps every forward in
(``transformers_flashinfer.py:24-34``, ``src/solort/model/executor.py:705-718``) -- each layer's
new K / V rows are mirrored into ``kv_cache.kv_cache[layer_idx]`` at the batch's slots, as the
reference's ``_mirror_to_solort_kv`` -> ``PagedKVCache.store_layer_tokens`` does
(``transformers_flashinfer.py:93,205-220``, ``kv_cache.py:191-235``), but as one
``torch.ops.solort_attn.kv_store`` launch instead of a Python loop over tokens. When the context
also carries the sequence's ``block_table`` (``Sequence.block_table``, the pages the allocator and
prefix cache handed out), decode and verify read SoloRT's own paged arena through that block table
(``torch.ops.solort_attn.gqa_decode_paged``) instead of HF's dense cache: the "tensor-backed paged
runner" the reference lists as pending (``executor.py:841-847``). Passing ``block_table`` states
that positions ``0 .. kv_len - 1`` of the sequence are in the arena once this forward's rows are
stored, which holds when every forward of the sequence ran inside the context.

Unlike the reference bridge there is no silent fallback (``:110-112, 127-129``): unsupported
inputs raise.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass
from typing import Any

import torch

from solort_b200 import ops

ATTENTION_NAME = "solort_b200"
MAX_PAGED_ROWS = 32  # query rows per KV head the decode / verify kernel handles in one CTA


@dataclass
class AttentionStats:
    prefill_calls: int = 0
    decode_calls: int = 0
    paged_calls: int = 0
    mirrored_tokens: int = 0
    mirror_skipped: int = 0


_STATS = AttentionStats()
_REGISTERED = False
_KV_CONTEXT: dict[str, Any] | None = None
_POS_BUF: dict[torch.device, torch.Tensor] = {}


@contextmanager
def solort_kv_write_context(kv_cache: Any | None, slot_mapping: list[int] | None,
                            block_table: list[int] | None = None):
    """Expose the current forward's SoloRT KV destination (``slot_mapping``: one physical slot per
    new token, ``PagedKVCache.slot_mapping``) and, optionally, the sequence's ``block_table`` to
    the attention callable -- the reference's ``solort_kv_write_context``
    (``transformers_flashinfer.py:24-34``) plus the block table the paged reads need."""
    global _KV_CONTEXT
    previous = _KV_CONTEXT
    _KV_CONTEXT = {"kv_cache": kv_cache, "slot_mapping": list(slot_mapping or []),
                   "block_table": None if block_table is None else list(block_table),
                   "device_tensors": {}}
    try:
        yield
    finally:
        _KV_CONTEXT = previous


def register_solort_b200_attention() -> None:
    """Register the callable with transformers under ``ATTENTION_NAME`` (idempotent)."""
    global _REGISTERED
    if _REGISTERED:
        return
    try:
        from transformers import AttentionInterface
    except ImportError:  # older transformers
        from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS as AttentionInterface
    AttentionInterface.register(ATTENTION_NAME, solort_b200_attention_forward)
    _REGISTERED = True


def attention_snapshot() -> dict[str, int | str]:
    return {"attention_backend": ATTENTION_NAME, "prefill_calls": _STATS.prefill_calls,
            "decode_calls": _STATS.decode_calls, "paged_calls": _STATS.paged_calls,
            "mirrored_tokens": _STATS.mirrored_tokens, "mirror_skipped": _STATS.mirror_skipped}


def _context_tensor(name: str, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """The context's list ``name`` as a device tensor, copied once per forward and device."""
    cache = _KV_CONTEXT["device_tensors"]
    key = (name, device)
    t = cache.get(key)
    if t is None:
        t = cache[key] = torch.as_tensor(_KV_CONTEXT[name], dtype=dtype, device=device)
    return t


def _position_buffer(device: torch.device) -> torch.Tensor:
    """One int64 device word per device for the decode position (no per-call allocation)."""
    buf = _POS_BUF.get(device)
    if buf is None:
        buf = _POS_BUF[device] = torch.zeros(1, dtype=torch.int64, device=device)
    return buf


def _arena_of(kv_cache: Any):
    arena = getattr(kv_cache, "kv_cache", None)
    return arena if isinstance(arena, torch.Tensor) else None


def _count(kv_cache: Any, attr: str, n: int) -> None:
    if hasattr(kv_cache, attr):
        setattr(kv_cache, attr, getattr(kv_cache, attr) + n)


def _mirror_to_solort_kv(module: Any, key: torch.Tensor, value: torch.Tensor) -> int | None:
    """Store this forward's K / V rows into the context's paged arena, with the skip rules of
    ``PagedKVCache.store_layer_tokens`` (``kv_cache.py:206-229``): no layer index, no slots or no
    tensors, a layer out of range, batch != 1 or mismatched heads / head dim skip the store; the
    last ``min(len(slots), kv_len)`` tokens go to the last slots. Returns the layer index stored
    to, or None when skipped (or when no context is active)."""
    if _KV_CONTEXT is None or _KV_CONTEXT.get("kv_cache") is None:
        return None
    kv_cache = _KV_CONTEXT["kv_cache"]
    arena = _arena_of(kv_cache)
    layer_idx = getattr(module, "layer_idx", None)
    slots = _KV_CONTEXT["slot_mapping"]
    ok = (layer_idx is not None and slots and arena is not None and 0 <= layer_idx < arena.shape[0]
          and key.shape[0] == 1 and value.shape[0] == 1
          and key.shape[1] == arena.shape[4] and value.shape[1] == arena.shape[4]
          and key.shape[-1] == arena.shape[5] and value.shape[-1] == arena.shape[5])
    token_count = min(len(slots), key.shape[-2], value.shape[-2]) if ok else 0
    if token_count <= 0:
        _STATS.mirror_skipped += 1
        _count(kv_cache, "mirror_skipped", 1)
        return None
    slot_t = _context_tensor("slot_mapping", torch.int64, key.device)[-token_count:]
    ops.kv_store(key[0, :, -token_count:].transpose(0, 1), value[0, :, -token_count:].transpose(0, 1),
                 slot_t, arena[layer_idx])
    _STATS.mirrored_tokens += token_count
    _count(kv_cache, "mirrored_tokens", token_count)
    return layer_idx


def solort_b200_attention_forward(
    module: Any,
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    attention_mask: torch.Tensor | None,
    scaling: float,
    dropout: float = 0.0,
    sliding_window: int | None = None,
    **kwargs: Any,
) -> tuple[torch.Tensor, None]:
    """``query [1, h, q, d]``, ``key/value [1, hkv, kv, d]`` (HF layout) -> ``([1, q, h, d], None)``."""
    del attention_mask, kwargs
    if query.shape[0] != 1:
        raise RuntimeError("solort_b200 attention currently supports batch_size=1")
    if query.device.type != "cuda":
        raise RuntimeError("solort_b200 attention requires CUDA tensors")
    if dropout:
        raise RuntimeError("solort_b200 attention does not implement dropout")
    if sliding_window:
        raise RuntimeError("solort_b200 attention does not implement sliding windows")
    q_len, kv_len = query.shape[2], key.shape[2]
    if q_len > kv_len:
        raise RuntimeError(f"query length {q_len} exceeds key length {kv_len}")
    layer = _mirror_to_solort_kv(module, key, value)
    groups = query.shape[1] // key.shape[1]
    if (layer is not None and _KV_CONTEXT.get("block_table") is not None
            and q_len * groups <= MAX_PAGED_ROWS):
        # decode / verify from SoloRT's own paged KV through the sequence's block table
        arena = _arena_of(_KV_CONTEXT["kv_cache"])[layer]
        bt = _context_tensor("block_table", torch.int32, query.device).view(1, -1)
        pos = _position_buffer(query.device)
        pos.fill_(kv_len - q_len)
        out = ops.gqa_decode_paged(query.transpose(1, 2), arena, bt, pos, max_kv_len=kv_len,
                                   scale=float(scaling))
        _STATS.paged_calls += 1
        return out, None
    if q_len == 1:
        pos = _position_buffer(query.device)
        pos.fill_(kv_len - 1)
        out = ops.gqa_decode(query.transpose(1, 2), key[0], value[0], pos, kv_layout="HND",
                             scale=float(scaling))
        _STATS.decode_calls += 1
        return out, None
    q = query[0].transpose(0, 1)  # [q, h, d] view: token stride d, head stride q*d
    k = key[0].transpose(0, 1)
    v = value[0].transpose(0, 1)
    out = ops.gqa_prefill(q, k, v, causal=True, scale=float(scaling))
    _STATS.prefill_calls += 1
    return out[None], None
