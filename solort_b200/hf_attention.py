"""Hugging Face ``AttentionInterface`` callable backed by the engine (the paged bridge's hook).

Drop-in for ``solort_flashinfer_attention_forward`` (``src/solort/backends/
transformers_flashinfer.py:68-129``): same signature, same layouts in and out, same semantics --
``q_len == 1`` is decode over every cached key, ``q_len > 1`` is causal prefill with bottom-right
alignment when the cache already holds keys (``:182-193``). Registration mirrors
``register_solort_flashinfer_attention`` (``:37-56``): call ``register_solort_b200_attention()``
and load the model with ``attn_implementation=ATTENTION_NAME``.

Unlike the reference bridge there is no silent fallback (``:110-112, 127-129``): unsupported
inputs raise.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

import torch

from solort_b200 import ops

ATTENTION_NAME = "solort_b200"


@dataclass
class AttentionStats:
    prefill_calls: int = 0
    decode_calls: int = 0


_STATS = AttentionStats()
_REGISTERED = False


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
            "decode_calls": _STATS.decode_calls}


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
    del attention_mask, module, kwargs
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
    if q_len == 1:
        q = query.transpose(1, 2)  # [1, 1, h, d], a view
        pos = torch.full((1,), kv_len - 1, dtype=torch.int64, device=query.device)
        out = ops.gqa_decode(q, key[0], value[0], pos, kv_layout="HND", scale=float(scaling))
        _STATS.decode_calls += 1
        return out, None
    q = query[0].transpose(0, 1)  # [q, h, d] view: token stride d, head stride q*d
    k = key[0].transpose(0, 1)
    v = value[0].transpose(0, 1)
    out = ops.gqa_prefill(q, k, v, causal=True, scale=float(scaling))
    _STATS.prefill_calls += 1
    return out[None], None
