"""CPU restatement of the reference's paged-KV addressing (test infrastructure only).

Follows ``src/solort/cache/kv_cache.py``: a per-layer NHD page arena
``[num_pages, 2, page_size, nkv, hd]`` (``:86-100``), FlashInfer-style metadata (``:116-134``),
the logical-position -> physical-slot map (``:136-149``), and the slot-mapped store / gather pair
(``:191-256``). These are the checkers for the device-side block-table reads of the paged decode
and verify kernels and for the paged append kernel.
"""

from __future__ import annotations

import torch


def pages_required(token_count: int, page_size: int) -> int:
    """``ceil(token_count / page_size)`` (``kv_cache.py:102-105``)."""
    if token_count <= 0:
        return 0
    return (token_count + page_size - 1) // page_size


def last_page_len(token_count: int, page_size: int) -> int:
    """Tokens on the last page (``kv_cache.py:151-155``)."""
    if token_count <= 0:
        return 0
    r = token_count % page_size
    return r if r else page_size


def slot_mapping(block_table: list[int], positions: list[int], page_size: int) -> list[int]:
    """``slot = block_table[pos // P] * P + pos % P`` (``kv_cache.py:136-149``).

    Raises ``IndexError`` when a position needs a page the block table does not have.
    """
    slots = []
    for position in positions:
        logical = position // page_size
        if logical >= len(block_table):
            raise IndexError(
                f"position {position} needs logical page {logical}, "
                f"but block table has {len(block_table)} pages"
            )
        slots.append(block_table[logical] * page_size + position % page_size)
    return slots


def metadata_for(
    block_table: list[int], *, token_count: int, page_size: int, positions: list[int] | None = None
) -> dict:
    """``page_indptr / page_indices / last_page_len / slot_mapping`` (``kv_cache.py:116-134``)."""
    active = pages_required(token_count, page_size)
    indices = list(block_table[:active])
    return {
        "page_indptr": [0, len(indices)],
        "page_indices": indices,
        "last_page_len": [last_page_len(token_count, page_size)],
        "slot_mapping": slot_mapping(block_table, positions or [], page_size),
    }


def store_layer_tokens(
    kv_layer: torch.Tensor, slots: list[int], key_nhd: torch.Tensor, value_nhd: torch.Tensor
) -> None:
    """Slot-mapped write of ``[tokens, nkv, hd]`` K/V into one layer's
    ``[num_pages, 2, P, nkv, hd]`` arena (the per-token loop of ``kv_cache.py:227-235``)."""
    page_size = kv_layer.shape[2]
    for i, slot in enumerate(slots):
        kv_layer[slot // page_size, 0, slot % page_size].copy_(key_nhd[i])
        kv_layer[slot // page_size, 1, slot % page_size].copy_(value_nhd[i])


def gather_layer_tokens(kv_layer: torch.Tensor, slots: list[int]):
    """Read ``[tokens, nkv, hd]`` K and V at physical slots (``kv_cache.py:237-256``)."""
    num_pages, _, page_size, nkv, hd = kv_layer.shape
    flat_k = kv_layer[:, 0].reshape(-1, nkv, hd)
    flat_v = kv_layer[:, 1].reshape(-1, nkv, hd)
    index = torch.as_tensor(slots, dtype=torch.long, device=kv_layer.device)
    return flat_k.index_select(0, index).clone(), flat_v.index_select(0, index).clone()


def dense_from_block_table(kv_layer: torch.Tensor, block_table: list[int], n_tokens: int):
    """Dense ``[n_tokens, nkv, hd]`` K/V of one sequence: slot mapping of positions
    ``0..n_tokens-1`` followed by the gather. This is how the paged oracle builds the input of
    ``attention_fp32``."""
    page_size = kv_layer.shape[2]
    slots = slot_mapping(block_table, list(range(n_tokens)), page_size)
    return gather_layer_tokens(kv_layer, slots)
