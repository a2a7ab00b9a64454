"""C-ABI call builders shared by the torch op registrations and the torch-facing helpers.

Each ``*_into`` function checks its tensors, packs the argument struct of ``include/solort_attn.h``
and makes one library call on ``torch.cuda.current_stream()``; it writes only the output and
workspace tensors it is given and allocates nothing. Errors raise ``RuntimeError``.
"""

from __future__ import annotations

import ctypes

import torch

from solort_b200 import _lib

HEAD_DIM = 128


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


# torch's raw getter of the current stream handle: the same value as
# ``torch.cuda.current_stream(device).cuda_stream`` (the capture stream while a graph is captured),
# without building a Stream object, which costs ~2 us of host time per call.
_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream_at(index: int) -> int:
    if _RAW_STREAM is not None:
        return _RAW_STREAM(index)
    return torch.cuda.current_stream(index).cuda_stream


def _stream(device: torch.device) -> int:
    return _stream_at(device.index if device.index is not None else torch.cuda.current_device())


def _check_cuda(name: str, t: torch.Tensor, dtype: torch.dtype | None = None) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise RuntimeError(f"{name} must be {dtype}, got {t.dtype}")


def _decode_args(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    q_pos: torch.Tensor,
    *,
    stride_token: int,
    stride_head: int,
    stride_page: int,
    kv_capacity: int,
    num_kv_heads: int,
    block_table: torch.Tensor | None,
    page_size: int,
    num_pages: int,
    scale: float | None,
    max_kv_len: int,
    out: torch.Tensor | None,
    out_f32: torch.Tensor | None,
    lse_out: torch.Tensor | None,
    q_lens: torch.Tensor | None,
    kv_pos_offset: int,
    num_splits: int,
    stable_prefix: bool = False,
) -> _lib.SolortDecodeArgs:
    _check_cuda("q", q, torch.bfloat16)
    if q.dim() != 4 or q.shape[-1] != HEAD_DIM or q.stride(-1) != 1:
        raise RuntimeError("q must be [batch, q_len, num_qo_heads, 128] with a contiguous head dim")
    _check_cuda("q_pos", q_pos, torch.int64)
    B, T, H, D = q.shape
    a = _lib.SolortDecodeArgs()
    a.q = q.data_ptr()
    a.q_stride_batch, a.q_stride_token, a.q_stride_head = q.stride(0), q.stride(1), q.stride(2)
    if out is not None:
        a.out = out.data_ptr()
        a.out_stride_batch, a.out_stride_token, a.out_stride_head = out.stride(0), out.stride(1), out.stride(2)
    a.out_f32 = _ptr(out_f32)
    a.lse_out = _ptr(lse_out)
    a.k, a.v = k.data_ptr(), v.data_ptr()
    a.kv_stride_token, a.kv_stride_head, a.kv_stride_page = stride_token, stride_head, stride_page
    a.kv_capacity = kv_capacity
    a.block_table = _ptr(block_table)
    a.block_table_stride = block_table.stride(0) if block_table is not None else 0
    a.page_size = page_size
    a.num_pages = num_pages
    a.q_pos = q_pos.data_ptr()
    a.q_lens = _ptr(q_lens)
    a.kv_pos_offset = int(kv_pos_offset)
    a.batch, a.q_len, a.num_qo_heads, a.num_kv_heads, a.head_dim = B, T, H, num_kv_heads, D
    a.max_kv_len = int(max_kv_len)
    a.scale = float(D ** -0.5 if scale is None else scale)
    a.num_splits = int(num_splits)
    a.flags = _lib.DECODE_STABLE_PREFIX if stable_prefix else 0
    return a


def _run_decode(a: _lib.SolortDecodeArgs, device: torch.device, workspace: torch.Tensor | None):
    """Attach ``workspace`` (when the call needs one) and launch. A missing or short workspace is
    the library's SOLORT_ERR_WORKSPACE, raised as ``RuntimeError``."""
    lib = _lib.load()
    if workspace is not None and workspace.numel() > 0:
        _check_cuda("workspace", workspace)
        a.workspace = workspace.data_ptr()
        a.workspace_bytes = workspace.numel() * workspace.element_size()
    _lib.check(lib.solort_attn_decode(ctypes.byref(a), ctypes.c_void_p(_stream(device))),
               "solort_attn_decode")


def decode_workspace_needed(a: _lib.SolortDecodeArgs) -> int:
    need = ctypes.c_size_t(0)
    _lib.check(_lib.load().solort_attn_decode_workspace_size(ctypes.byref(a), ctypes.byref(need)),
               "solort_attn_decode_workspace_size")
    return int(need.value)


def _static_kv(k_cache: torch.Tensor, v_cache: torch.Tensor, kv_layout: str):
    _check_cuda("k_cache", k_cache, torch.bfloat16)
    _check_cuda("v_cache", v_cache, torch.bfloat16)
    if k_cache.shape != v_cache.shape or k_cache.stride() != v_cache.stride():
        raise RuntimeError("k_cache and v_cache must have the same shape and strides")
    if k_cache.dim() != 3 or k_cache.shape[-1] != HEAD_DIM or k_cache.stride(-1) != 1:
        raise RuntimeError("static KV must be 3-D with a contiguous head dim of 128")
    if kv_layout == "NHD":
        cap, nkv = k_cache.shape[0], k_cache.shape[1]
        st, sh = k_cache.stride(0), k_cache.stride(1)
    elif kv_layout == "HND":
        nkv, cap = k_cache.shape[0], k_cache.shape[1]
        sh, st = k_cache.stride(0), k_cache.stride(1)
    else:
        raise RuntimeError(f"kv_layout must be 'NHD' or 'HND', got {kv_layout!r}")
    return cap, nkv, st, sh


def decode_workspace_bytes(
    batch: int, q_len: int, num_qo_heads: int, num_kv_heads: int, max_kv_len: int,
    *, kv_capacity: int | None = None, page_size: int = 0, num_splits: int = 0,
) -> int:
    """Workspace bytes a decode call with these sizes needs on the current device."""
    a = _lib.SolortDecodeArgs()
    a.batch, a.q_len, a.num_qo_heads, a.num_kv_heads, a.head_dim = (
        batch, q_len, num_qo_heads, num_kv_heads, HEAD_DIM)
    a.max_kv_len = max_kv_len
    a.kv_capacity = kv_capacity if kv_capacity is not None else max_kv_len
    if page_size:
        a.block_table = 1  # any non-null pointer selects the paged plan
        a.page_size = page_size
        a.num_pages = 1
    a.num_splits = num_splits
    need = ctypes.c_size_t(0)
    _lib.check(_lib.load().solort_attn_decode_workspace_size(ctypes.byref(a), ctypes.byref(need)),
               "solort_attn_decode_workspace_size")
    return int(need.value)




def decode_static_into(q, k_cache, v_cache, q_pos, out, workspace, kv_layout: str,
                       scale: float | None, max_kv_len: int, q_lens, num_splits: int,
                       stable_prefix: bool) -> None:
    """``out = attention(q, static K/V)``: the body of ``solort_attn::gqa_decode``."""
    cap, nkv, st, sh = _static_kv(k_cache, v_cache, kv_layout)
    if q_pos.numel() != q.shape[0]:
        raise RuntimeError(f"q_pos has {q_pos.numel()} entries for batch {q.shape[0]}")
    _check_out_like(out, q)
    a = _decode_args(
        q, k_cache, v_cache, q_pos, stride_token=st, stride_head=sh, stride_page=0,
        kv_capacity=cap, num_kv_heads=nkv, block_table=None, page_size=0, num_pages=0,
        scale=scale, max_kv_len=max_kv_len or cap, out=out, out_f32=None, lse_out=None,
        q_lens=q_lens, kv_pos_offset=0, num_splits=num_splits, stable_prefix=stable_prefix)
    _run_decode(a, q.device, workspace)


def _paged_geometry(q, kv_pages, block_table, max_kv_len):
    _check_cuda("kv_pages", kv_pages, torch.bfloat16)
    _check_cuda("block_table", block_table, torch.int32)
    if kv_pages.dim() != 5 or kv_pages.shape[1] != 2 or kv_pages.shape[-1] != HEAD_DIM:
        raise RuntimeError("kv_pages must be [num_pages, 2, page_size, nkv, 128]")
    if kv_pages.stride(-1) != 1:
        raise RuntimeError("kv_pages must have a contiguous head dim")
    if block_table.dim() != 2 or block_table.stride(1) != 1 or block_table.shape[0] != q.shape[0]:
        raise RuntimeError("block_table must be [batch, max_pages] with contiguous rows")
    num_pages, _, P, nkv, _ = kv_pages.shape
    if max_kv_len > block_table.shape[1] * P:
        raise RuntimeError("max_kv_len exceeds the pages a block-table row can hold")
    return num_pages, P, nkv


def decode_paged_into(q, kv_pages, block_table, q_pos, out, workspace, max_kv_len: int,
                      scale: float | None, q_lens, num_splits: int, stable_prefix: bool) -> None:
    """``out = attention(q, paged K/V)``: the body of ``solort_attn::gqa_decode_paged``."""
    num_pages, P, nkv = _paged_geometry(q, kv_pages, block_table, max_kv_len)
    _check_out_like(out, q)
    a = _decode_args(
        q, kv_pages[:, 0], kv_pages[:, 1], q_pos, stride_token=kv_pages.stride(2),
        stride_head=kv_pages.stride(3), stride_page=kv_pages.stride(0), kv_capacity=0,
        num_kv_heads=nkv, block_table=block_table, page_size=P, num_pages=num_pages, scale=scale,
        max_kv_len=max_kv_len, out=out, out_f32=None, lse_out=None, q_lens=q_lens,
        kv_pos_offset=0, num_splits=num_splits, stable_prefix=stable_prefix)
    _run_decode(a, q.device, workspace)


def decode_partial_into(q, k_cache, v_cache, q_pos, out_f32, lse_out, workspace,
                        kv_pos_offset: int, kv_layout: str, scale: float | None,
                        max_kv_len: int, num_splits: int) -> None:
    """Partial ``(O fp32, LSE)`` over one key shard: the body of ``solort_attn::gqa_decode_partial``."""
    cap, nkv, st, sh = _static_kv(k_cache, v_cache, kv_layout)
    B, T, H, D = q.shape
    _check_cuda("out_f32", out_f32, torch.float32)
    _check_cuda("lse_out", lse_out, torch.float32)
    if tuple(out_f32.shape) != (B, T, H, D) or not out_f32.is_contiguous():
        raise RuntimeError(f"out_f32 must be a contiguous [{B}, {T}, {H}, {D}] tensor")
    if tuple(lse_out.shape) != (B, T, H) or not lse_out.is_contiguous():
        raise RuntimeError(f"lse_out must be a contiguous [{B}, {T}, {H}] tensor")
    a = _decode_args(
        q, k_cache, v_cache, q_pos, stride_token=st, stride_head=sh, stride_page=0,
        kv_capacity=cap, num_kv_heads=nkv, block_table=None, page_size=0, num_pages=0,
        scale=scale, max_kv_len=max_kv_len or cap, out=None, out_f32=out_f32, lse_out=lse_out,
        q_lens=None, kv_pos_offset=kv_pos_offset, num_splits=num_splits)
    _run_decode(a, q.device, workspace)


def lse_merge_into(o_parts, lse_parts, out, out_f32=None, lse_out=None) -> None:
    """Merge of ``R`` partials: the body of ``solort_attn::lse_merge`` (bf16 ``out``), or the
    fp32 ``(out_f32, lse_out)`` form when those are given."""
    _check_cuda("o_parts", o_parts, torch.float32)
    _check_cuda("lse_parts", lse_parts, torch.float32)
    if o_parts.dim() != 5 or o_parts.shape[-1] != HEAD_DIM:
        raise RuntimeError("o_parts must be [parts, batch, q_len, num_qo_heads, 128]")
    R, B, T, H, D = o_parts.shape
    if tuple(lse_parts.shape) != (R, B, T, H):
        raise RuntimeError("lse_parts must be [parts, batch, q_len, num_qo_heads]")
    if not o_parts[0].is_contiguous() or not lse_parts[0].is_contiguous():
        raise RuntimeError("each part of o_parts / lse_parts must be contiguous")
    m = _lib.SolortMergeArgs()
    m.o_parts, m.part_stride = o_parts.data_ptr(), o_parts.stride(0)
    m.lse_parts, m.lse_part_stride = lse_parts.data_ptr(), lse_parts.stride(0)
    m.num_parts, m.batch, m.q_len, m.num_qo_heads, m.head_dim = R, B, T, H, D
    if out_f32 is not None:
        m.out_f32, m.lse_out = out_f32.data_ptr(), lse_out.data_ptr()
    else:
        _check_cuda("out", out, torch.bfloat16)
        if tuple(out.shape) != (B, T, H, D) or out.stride(-1) != 1:
            raise RuntimeError(f"out must be [{B}, {T}, {H}, {D}] with a contiguous head dim")
        m.out = out.data_ptr()
        m.out_stride_batch, m.out_stride_token, m.out_stride_head = out.stride(0), out.stride(1), out.stride(2)
    _lib.check(_lib.load().solort_attn_lse_merge(ctypes.byref(m), ctypes.c_void_p(_stream(o_parts.device))),
               "solort_attn_lse_merge")


def prefill_into(q, k, v, out, causal: bool, scale: float | None) -> None:
    """Causal (or full) GQA prefill: the body of ``solort_attn::gqa_prefill``."""
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out)):
        _check_cuda(name, t, torch.bfloat16)
        if t.dim() != 3 or t.shape[-1] != HEAD_DIM or t.stride(-1) != 1:
            raise RuntimeError(f"{name} must be [tokens, heads, 128] with a contiguous head dim")
    if k.shape != v.shape or k.stride() != v.stride():
        raise RuntimeError("k and v must have the same shape and strides")
    if out.shape != q.shape:
        raise RuntimeError("out must have the shape of q")
    T, H, D = q.shape
    a = _lib.SolortPrefillArgs()
    a.q, a.q_stride_token, a.q_stride_head = q.data_ptr(), q.stride(0), q.stride(1)
    a.k, a.v = k.data_ptr(), v.data_ptr()
    a.kv_stride_token, a.kv_stride_head = k.stride(0), k.stride(1)
    a.out, a.out_stride_token, a.out_stride_head = out.data_ptr(), out.stride(0), out.stride(1)
    a.q_len, a.kv_len, a.num_qo_heads, a.num_kv_heads, a.head_dim = T, k.shape[0], H, k.shape[1], D
    a.causal = 1 if causal else 0
    a.scale = float(D ** -0.5 if scale is None else scale)
    _lib.check(_lib.load().solort_attn_prefill(ctypes.byref(a), ctypes.c_void_p(_stream(q.device))),
               "solort_attn_prefill")


def kv_store_into(key, value, slots, kv_pages) -> None:
    """Slot-mapped store of ``key / value [tokens, nkv, 128]`` into one layer's paged arena
    ``kv_pages [pages, 2, P, nkv, 128]``: the body of ``solort_attn::kv_store``."""
    for name, t in (("key", key), ("value", value)):
        _check_cuda(name, t, torch.bfloat16)
        if t.dim() != 3 or t.shape[-1] != HEAD_DIM or t.stride(-1) != 1:
            raise RuntimeError(f"{name} must be [tokens, nkv, 128] with a contiguous head dim")
    if key.shape != value.shape or key.stride() != value.stride():
        raise RuntimeError("key and value must have the same shape and strides")
    _check_cuda("slots", slots, torch.int64)
    if slots.dim() != 1 or slots.numel() != key.shape[0] or not slots.is_contiguous():
        raise RuntimeError(f"slots must be a contiguous int64 vector of {key.shape[0]} entries")
    _check_cuda("kv_pages", kv_pages, torch.bfloat16)
    if kv_pages.dim() != 5 or kv_pages.shape[1] != 2 or kv_pages.shape[-1] != HEAD_DIM or \
            kv_pages.stride(-1) != 1 or kv_pages.shape[3] != key.shape[1]:
        raise RuntimeError("kv_pages must be [num_pages, 2, page_size, nkv, 128] with the key's nkv")
    a = _lib.SolortKVStoreArgs()
    a.key, a.value = key.data_ptr(), value.data_ptr()
    a.src_stride_token, a.src_stride_head = key.stride(0), key.stride(1)
    a.num_tokens, a.num_kv_heads, a.head_dim = key.shape[0], key.shape[1], HEAD_DIM
    a.slots = slots.data_ptr()
    a.k_pages, a.v_pages = kv_pages[:, 0].data_ptr(), kv_pages[:, 1].data_ptr()
    a.dst_stride_page, a.dst_stride_token, a.dst_stride_head = (
        kv_pages.stride(0), kv_pages.stride(2), kv_pages.stride(3))
    a.page_size, a.num_pages = kv_pages.shape[2], kv_pages.shape[0]
    _lib.check(_lib.load().solort_attn_kv_store(ctypes.byref(a), ctypes.c_void_p(_stream(key.device))),
               "solort_attn_kv_store")


def _check_out_like(out, q) -> None:
    _check_cuda("out", out, torch.bfloat16)
    if out.shape != q.shape or out.stride(-1) != 1:
        raise RuntimeError("out must have the shape of q and a contiguous head dim")
