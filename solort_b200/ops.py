"""torch-facing entry points of the attention engine.

Thin wrappers that read pointers, strides and the current CUDA stream from torch tensors and
call the C ABI (``include/solort_attn.h``) through ``solort_b200._lib``. They launch on
``torch.cuda.current_stream()``, never synchronise, and allocate only when the caller did not
pass an output or workspace buffer, so a call with preallocated buffers can be captured in a
CUDA graph (the reference captures its decode and verify steps: ``cuda_graph_executor.py:195-207,
272-285``). Errors raise ``RuntimeError``; there is no fallback path.
"""

from __future__ import annotations

import ctypes
import math

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
    lib = _lib.load()
    need = ctypes.c_size_t(0)
    _lib.check(lib.solort_attn_decode_workspace_size(ctypes.byref(a), ctypes.byref(need)),
               "solort_attn_decode_workspace_size")
    if need.value > 0:
        if workspace is None:
            workspace = torch.empty(need.value, dtype=torch.uint8, device=device)
        a.workspace = workspace.data_ptr()
        a.workspace_bytes = workspace.numel() * workspace.element_size()
    _lib.check(lib.solort_attn_decode(ctypes.byref(a), ctypes.c_void_p(_stream(device))),
               "solort_attn_decode")


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


def gqa_decode(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    q_pos: torch.Tensor,
    *,
    kv_layout: str = "NHD",
    scale: float | None = None,
    max_kv_len: int | None = None,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    q_lens: torch.Tensor | None = None,
    num_splits: int = 0,
    stable_prefix: bool = False,
) -> torch.Tensor:
    """GQA attention of ``q [B, q_len, nh, 128]`` against one layer's static KV buffer.

    ``k_cache``/``v_cache`` are ``[max_len, nkv, 128]`` (``kv_layout="NHD"``, the reference's
    ``kc[li]``/``vc[li]`` of ``cuda_graph_executor.py:67-69``) or ``[nkv, max_len, 128]``
    (``"HND"``). ``q_pos`` (int64, ``[B]``, on the device) is the position of query row 0: row
    ``i`` sees keys ``0 .. q_pos + i`` -- decode (``:168,180-184``) with ``q_len == 1`` and verify
    (``:250,261-263``) with ``q_len == K + 1``. ``max_kv_len`` bounds the keys read (the decode
    bucket ``bound``); it defaults to the buffer length. ``stable_prefix``: ``q_pos`` and the keys
    below it were written before the kernel launched just before this call (earlier steps), so
    their loads may start during that kernel's tail (``SOLORT_DECODE_STABLE_PREFIX``).
    """
    cap, nkv, st, sh = _static_kv(k_cache, v_cache, kv_layout)
    if q_pos.numel() != q.shape[0]:
        raise RuntimeError(f"q_pos has {q_pos.numel()} entries for batch {q.shape[0]}")
    if out is None:
        out = torch.empty_like(q)
    a = _decode_args(
        q, k_cache, v_cache, q_pos, stride_token=st, stride_head=sh, stride_page=0,
        kv_capacity=cap, num_kv_heads=nkv, block_table=None, page_size=0, num_pages=0,
        scale=scale, max_kv_len=max_kv_len or cap, out=out, out_f32=None, lse_out=None,
        q_lens=q_lens, kv_pos_offset=0, num_splits=num_splits, stable_prefix=stable_prefix)
    _run_decode(a, q.device, workspace)
    return out


class DecodeCall:
    """A prepared ``gqa_decode`` on fixed buffers: arguments are checked and packed once, and
    each call is one C-ABI launch on the current stream (the shape of the reference's static
    buffers, which never move between decode steps; ``cuda_graph_executor.py:67-71``)."""

    def __init__(self, q, k_cache, v_cache, q_pos, *, kv_layout="NHD", scale=None,
                 max_kv_len=None, out, workspace=None, num_splits=0, stable_prefix=False):
        cap, nkv, st, sh = _static_kv(k_cache, v_cache, kv_layout)
        self._keep = (q, k_cache, v_cache, q_pos, out)
        self.args = _decode_args(
            q, k_cache, v_cache, q_pos, stride_token=st, stride_head=sh, stride_page=0,
            kv_capacity=cap, num_kv_heads=nkv, block_table=None, page_size=0, num_pages=0,
            scale=scale, max_kv_len=max_kv_len or cap, out=out, out_f32=None, lse_out=None,
            q_lens=None, kv_pos_offset=0, num_splits=num_splits, stable_prefix=stable_prefix)
        lib = _lib.load()
        need = ctypes.c_size_t(0)
        _lib.check(lib.solort_attn_decode_workspace_size(ctypes.byref(self.args), ctypes.byref(need)),
                   "solort_attn_decode_workspace_size")
        if need.value > 0:
            if workspace is None or workspace.numel() * workspace.element_size() < need.value:
                raise RuntimeError(f"DecodeCall needs a workspace of {need.value} bytes")
            self.args.workspace = workspace.data_ptr()
            self.args.workspace_bytes = workspace.numel() * workspace.element_size()
            self._keep = self._keep + (workspace,)
        self._fn = lib.solort_attn_decode
        self._ref = ctypes.byref(self.args)
        self._device = q.device
        self._index = q.device.index

    def __call__(self) -> None:
        rc = self._fn(self._ref, ctypes.c_void_p(_stream_at(self._index)))
        if rc != 0:
            _lib.check(rc, "solort_attn_decode")


class ShardedDecodeCall:
    """A prepared sharded-decode layer on fixed buffers: ``gqa_decode_exchange`` over this rank's
    shard followed by ``exchange_merge``, both packed once, each call two C-ABI launches on the
    current stream."""

    def __init__(self, q, k_shard, v_shard, q_pos, exchange, recv_slots: int, slot_stride: int,
                 num_ranks: int, *, kv_pos_offset=0, kv_layout="NHD", scale=None, out,
                 workspace, stable_prefix=False):
        cap, nkv, st, sh = _static_kv(k_shard, v_shard, kv_layout)
        _check_cuda("out", out, torch.bfloat16)
        self._keep = (q, k_shard, v_shard, q_pos, out, workspace, exchange)
        self.args = _decode_args(
            q, k_shard, v_shard, q_pos, stride_token=st, stride_head=sh, stride_page=0,
            kv_capacity=cap, num_kv_heads=nkv, block_table=None, page_size=0, num_pages=0,
            scale=scale, max_kv_len=cap, out=None, out_f32=None, lse_out=None, q_lens=None,
            kv_pos_offset=kv_pos_offset, num_splits=0, stable_prefix=stable_prefix)
        lib = _lib.load()
        need = ctypes.c_size_t(0)
        _lib.check(lib.solort_attn_decode_exchange_workspace_size(ctypes.byref(self.args),
                                                                  ctypes.byref(need)),
                   "solort_attn_decode_exchange_workspace_size")
        if workspace.numel() * workspace.element_size() < need.value:
            raise RuntimeError(f"ShardedDecodeCall needs a workspace of {need.value} bytes")
        self.args.workspace = workspace.data_ptr()
        self.args.workspace_bytes = workspace.numel() * workspace.element_size()
        B, T, H, D = out.shape
        self.margs = _lib.SolortExchangeMergeArgs()
        self.margs.slots, self.margs.slot_stride, self.margs.num_ranks = recv_slots, slot_stride, num_ranks
        self.margs.batch, self.margs.q_len, self.margs.num_qo_heads, self.margs.head_dim = B, T, H, D
        self.margs.out = out.data_ptr()
        self.margs.out_stride_batch, self.margs.out_stride_token, self.margs.out_stride_head = (
            out.stride(0), out.stride(1), out.stride(2))
        self._send, self._merge = lib.solort_attn_decode_exchange, lib.solort_attn_exchange_merge
        self._a, self._x, self._m = ctypes.byref(self.args), ctypes.byref(exchange), ctypes.byref(self.margs)
        self._device = q.device
        self._index = q.device.index

    def __call__(self) -> None:
        st = ctypes.c_void_p(_stream_at(self._index))
        rc = self._send(self._a, self._x, st)
        if rc != 0:
            _lib.check(rc, "solort_attn_decode_exchange")
        rc = self._merge(self._m, st)
        if rc != 0:
            _lib.check(rc, "solort_attn_exchange_merge")


def gqa_decode_partial(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    q_pos: torch.Tensor,
    *,
    kv_pos_offset: int = 0,
    kv_layout: str = "NHD",
    scale: float | None = None,
    max_kv_len: int | None = None,
    out_f32: torch.Tensor | None = None,
    lse_out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    num_splits: int = 0,
):
    """Like ``gqa_decode`` over one shard of the keys, returning the partial
    ``(O fp32 [B, q_len, nh, 128], LSE fp32 [B, q_len, nh])`` for ``lse_merge``. Local key ``t``
    of the shard sits at absolute position ``kv_pos_offset + t``."""
    cap, nkv, st, sh = _static_kv(k_cache, v_cache, kv_layout)
    B, T, H, D = q.shape
    if out_f32 is None:
        out_f32 = torch.empty(B, T, H, D, dtype=torch.float32, device=q.device)
    if lse_out is None:
        lse_out = torch.empty(B, T, H, dtype=torch.float32, device=q.device)
    a = _decode_args(
        q, k_cache, v_cache, q_pos, stride_token=st, stride_head=sh, stride_page=0,
        kv_capacity=cap, num_kv_heads=nkv, block_table=None, page_size=0, num_pages=0,
        scale=scale, max_kv_len=max_kv_len or cap, out=None, out_f32=out_f32, lse_out=lse_out,
        q_lens=None, kv_pos_offset=kv_pos_offset, num_splits=num_splits)
    _run_decode(a, q.device, workspace)
    return out_f32, lse_out


def gqa_decode_paged(
    q: torch.Tensor,
    kv_pages: torch.Tensor,
    block_table: torch.Tensor,
    q_pos: torch.Tensor,
    *,
    max_kv_len: int,
    scale: float | None = None,
    out: torch.Tensor | None = None,
    workspace: torch.Tensor | None = None,
    q_lens: torch.Tensor | None = None,
    num_splits: int = 0,
    stable_prefix: bool = False,
) -> torch.Tensor:
    """GQA attention against one layer of SoloRT's paged arena.

    ``kv_pages [num_pages, 2, P, nkv, 128]`` is one layer of ``PagedKVCache.kv_cache``
    (``kv_cache.py:86-100``); ``block_table [B, max_pages]`` int32 holds physical page ids as the
    page allocator and prefix cache hand them out (shared prefix pages may appear in several
    rows). Logical position ``p`` lives at page ``block_table[b, p // P]``, row ``p % P``
    (``kv_cache.py:136-149``). ``q_pos``/``q_lens`` as in ``gqa_decode``; ``max_kv_len`` bounds
    the keys any sequence may see; ``stable_prefix`` as in ``gqa_decode`` (it also covers the
    block table).
    """
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
    if out is None:
        out = torch.empty_like(q)
    k = kv_pages[:, 0]
    v = kv_pages[:, 1]
    a = _decode_args(
        q, k, v, q_pos, stride_token=kv_pages.stride(2), stride_head=kv_pages.stride(3),
        stride_page=kv_pages.stride(0), kv_capacity=0, num_kv_heads=nkv,
        block_table=block_table, page_size=P, num_pages=num_pages, scale=scale,
        max_kv_len=max_kv_len, out=out, out_f32=None, lse_out=None, q_lens=q_lens,
        kv_pos_offset=0, num_splits=num_splits, stable_prefix=stable_prefix)
    _run_decode(a, q.device, workspace)
    return out


def lse_merge(
    o_parts: torch.Tensor,
    lse_parts: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
    return_lse: bool = False,
):
    """Merge ``o_parts [R, B, q_len, nh, 128]`` fp32 with ``lse_parts [R, B, q_len, nh]``.

    Returns bf16 ``out [B, q_len, nh, 128]``, or ``(O fp32, LSE fp32)`` with ``return_lse``.
    """
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
    lse = None
    if return_lse:
        o32 = torch.empty(B, T, H, D, dtype=torch.float32, device=o_parts.device)
        lse = torch.empty(B, T, H, dtype=torch.float32, device=o_parts.device)
        m.out_f32, m.lse_out = o32.data_ptr(), lse.data_ptr()
        res = (o32, lse)
    else:
        if out is None:
            out = torch.empty(B, T, H, D, dtype=torch.bfloat16, device=o_parts.device)
        m.out = out.data_ptr()
        m.out_stride_batch, m.out_stride_token, m.out_stride_head = out.stride(0), out.stride(1), out.stride(2)
        res = out
    _lib.check(_lib.load().solort_attn_lse_merge(ctypes.byref(m), ctypes.c_void_p(_stream(o_parts.device))),
               "solort_attn_lse_merge")
    return res


def decode_exchange_workspace_bytes(
    batch: int, q_len: int, num_qo_heads: int, num_kv_heads: int, max_kv_len: int,
    *, kv_capacity: int | None = None, num_splits: int = 0,
) -> int:
    """Workspace bytes a ``gqa_decode_exchange`` call with these sizes needs on the current device."""
    a = _lib.SolortDecodeArgs()
    a.batch, a.q_len, a.num_qo_heads, a.num_kv_heads, a.head_dim = (
        batch, q_len, num_qo_heads, num_kv_heads, HEAD_DIM)
    a.max_kv_len = max_kv_len
    a.kv_capacity = kv_capacity if kv_capacity is not None else max_kv_len
    a.num_splits = num_splits
    need = ctypes.c_size_t(0)
    _lib.check(_lib.load().solort_attn_decode_exchange_workspace_size(ctypes.byref(a), ctypes.byref(need)),
               "solort_attn_decode_exchange_workspace_size")
    return int(need.value)


def gqa_decode_exchange(
    q: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    q_pos: torch.Tensor,
    exchange: _lib.SolortExchangeArgs,
    *,
    kv_pos_offset: int = 0,
    kv_layout: str = "NHD",
    scale: float | None = None,
    max_kv_len: int | None = None,
    workspace: torch.Tensor | None = None,
    num_splits: int = 0,
    stable_prefix: bool = False,
) -> None:
    """Decode over this rank's key shard and store the rank's partial ``(O, LSE)`` into its slot
    on every rank named by ``exchange`` (peer-memory stores of self-marking 64-bit words)."""
    cap, nkv, st, sh = _static_kv(k_cache, v_cache, kv_layout)
    a = _decode_args(
        q, k_cache, v_cache, q_pos, stride_token=st, stride_head=sh, stride_page=0,
        kv_capacity=cap, num_kv_heads=nkv, block_table=None, page_size=0, num_pages=0,
        scale=scale, max_kv_len=max_kv_len or cap, out=None, out_f32=None, lse_out=None,
        q_lens=None, kv_pos_offset=kv_pos_offset, num_splits=num_splits,
        stable_prefix=stable_prefix)
    lib = _lib.load()
    need = ctypes.c_size_t(0)
    _lib.check(lib.solort_attn_decode_exchange_workspace_size(ctypes.byref(a), ctypes.byref(need)),
               "solort_attn_decode_exchange_workspace_size")
    if workspace is None:
        workspace = torch.empty(need.value, dtype=torch.uint8, device=q.device)
    a.workspace = workspace.data_ptr()
    a.workspace_bytes = workspace.numel() * workspace.element_size()
    _lib.check(lib.solort_attn_decode_exchange(ctypes.byref(a), ctypes.byref(exchange),
                                               ctypes.c_void_p(_stream(q.device))),
               "solort_attn_decode_exchange")


def exchange_merge(slots: int, slot_stride: int, num_ranks: int, out: torch.Tensor) -> torch.Tensor:
    """Wait for every rank's partial in this rank's receive slots (device address; rank ``s``'s
    slot at ``slots + s * slot_stride`` 64-bit words), merge them into bf16 ``out [B, q_len, nh,
    128]`` and zero the slots for their next use."""
    _check_cuda("out", out, torch.bfloat16)
    B, T, H, D = out.shape
    m = _lib.SolortExchangeMergeArgs()
    m.slots, m.slot_stride, m.num_ranks = slots, slot_stride, num_ranks
    m.batch, m.q_len, m.num_qo_heads, m.head_dim = B, T, H, D
    m.out = out.data_ptr()
    m.out_stride_batch, m.out_stride_token, m.out_stride_head = out.stride(0), out.stride(1), out.stride(2)
    _lib.check(_lib.load().solort_attn_exchange_merge(ctypes.byref(m), ctypes.c_void_p(_stream(out.device))),
               "solort_attn_exchange_merge")
    return out


def qk_norm_rope_append(
    qkv: torch.Tensor,
    q_norm_weight: torch.Tensor,
    k_norm_weight: torch.Tensor,
    eps: float,
    cos: torch.Tensor,
    sin: torch.Tensor,
    pos: torch.Tensor,
    k_cache: torch.Tensor,
    v_cache: torch.Tensor,
    *,
    num_qo_heads: int,
    num_kv_heads: int,
    q_out: torch.Tensor | None = None,
    block_table: torch.Tensor | None = None,
) -> torch.Tensor:
    """One layer's attention prologue: QK-RMSNorm + RoPE of ``qkv [t, (nh + 2 nkv) * 128]``,
    queries to ``q_out [t, nh, 128]``, K / V appended at positions ``pos[0] .. pos[0] + t - 1``.

    ``k_cache``/``v_cache``: one layer's static NHD buffers ``[max_len, nkv, 128]`` (the reference's
    ``kc[li]``/``vc[li]``), or with ``block_table`` (int32, the sequence's physical pages) the K / V
    halves of a paged arena, ``arena[:, 0]`` / ``arena[:, 1]`` of ``[pages, 2, P, nkv, 128]``.
    ``cos``/``sin``: the model's bf16 tables ``[rows, 128]`` indexed by position."""
    _check_cuda("qkv", qkv, torch.bfloat16)
    t = qkv.shape[0]
    if qkv.dim() != 2 or qkv.shape[1] != (num_qo_heads + 2 * num_kv_heads) * HEAD_DIM or qkv.stride(1) != 1:
        raise RuntimeError("qkv must be [t, (num_qo_heads + 2 * num_kv_heads) * 128], rows contiguous")
    for name, tsr in (("cos", cos), ("sin", sin)):
        _check_cuda(name, tsr, torch.bfloat16)
        if tsr.dim() != 2 or tsr.shape[1] != HEAD_DIM or tsr.stride(1) != 1:
            raise RuntimeError(f"{name} must be [rows, 128] with contiguous rows")
    _check_cuda("pos", pos, torch.int64)
    if q_out is None:
        q_out = torch.empty(t, num_qo_heads, HEAD_DIM, dtype=torch.bfloat16, device=qkv.device)
    a = _lib.SolortPrologueArgs()
    a.qkv, a.qkv_stride_token = qkv.data_ptr(), qkv.stride(0)
    a.num_tokens, a.num_qo_heads, a.num_kv_heads, a.head_dim = t, num_qo_heads, num_kv_heads, HEAD_DIM
    a.q_norm_weight, a.k_norm_weight, a.eps = q_norm_weight.data_ptr(), k_norm_weight.data_ptr(), float(eps)
    a.cos, a.sin, a.rope_stride, a.rope_rows = cos.data_ptr(), sin.data_ptr(), cos.stride(0), cos.shape[0]
    a.pos = pos.data_ptr()
    a.q_out, a.q_out_stride_token, a.q_out_stride_head = q_out.data_ptr(), q_out.stride(0), q_out.stride(1)
    a.k_cache, a.v_cache = k_cache.data_ptr(), v_cache.data_ptr()
    if block_table is None:
        if k_cache.dim() != 3 or k_cache.stride() != v_cache.stride():
            raise RuntimeError("static k_cache / v_cache must be [max_len, nkv, 128] with equal strides")
        a.kv_stride_token, a.kv_stride_head, a.kv_stride_page = k_cache.stride(0), k_cache.stride(1), 0
        a.kv_capacity = k_cache.shape[0]
    else:
        _check_cuda("block_table", block_table, torch.int32)
        if k_cache.dim() != 4 or k_cache.stride() != v_cache.stride():
            raise RuntimeError("paged k_cache / v_cache must be [pages, P, nkv, 128] views with equal strides")
        P = k_cache.shape[1]
        a.kv_stride_page, a.kv_stride_token, a.kv_stride_head = k_cache.stride(0), k_cache.stride(1), k_cache.stride(2)
        a.kv_capacity = block_table.numel() * P  # positions the table covers
        a.block_table, a.page_size = block_table.data_ptr(), P
    _lib.check(_lib.load().solort_attn_qk_norm_rope_append(ctypes.byref(a), ctypes.c_void_p(_stream(qkv.device))),
               "solort_attn_qk_norm_rope_append")
    return q_out


def add_rmsnorm(
    x: torch.Tensor,
    delta: torch.Tensor | None,
    weight: torch.Tensor,
    eps: float,
    *,
    x_out: torch.Tensor | None = None,
    h_out: torch.Tensor | None = None,
) -> tuple[torch.Tensor, torch.Tensor]:
    """``x_out = x + delta`` (when ``delta`` is given; ``x_out`` may be ``x``) and
    ``h_out = rmsnorm(x_out) * weight`` for ``[rows, hidden]`` bf16 rows, the reference's residual
    add and ``_rmsnorm`` in one launch. Returns ``(x_out, h_out)`` (``x_out`` is ``x`` without a
    delta)."""
    _check_cuda("x", x, torch.bfloat16)
    if x.dim() != 2 or x.stride(1) != 1:
        raise RuntimeError("x must be [rows, hidden] with contiguous rows")
    rows, hidden = x.shape
    if h_out is None:
        h_out = torch.empty_like(x)
    a = _lib.SolortAddRmsNormArgs()
    a.x, a.x_stride = x.data_ptr(), x.stride(0)
    if delta is not None:
        _check_cuda("delta", delta, torch.bfloat16)
        if x_out is None:
            x_out = torch.empty_like(x)
        a.delta, a.delta_stride = delta.data_ptr(), delta.stride(0)
        a.x_out, a.x_out_stride = x_out.data_ptr(), x_out.stride(0)
    else:
        x_out = x
    a.weight = weight.data_ptr()
    a.h_out, a.h_out_stride = h_out.data_ptr(), h_out.stride(0)
    a.rows, a.hidden, a.eps = rows, hidden, float(eps)
    _lib.check(_lib.load().solort_attn_add_rmsnorm(ctypes.byref(a), ctypes.c_void_p(_stream(x.device))),
               "solort_attn_add_rmsnorm")
    return x_out, h_out


def silu_mul(gate_up: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``silu(gate) * up`` of a fused ``[rows, 2 * inter]`` gate/up projection (bf16)."""
    _check_cuda("gate_up", gate_up, torch.bfloat16)
    if gate_up.dim() != 2 or gate_up.stride(1) != 1 or gate_up.shape[1] % 2:
        raise RuntimeError("gate_up must be [rows, 2 * inter] with contiguous rows")
    rows, inter = gate_up.shape[0], gate_up.shape[1] // 2
    if out is None:
        out = torch.empty(rows, inter, dtype=torch.bfloat16, device=gate_up.device)
    a = _lib.SolortSiluMulArgs()
    a.gate_up, a.gate_up_stride = gate_up.data_ptr(), gate_up.stride(0)
    a.out, a.out_stride = out.data_ptr(), out.stride(0)
    a.rows, a.inter = rows, inter
    _lib.check(_lib.load().solort_attn_silu_mul(ctypes.byref(a), ctypes.c_void_p(_stream(gate_up.device))),
               "solort_attn_silu_mul")
    return out


def gemv(a: torch.Tensor, weight: torch.Tensor, *, silu_gate_up: bool = False,
         out: torch.Tensor | None = None, norm_weight: torch.Tensor | None = None,
         delta: torch.Tensor | None = None, x_out: torch.Tensor | None = None,
         eps: float = 1e-6) -> torch.Tensor:
    """``act @ weight[n, k].T`` for ``t <= 8`` token rows as a weight stream (bf16 out, fp32
    accumulation). ``act`` is ``a [t, k]``; with ``silu_gate_up``, ``silu(gate) * up`` of a fused
    ``[t, 2k]`` gate/up projection ``a``; with ``norm_weight``, ``RMSNorm(x) * norm_weight`` of the
    residual stream ``x = a`` or, given ``delta``, of ``x = a + delta``, which is then also written
    to ``x_out`` (a separate buffer; the residual add and norm of the layer loop, bit-identical to
    :func:`add_rmsnorm`)."""
    _check_cuda("a", a, torch.bfloat16)
    _check_cuda("weight", weight, torch.bfloat16)
    if a.dim() != 2 or a.stride(1) != 1 or weight.dim() != 2 or weight.stride(1) != 1:
        raise RuntimeError("a and weight must be 2-D with contiguous rows")
    t = a.shape[0]
    n, k = weight.shape
    if silu_gate_up and norm_weight is not None:
        raise RuntimeError("silu_gate_up and norm_weight are exclusive")
    if a.shape[1] != (2 * k if silu_gate_up else k):
        raise RuntimeError(f"a has {a.shape[1]} columns for a weight with k={k}")
    if out is None:
        out = torch.empty(t, n, dtype=torch.bfloat16, device=a.device)
    g = _lib.SolortGemvArgs()
    g.a, g.a_stride = a.data_ptr(), a.stride(0)
    g.w, g.w_stride = weight.data_ptr(), weight.stride(0)
    g.y, g.y_stride = out.data_ptr(), out.stride(0)
    g.t, g.n, g.k, g.mode = t, n, k, 1 if silu_gate_up else 0
    if norm_weight is not None:
        _check_cuda("norm_weight", norm_weight, torch.bfloat16)
        if norm_weight.shape != (k,) or not norm_weight.is_contiguous():
            raise RuntimeError(f"norm_weight must be a contiguous [{k}] vector")
        g.mode, g.norm_weight, g.eps = 2, norm_weight.data_ptr(), float(eps)
        if delta is not None:
            _check_cuda("delta", delta, torch.bfloat16)
            if x_out is None:
                raise RuntimeError("delta needs x_out (the updated residual stream)")
            _check_cuda("x_out", x_out, torch.bfloat16)
            for name, ten in (("delta", delta), ("x_out", x_out)):
                if ten.shape != a.shape or ten.stride(1) != 1:
                    raise RuntimeError(f"{name} must be [{t}, {k}] with contiguous rows")
            g.delta, g.delta_stride = delta.data_ptr(), delta.stride(0)
            g.x_out, g.x_out_stride = x_out.data_ptr(), x_out.stride(0)
    _lib.check(_lib.load().solort_attn_gemv(ctypes.byref(g), ctypes.c_void_p(_stream(a.device))),
               "solort_attn_gemv")
    return out


def device_status() -> int:
    """Read and clear the library's device status word (nonzero: an in-kernel wait timed out)."""
    flags = ctypes.c_uint(0)
    _lib.check(_lib.load().solort_attn_device_status(ctypes.byref(flags)), "solort_attn_device_status")
    return int(flags.value)


def default_scale(head_dim: int = HEAD_DIM) -> float:
    return 1.0 / math.sqrt(head_dim)


def gqa_prefill(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    *,
    causal: bool = True,
    scale: float | None = None,
    out: torch.Tensor | None = None,
) -> torch.Tensor:
    """Causal GQA prefill of one sequence on the tcgen05 tensor cores.

    ``q [q_len, nh, 128]``, ``k, v [kv_len, nkv, 128]`` bf16 (token-major NHD views such as the
    reference's ``qkv.view(t, heads, hd)``; any token / head strides that are multiples of 8).
    With ``causal`` query ``i`` sees keys ``j <= kv_len - q_len + i``: the square prompt prefill
    of ``cuda_graph_executor.py:124-130`` and the HF bridge's bottom-right alignment
    (``transformers_flashinfer.py:182-193``). Returns ``out [q_len, nh, 128]`` bf16.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_cuda(name, t, torch.bfloat16)
        if t.dim() != 3 or t.shape[-1] != HEAD_DIM or t.stride(-1) != 1:
            raise RuntimeError(f"{name} must be [tokens, heads, 128] with a contiguous head dim")
    if k.shape != v.shape or k.stride() != v.stride():
        raise RuntimeError("k and v must have the same shape and strides")
    T, H, D = q.shape
    if out is None:
        out = torch.empty(T, H, D, dtype=torch.bfloat16, device=q.device)
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
    return out
