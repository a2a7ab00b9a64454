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

from solort_b200 import _calls, _lib
from solort_b200 import torch_ops  # noqa: F401  (registers torch.ops.solort_attn.*)
from solort_b200._calls import (  # noqa: F401  (re-exported for callers of the C-ABI helpers)
    HEAD_DIM, _check_cuda, _decode_args, _ptr, _run_decode, _static_kv, _stream, _stream_at,
    decode_workspace_bytes)

_OPS = torch.ops.solort_attn
_NO_WORKSPACE: dict[torch.device, torch.Tensor] = {}


def _empty_workspace(device: torch.device) -> torch.Tensor:
    """A zero-byte tensor standing for "no workspace" (calls whose split plan needs none)."""
    ws = _NO_WORKSPACE.get(device)
    if ws is None:
        ws = _NO_WORKSPACE[device] = torch.empty(0, dtype=torch.uint8, device=device)
    return ws


def _workspace_for(a: _lib.SolortDecodeArgs, device: torch.device,
                   workspace: torch.Tensor | None) -> torch.Tensor:
    if workspace is not None:
        return workspace
    need = _calls.decode_workspace_needed(a)
    if need == 0:
        return _empty_workspace(device)
    return torch.empty(need, dtype=torch.uint8, device=device)

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
    """GQA attention of ``q [B, q_len, nh, 128]`` against one layer's static KV buffer, through
    ``torch.ops.solort_attn.gqa_decode``.

    ``k_cache``/``v_cache`` are ``[max_len, nkv, 128]`` (``kv_layout="NHD"``, the reference's
    ``kc[li]``/``vc[li]`` of ``cuda_graph_executor.py:67-69``) or ``[nkv, max_len, 128]``
    (``"HND"``). ``q_pos`` (int64, ``[B]``, on the device) is the position of query row 0: row
    ``i`` sees keys ``0 .. q_pos + i`` -- decode (``:168,180-184``) with ``q_len == 1`` and verify
    (``:250,261-263``) with ``q_len == K + 1``. ``max_kv_len`` bounds the keys read (the decode
    bucket ``bound``); it defaults to the buffer length. ``stable_prefix``: ``q_pos`` and the keys
    below it were written before the kernel launched just before this call (earlier steps), so
    their loads may start during that kernel's tail (``SOLORT_DECODE_STABLE_PREFIX``). ``out`` and
    ``workspace`` are allocated when not given (pass both to capture the call in a CUDA graph).
    """
    cap, nkv, _, _ = _static_kv(k_cache, v_cache, kv_layout)
    _check_cuda("q", q, torch.bfloat16)
    if out is None:
        out = torch.empty_like(q)
    if workspace is None:
        need = decode_workspace_bytes(q.shape[0], q.shape[1], q.shape[2], nkv, max_kv_len or cap,
                                      kv_capacity=cap, num_splits=num_splits)
        workspace = (torch.empty(need, dtype=torch.uint8, device=q.device) if need
                     else _empty_workspace(q.device))
    _OPS.gqa_decode(q, k_cache, v_cache, q_pos, out, workspace, kv_layout, scale,
                    int(max_kv_len or 0), q_lens, int(num_splits), bool(stable_prefix))
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
    ``(O fp32 [B, q_len, nh, 128], LSE fp32 [B, q_len, nh])`` for ``lse_merge``
    (``torch.ops.solort_attn.gqa_decode_partial``). Local key ``t`` of the shard sits at absolute
    position ``kv_pos_offset + t``."""
    cap, nkv, _, _ = _static_kv(k_cache, v_cache, kv_layout)
    _check_cuda("q", q, torch.bfloat16)
    B, T, H, D = q.shape
    if out_f32 is None:
        out_f32 = torch.empty(B, T, H, D, dtype=torch.float32, device=q.device)
    if lse_out is None:
        lse_out = torch.empty(B, T, H, dtype=torch.float32, device=q.device)
    if workspace is None:
        need = decode_workspace_bytes(B, T, H, nkv, max_kv_len or cap, kv_capacity=cap,
                                      num_splits=num_splits)
        workspace = (torch.empty(need, dtype=torch.uint8, device=q.device) if need
                     else _empty_workspace(q.device))
    _OPS.gqa_decode_partial(q, k_cache, v_cache, q_pos, out_f32, lse_out, workspace,
                            int(kv_pos_offset), kv_layout, scale, int(max_kv_len or 0),
                            int(num_splits))
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
    """GQA attention against one layer of SoloRT's paged arena
    (``torch.ops.solort_attn.gqa_decode_paged``).

    ``kv_pages [num_pages, 2, P, nkv, 128]`` is one layer of ``PagedKVCache.kv_cache``
    (``kv_cache.py:86-100``); ``block_table [B, max_pages]`` int32 holds physical page ids as the
    page allocator and prefix cache hand them out (shared prefix pages may appear in several
    rows). Logical position ``p`` lives at page ``block_table[b, p // P]``, row ``p % P``
    (``kv_cache.py:136-149``). ``q_pos``/``q_lens`` as in ``gqa_decode``; ``max_kv_len`` bounds
    the keys any sequence may see; ``stable_prefix`` as in ``gqa_decode`` (it also covers the
    block table).
    """
    _check_cuda("q", q, torch.bfloat16)
    if out is None:
        out = torch.empty_like(q)
    if workspace is None:
        need = decode_workspace_bytes(q.shape[0], q.shape[1], q.shape[2], kv_pages.shape[3],
                                      max_kv_len, kv_capacity=0, page_size=kv_pages.shape[2],
                                      num_splits=num_splits)
        workspace = (torch.empty(need, dtype=torch.uint8, device=q.device) if need
                     else _empty_workspace(q.device))
    _OPS.gqa_decode_paged(q, kv_pages, block_table, q_pos, out, workspace, int(max_kv_len), scale,
                          q_lens, int(num_splits), bool(stable_prefix))
    return out

def lse_merge(
    o_parts: torch.Tensor,
    lse_parts: torch.Tensor,
    *,
    out: torch.Tensor | None = None,
    return_lse: bool = False,
):
    """Merge ``o_parts [R, B, q_len, nh, 128]`` fp32 with ``lse_parts [R, B, q_len, nh]``.

    Returns bf16 ``out [B, q_len, nh, 128]`` (``torch.ops.solort_attn.lse_merge``), or
    ``(O fp32, LSE fp32)`` with ``return_lse``.
    """
    _check_cuda("o_parts", o_parts, torch.float32)
    if o_parts.dim() != 5:
        raise RuntimeError("o_parts must be [parts, batch, q_len, num_qo_heads, 128]")
    R, B, T, H, D = o_parts.shape
    if return_lse:
        o32 = torch.empty(B, T, H, D, dtype=torch.float32, device=o_parts.device)
        lse = torch.empty(B, T, H, dtype=torch.float32, device=o_parts.device)
        _calls.lse_merge_into(o_parts, lse_parts, None, out_f32=o32, lse_out=lse)
        return o32, lse
    if out is None:
        out = torch.empty(B, T, H, D, dtype=torch.bfloat16, device=o_parts.device)
    _OPS.lse_merge(o_parts, lse_parts, out)
    return out

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
    """Causal GQA prefill of one sequence on the tcgen05 tensor cores
    (``torch.ops.solort_attn.gqa_prefill``).

    ``q [q_len, nh, 128]``, ``k, v [kv_len, nkv, 128]`` bf16 (token-major NHD views such as the
    reference's ``qkv.view(t, heads, hd)``; any token / head strides that are multiples of 8).
    With ``causal`` query ``i`` sees keys ``j <= kv_len - q_len + i``: the square prompt prefill
    of ``cuda_graph_executor.py:124-130`` and the HF bridge's bottom-right alignment
    (``transformers_flashinfer.py:182-193``). Returns ``out [q_len, nh, 128]`` bf16.
    """
    _check_cuda("q", q, torch.bfloat16)
    if out is None:
        out = torch.empty(q.shape, dtype=torch.bfloat16, device=q.device)
    _OPS.gqa_prefill(q, k, v, out, bool(causal), scale)
    return out


def kv_store(key: torch.Tensor, value: torch.Tensor, slots: torch.Tensor,
             kv_pages: torch.Tensor) -> None:
    """Write ``key / value [tokens, nkv, 128]`` (any token / head strides that are multiples of 8)
    to physical slots ``slots`` (int64 on the device, ``page * P + row``) of one layer's paged
    arena ``kv_pages [pages, 2, P, nkv, 128]`` (``torch.ops.solort_attn.kv_store``): the
    slot-mapped store of ``PagedKVCache.store_layer_tokens`` (``kv_cache.py:191-235``) in one
    launch instead of a Python loop over tokens."""
    _OPS.kv_store(key, value, slots, kv_pages)

