"""ctypes binding of ``libsolort_attn.so`` (the C ABI declared in ``include/solort_attn.h``).

The library is built in-tree by ``solort_b200.build``; it is loaded once, from the package
directory. There is no fallback: if the library is missing or fails to load, importing the ops
raises.
"""

from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsolort_attn.so")

SOLORT_OK = 0
STATUS_NAMES = {
    0: "SOLORT_OK",
    -1: "SOLORT_ERR_INVALID_ARGUMENT",
    -2: "SOLORT_ERR_UNSUPPORTED",
    -3: "SOLORT_ERR_WORKSPACE",
    -4: "SOLORT_ERR_CUDA",
    -5: "SOLORT_ERR_TENSOR_MAP",
    -6: "SOLORT_ERR_NO_DEVICE",
    -7: "SOLORT_ERR_SCRATCH_LIMIT",
    -8: "SOLORT_ERR_IPC",
}

# Every symbol the header declares; tests check the library exports each one.
EXPORTED_SYMBOLS = (
    "solort_attn_decode_workspace_size",
    "solort_attn_decode",
    "solort_attn_decode_static_scratch",
    "solort_attn_lse_merge",
    "solort_attn_prefill",
    "solort_attn_device_status",
    "solort_attn_status_string",
    "solort_attn_abi_version",
    "solort_attn_decode_exchange_workspace_size",
    "solort_attn_decode_exchange",
    "solort_attn_exchange_merge",
    "solort_attn_exchange_buffer_create",
    "solort_attn_exchange_buffer_open",
    "solort_attn_exchange_buffer_close",
    "solort_attn_exchange_buffer_destroy",
    "solort_attn_qk_norm_rope_append",
    "solort_attn_add_rmsnorm",
    "solort_attn_silu_mul",
    "solort_attn_gemv",
    "solort_attn_kv_store",
)

MAX_RANKS = 8  # SOLORT_MAX_RANKS
DECODE_STABLE_PREFIX = 1  # SOLORT_DECODE_STABLE_PREFIX
IPC_HANDLE_BYTES = 64

c_i32, c_i64, c_f32, c_vp, c_sz = ctypes.c_int32, ctypes.c_int64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t


class SolortDecodeArgs(ctypes.Structure):
    """Mirror of ``SolortDecodeArgs`` in ``include/solort_attn.h`` (same field order)."""

    _fields_ = [
        ("q", c_vp),
        ("q_stride_batch", c_i64), ("q_stride_token", c_i64), ("q_stride_head", c_i64),
        ("out", c_vp),
        ("out_stride_batch", c_i64), ("out_stride_token", c_i64), ("out_stride_head", c_i64),
        ("out_f32", c_vp),
        ("lse_out", c_vp),
        ("k", c_vp),
        ("v", c_vp),
        ("kv_stride_token", c_i64), ("kv_stride_head", c_i64), ("kv_stride_page", c_i64),
        ("kv_capacity", c_i32),
        ("block_table", c_vp),
        ("block_table_stride", c_i64),
        ("page_size", c_i32),
        ("num_pages", c_i32),
        ("q_pos", c_vp),
        ("q_lens", c_vp),
        ("kv_pos_offset", c_i64),
        ("batch", c_i32), ("q_len", c_i32), ("num_qo_heads", c_i32), ("num_kv_heads", c_i32),
        ("head_dim", c_i32),
        ("max_kv_len", c_i32),
        ("scale", c_f32),
        ("num_splits", c_i32),
        ("workspace", c_vp),
        ("workspace_bytes", c_sz),
        ("flags", ctypes.c_uint32),
    ]


class SolortMergeArgs(ctypes.Structure):
    """Mirror of ``SolortMergeArgs`` in ``include/solort_attn.h``."""

    _fields_ = [
        ("o_parts", c_vp),
        ("part_stride", c_i64),
        ("lse_parts", c_vp),
        ("lse_part_stride", c_i64),
        ("num_parts", c_i32),
        ("batch", c_i32), ("q_len", c_i32), ("num_qo_heads", c_i32), ("head_dim", c_i32),
        ("out", c_vp),
        ("out_stride_batch", c_i64), ("out_stride_token", c_i64), ("out_stride_head", c_i64),
        ("out_f32", c_vp),
        ("lse_out", c_vp),
    ]


class SolortExchangeArgs(ctypes.Structure):
    """Mirror of ``SolortExchangeArgs`` in ``include/solort_attn.h``."""

    _fields_ = [
        ("num_ranks", c_i32),
        ("rank", c_i32),
        ("slot_in_rank", c_vp * MAX_RANKS),
    ]


class SolortExchangeMergeArgs(ctypes.Structure):
    """Mirror of ``SolortExchangeMergeArgs`` in ``include/solort_attn.h``."""

    _fields_ = [
        ("slots", c_vp),
        ("slot_stride", c_i64),
        ("num_ranks", c_i32),
        ("batch", c_i32), ("q_len", c_i32), ("num_qo_heads", c_i32), ("head_dim", c_i32),
        ("out", c_vp),
        ("out_stride_batch", c_i64), ("out_stride_token", c_i64), ("out_stride_head", c_i64),
    ]


class SolortPrologueArgs(ctypes.Structure):
    """Mirror of ``SolortPrologueArgs`` in ``include/solort_attn.h``."""

    _fields_ = [
        ("qkv", c_vp),
        ("qkv_stride_token", c_i64),
        ("num_tokens", c_i32), ("num_qo_heads", c_i32), ("num_kv_heads", c_i32), ("head_dim", c_i32),
        ("q_norm_weight", c_vp),
        ("k_norm_weight", c_vp),
        ("eps", c_f32),
        ("cos", c_vp),
        ("sin", c_vp),
        ("rope_stride", c_i64),
        ("rope_rows", c_i32),
        ("pos", c_vp),
        ("q_out", c_vp),
        ("q_out_stride_token", c_i64), ("q_out_stride_head", c_i64),
        ("k_cache", c_vp),
        ("v_cache", c_vp),
        ("kv_stride_token", c_i64), ("kv_stride_head", c_i64), ("kv_stride_page", c_i64),
        ("kv_capacity", c_i32),
        ("block_table", c_vp),
        ("page_size", c_i32),
    ]


class SolortAddRmsNormArgs(ctypes.Structure):
    """Mirror of ``SolortAddRmsNormArgs`` in ``include/solort_attn.h``."""

    _fields_ = [
        ("x", c_vp), ("x_stride", c_i64),
        ("delta", c_vp), ("delta_stride", c_i64),
        ("weight", c_vp),
        ("x_out", c_vp), ("x_out_stride", c_i64),
        ("h_out", c_vp), ("h_out_stride", c_i64),
        ("rows", c_i32), ("hidden", c_i32),
        ("eps", c_f32),
    ]


class SolortSiluMulArgs(ctypes.Structure):
    """Mirror of ``SolortSiluMulArgs`` in ``include/solort_attn.h``."""

    _fields_ = [
        ("gate_up", c_vp), ("gate_up_stride", c_i64),
        ("out", c_vp), ("out_stride", c_i64),
        ("rows", c_i32), ("inter", c_i32),
    ]


class SolortGemvArgs(ctypes.Structure):
    """Mirror of ``SolortGemvArgs`` in ``include/solort_attn.h``."""

    _fields_ = [
        ("a", c_vp), ("a_stride", c_i64),
        ("w", c_vp), ("w_stride", c_i64),
        ("y", c_vp), ("y_stride", c_i64),
        ("t", c_i32), ("n", c_i32), ("k", c_i32), ("mode", c_i32),
        ("delta", c_vp), ("delta_stride", c_i64),
        ("norm_weight", c_vp),
        ("x_out", c_vp), ("x_out_stride", c_i64),
        ("eps", ctypes.c_float),
    ]


class SolortKVStoreArgs(ctypes.Structure):
    """Mirror of ``SolortKVStoreArgs`` in ``include/solort_attn.h``."""

    _fields_ = [
        ("key", c_vp),
        ("value", c_vp),
        ("src_stride_token", c_i64), ("src_stride_head", c_i64),
        ("num_tokens", c_i32), ("num_kv_heads", c_i32), ("head_dim", c_i32),
        ("slots", c_vp),
        ("k_pages", c_vp),
        ("v_pages", c_vp),
        ("dst_stride_page", c_i64), ("dst_stride_token", c_i64), ("dst_stride_head", c_i64),
        ("page_size", c_i32), ("num_pages", c_i32),
    ]


_LIB: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the in-tree library (once). Raises if it has not been built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(
            f"{LIB_PATH} is missing: build it with `python -m solort_b200.build` "
            "(or __graft_entry__.build()); there is no non-CUDA fallback"
        )
    lib = ctypes.CDLL(LIB_PATH)
    P = ctypes.POINTER
    lib.solort_attn_decode_workspace_size.argtypes = [P(SolortDecodeArgs), P(c_sz)]
    lib.solort_attn_decode_workspace_size.restype = ctypes.c_int
    lib.solort_attn_decode.argtypes = [P(SolortDecodeArgs), c_vp]
    lib.solort_attn_decode.restype = ctypes.c_int
    lib.solort_attn_decode_static_scratch.argtypes = [P(SolortDecodeArgs), c_vp]
    lib.solort_attn_decode_static_scratch.restype = ctypes.c_int
    lib.solort_attn_lse_merge.argtypes = [P(SolortMergeArgs), c_vp]
    lib.solort_attn_lse_merge.restype = ctypes.c_int
    lib.solort_attn_device_status.argtypes = [P(ctypes.c_uint)]
    lib.solort_attn_device_status.restype = ctypes.c_int
    lib.solort_attn_status_string.argtypes = [ctypes.c_int]
    lib.solort_attn_status_string.restype = ctypes.c_char_p
    lib.solort_attn_abi_version.argtypes = []
    lib.solort_attn_abi_version.restype = ctypes.c_int
    _optional_symbols(lib)
    _LIB = lib
    return lib


def _optional_symbols(lib: ctypes.CDLL) -> None:
    P = ctypes.POINTER
    lib.solort_attn_prefill.argtypes = [P(SolortPrefillArgs), c_vp]
    lib.solort_attn_prefill.restype = ctypes.c_int
    lib.solort_attn_decode_exchange_workspace_size.argtypes = [P(SolortDecodeArgs), P(c_sz)]
    lib.solort_attn_decode_exchange_workspace_size.restype = ctypes.c_int
    lib.solort_attn_decode_exchange.argtypes = [P(SolortDecodeArgs), P(SolortExchangeArgs), c_vp]
    lib.solort_attn_decode_exchange.restype = ctypes.c_int
    lib.solort_attn_exchange_merge.argtypes = [P(SolortExchangeMergeArgs), c_vp]
    lib.solort_attn_exchange_merge.restype = ctypes.c_int
    lib.solort_attn_exchange_buffer_create.argtypes = [c_sz, P(c_vp), c_vp]
    lib.solort_attn_exchange_buffer_create.restype = ctypes.c_int
    lib.solort_attn_exchange_buffer_open.argtypes = [c_vp, P(c_vp)]
    lib.solort_attn_exchange_buffer_open.restype = ctypes.c_int
    lib.solort_attn_exchange_buffer_close.argtypes = [c_vp]
    lib.solort_attn_exchange_buffer_close.restype = ctypes.c_int
    lib.solort_attn_exchange_buffer_destroy.argtypes = [c_vp]
    lib.solort_attn_exchange_buffer_destroy.restype = ctypes.c_int
    lib.solort_attn_qk_norm_rope_append.argtypes = [P(SolortPrologueArgs), c_vp]
    lib.solort_attn_qk_norm_rope_append.restype = ctypes.c_int
    lib.solort_attn_add_rmsnorm.argtypes = [P(SolortAddRmsNormArgs), c_vp]
    lib.solort_attn_add_rmsnorm.restype = ctypes.c_int
    lib.solort_attn_silu_mul.argtypes = [P(SolortSiluMulArgs), c_vp]
    lib.solort_attn_silu_mul.restype = ctypes.c_int
    lib.solort_attn_gemv.argtypes = [P(SolortGemvArgs), c_vp]
    lib.solort_attn_gemv.restype = ctypes.c_int
    lib.solort_attn_kv_store.argtypes = [P(SolortKVStoreArgs), c_vp]
    lib.solort_attn_kv_store.restype = ctypes.c_int


class SolortPrefillArgs(ctypes.Structure):
    """Mirror of ``SolortPrefillArgs`` in ``include/solort_attn.h``."""

    _fields_ = [
        ("q", c_vp),
        ("q_stride_token", c_i64), ("q_stride_head", c_i64),
        ("k", c_vp),
        ("v", c_vp),
        ("kv_stride_token", c_i64), ("kv_stride_head", c_i64),
        ("out", c_vp),
        ("out_stride_token", c_i64), ("out_stride_head", c_i64),
        ("q_len", c_i32), ("kv_len", c_i32),
        ("num_qo_heads", c_i32), ("num_kv_heads", c_i32), ("head_dim", c_i32),
        ("causal", c_i32),
        ("scale", c_f32),
    ]


def status_string(code: int) -> str:
    lib = load()
    return f"{STATUS_NAMES.get(code, code)}: {lib.solort_attn_status_string(code).decode()}"


def check(code: int, what: str) -> None:
    if code != SOLORT_OK:
        raise RuntimeError(f"{what} failed: {status_string(code)}")
