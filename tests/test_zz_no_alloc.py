"""The allocation-free decode entry point, for callers that cannot allocate device memory.

Some callers have no way to pass a workspace: a plugin host whose operator interface hands over
only input and output buffers, or a host runtime that binds the C ABI without a CUDA allocator.
`solort_attn_decode_static_scratch` serves them from a static 4 MiB device array inside the
library. These tests call it through the C ABI several times in a row and compare each output with
the regular `solort_attn_decode` (given a workspace) and with the oracle, within the parity
tolerance used everywhere else (max-abs 2e-2, mean-abs 2e-3): a full 8192-key decode; the same
buffer, split count and row layout with the query at position 700, so 33 of the 37 splits hold no
visible key and must overwrite the previous call's partials at the same offsets with empty ones;
and a 5-token verify at 3000 keys, a different layout over the same array. The file is collected
last so a stop-at-first-failure run has run every other test before it; it passes alone in a fresh
process too.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from oracle import attention as A
from solort_b200 import _lib, ops

pytestmark = pytest.mark.gpu

SCRATCH_LIMIT = 4 << 20
MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _args(q, k, v, qpos, out, num_splits=0):
    return ops._decode_args(
        q, k, v, qpos, stride_token=k.stride(0), stride_head=k.stride(1), stride_page=0,
        kv_capacity=k.shape[0], num_kv_heads=k.shape[1], block_table=None, page_size=0,
        num_pages=0, scale=None, max_kv_len=k.shape[0], out=out, out_f32=None, lse_out=None,
        q_lens=None, kv_pos_offset=0, num_splits=num_splits)


def _close(got, ref, what):
    d = (got.float() - ref.float()).abs()
    assert torch.isfinite(got.float()).all(), what
    assert d.max().item() <= MAX_ABS, f"{what}: max-abs {d.max().item():.3g}"
    assert d.mean().item() <= MEAN_ABS, f"{what}: mean-abs {d.mean().item():.3g}"


def test_static_scratch_matches_workspace_entry_point_on_calls_in_a_row():
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # An explicit split count keeps the split partials in scratch memory: with one split a call
    # needs no workspace at all. Calls: (seed, keys in the buffer, query rows, splits, q_pos).
    for seed, L, q_len, splits, pos in ((1, 8192, 1, 37, 8191), (3, 8192, 1, 37, 700),
                                        (2, 3000, 5, 12, 2995)):
        q, k, v = A.make_attention_inputs(seed, 32, 8, 128, q_len, L, pos)
        dq, dk, dv = q[None].cuda(), k.cuda(), v.cuda()
        qpos = torch.tensor([pos], dtype=torch.int64, device="cuda")

        out_ref = torch.empty_like(dq)
        a = _args(dq, dk, dv, qpos, out_ref, splits)
        need = ctypes.c_size_t(0)
        assert lib.solort_attn_decode_workspace_size(ctypes.byref(a), ctypes.byref(need)) == 0
        assert 0 < need.value <= SCRATCH_LIMIT
        ws = torch.empty(need.value, dtype=torch.uint8, device="cuda")
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        assert lib.solort_attn_decode(ctypes.byref(a), stream) == 0

        out_new = torch.full_like(dq, float("nan"))
        b = _args(dq, dk, dv, qpos, out_new, splits)
        b.workspace, b.workspace_bytes = None, 0  # no workspace: the static array is used
        assert lib.solort_attn_decode_static_scratch(ctypes.byref(b), stream) == 0
        torch.cuda.synchronize()

        _close(out_new, out_ref, f"static scratch vs workspace, L={L} q_len={q_len} pos={pos}")
        ref, _ = A.attention_fp32(q, k, v, 128 ** -0.5, pos)
        _close(out_new[0].cpu(), ref, f"static scratch vs oracle, L={L} q_len={q_len} pos={pos}")
    assert ops.device_status() == 0


def test_static_scratch_rejects_calls_beyond_its_limit():
    lib = _lib.load()
    # 16 sequences x 8 query tokens x 32 heads need more than 4 MiB of split partials
    q = torch.zeros(16, 8, 32, 128, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(8192, 8, 128, dtype=torch.bfloat16, device="cuda")
    qpos = torch.zeros(16, dtype=torch.int64, device="cuda")
    out = torch.empty_like(q)
    a = _args(q, k, k, qpos, out, 2)
    need = ctypes.c_size_t(0)
    assert lib.solort_attn_decode_workspace_size(ctypes.byref(a), ctypes.byref(need)) == 0
    assert need.value > SCRATCH_LIMIT
    rc = lib.solort_attn_decode_static_scratch(ctypes.byref(a), ctypes.c_void_p(0))
    assert rc == -7, _lib.status_string(rc)
    assert b"4 MiB" in lib.solort_attn_status_string(rc)
