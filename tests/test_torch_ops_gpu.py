"""``torch.ops.solort_attn.*`` on the GPU: each op against the fp32 oracle, captured inside a CUDA
graph and replayed with a moving position (the reference captures its decode and verify steps,
``cuda_graph_executor.py:195-207,272-285``), and the slot-mapped ``kv_store`` bit-exact against the
reference's ``store_layer_tokens`` semantics (``kv_cache.py:191-235``).

Tolerance: max-abs <= 2e-2, mean-abs <= 2e-3 on the attention output.
"""

from __future__ import annotations

import pytest
import torch

from oracle import attention as A
from oracle import paged as OP

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3
SCALE = 128 ** -0.5


def _close(got, ref, what):
    d = (got.float().cpu() - ref.float().cpu()).abs()
    assert torch.isfinite(got.float()).all(), what
    assert d.max().item() <= MAX_ABS, f"{what}: max-abs {d.max().item():.4g}"
    assert d.mean().item() <= MEAN_ABS, f"{what}: mean-abs {d.mean().item():.4g}"


def _ops():
    from solort_b200 import ops

    return ops


def test_gqa_decode_op_captured_in_a_graph_replays_at_moving_positions():
    ops = _ops()
    cap, q_len = 4096, 1
    q_all, k, v = A.make_attention_inputs(7, 32, 8, 128, 1, cap, cap - 1)
    dk, dv = k.cuda(), v.cuda()
    q = torch.zeros(1, q_len, 32, 128, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros_like(q)
    pos = torch.zeros(1, dtype=torch.int64, device="cuda")
    ws = torch.empty(ops.decode_workspace_bytes(1, q_len, 32, 8, cap), dtype=torch.uint8,
                     device="cuda")
    q.copy_(q_all[None].cuda())
    pos.fill_(100)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):  # warm-up outside the capture, as the reference does
        torch.ops.solort_attn.gqa_decode(q, dk, dv, pos, out, ws, "NHD", SCALE, cap)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        torch.ops.solort_attn.gqa_decode(q, dk, dv, pos, out, ws, "NHD", SCALE, cap)
    for p in (5, 1000, 2047, 4095):
        pos.fill_(p)
        g.replay()
        torch.cuda.synchronize()
        ref, _ = A.attention_fp32(q_all, k, v, SCALE, p)
        _close(out[0], ref, f"graph replay at pos {p}")
    assert ops.device_status() == 0


def test_gqa_decode_paged_op_captured_verify():
    ops = _ops()
    P, n, K = 16, 900, 4
    q, k, v = A.make_attention_inputs(8, 32, 8, 128, K, n, n - K)
    g = torch.Generator().manual_seed(3)
    table = torch.randperm(128, generator=g)[: OP.pages_required(n, P)].tolist()
    arena = torch.zeros(128, 2, P, 8, 128, dtype=torch.bfloat16)
    OP.store_layer_tokens(arena, OP.slot_mapping(table, list(range(n)), P), k, v)
    darena = arena.cuda()
    bt = torch.tensor([table], dtype=torch.int32, device="cuda")
    pos = torch.tensor([n - K], dtype=torch.int64, device="cuda")
    dq = q[None].cuda()
    out = torch.zeros_like(dq)
    ws = torch.empty(ops.decode_workspace_bytes(1, K, 32, 8, n, kv_capacity=0, page_size=P),
                     dtype=torch.uint8, device="cuda")
    torch.ops.solort_attn.gqa_decode_paged(dq, darena, bt, pos, out, ws, n, SCALE)  # warm-up
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        torch.ops.solort_attn.gqa_decode_paged(dq, darena, bt, pos, out, ws, n, SCALE)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    ref, _ = A.attention_fp32(q, k, v, SCALE, n - K)
    _close(out[0], ref, "captured paged verify")


def test_gqa_prefill_op_captured():
    T = 700
    q, k, v = A.make_attention_inputs(9, 32, 8, 128, T, T, 0)
    dq, dk, dv = q.cuda(), k.cuda(), v.cuda()
    out = torch.empty_like(dq)
    torch.ops.solort_attn.gqa_prefill(dq, dk, dv, out, True, SCALE)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        torch.ops.solort_attn.gqa_prefill(dq, dk, dv, out, True, SCALE)
    out.zero_()
    graph.replay()
    torch.cuda.synchronize()
    ref, _ = A.attention_fp32(q, k, v, SCALE, 0)
    _close(out, ref, "captured prefill")


def test_partial_and_lse_merge_ops_equal_one_decode():
    """Two key shards through gqa_decode_partial, merged by lse_merge, against the whole decode."""
    ops = _ops()
    L = 6000
    q, k, v = A.make_attention_inputs(10, 32, 8, 128, 1, L, L - 1)
    dq, dk, dv = q[None].cuda(), k.cuda(), v.cuda()
    pos = torch.tensor([L - 1], dtype=torch.int64, device="cuda")
    half = 3000
    o = torch.empty(2, 1, 1, 32, 128, dtype=torch.float32, device="cuda")
    lse = torch.empty(2, 1, 1, 32, dtype=torch.float32, device="cuda")
    for r, (s, e) in enumerate(((0, half), (half, L))):
        ws = torch.empty(ops.decode_workspace_bytes(1, 1, 32, 8, e - s), dtype=torch.uint8,
                         device="cuda")
        torch.ops.solort_attn.gqa_decode_partial(dq, dk[s:e], dv[s:e], pos, o[r], lse[r], ws, s)
    out = torch.empty_like(dq)
    torch.ops.solort_attn.lse_merge(o, lse, out)
    torch.cuda.synchronize()
    ref, ref_lse = A.attention_fp32(q, k, v, SCALE, L - 1)
    _close(out[0], ref, "partial + merge")
    o32, lse32 = ops.lse_merge(o, lse, return_lse=True)
    assert (lse32[0, 0].cpu() - ref_lse[0]).abs().max().item() <= 1e-3


def test_kv_store_is_the_reference_slot_mapped_store():
    """``kv_store`` writes exactly what ``store_layer_tokens``'s loop writes (bit-exact), from the
    HF layout ``[1, nkv, kv, 128]`` (a strided view of its last tokens), and nothing else."""
    ops = _ops()
    P, pages, nkv, kv_len, tc = 16, 40, 8, 300, 37
    g = torch.Generator().manual_seed(11)
    key = torch.randn(1, nkv, kv_len, 128, generator=g).to(torch.bfloat16)
    value = torch.randn(1, nkv, kv_len, 128, generator=g).to(torch.bfloat16)
    arena = torch.randn(pages, 2, P, nkv, 128, generator=g).to(torch.bfloat16)
    table = torch.randperm(pages, generator=g)[:20].tolist()
    slots = OP.slot_mapping(table, list(range(kv_len - tc, kv_len)), P)
    expect = arena.clone()
    OP.store_layer_tokens(expect, slots, key[0, :, -tc:].transpose(0, 1), value[0, :, -tc:].transpose(0, 1))
    darena = arena.cuda()
    dkey, dval = key.cuda(), value.cuda()
    ops.kv_store(dkey[0, :, -tc:].transpose(0, 1), dval[0, :, -tc:].transpose(0, 1),
                 torch.tensor(slots, dtype=torch.int64, device="cuda"), darena)
    torch.cuda.synchronize()
    assert torch.equal(darena.cpu(), expect)
    assert ops.device_status() == 0


def test_kv_store_skips_slots_outside_the_arena_and_reports_them():
    """A slot past the arena is not written (the kernel checks each slot against the arena size
    before its store) and raises bit 4 of the device status; the other rows are stored."""
    ops = _ops()
    P, pages = 16, 4
    arena = torch.zeros(pages, 2, P, 8, 128, dtype=torch.bfloat16, device="cuda")
    key = torch.ones(3, 8, 128, dtype=torch.bfloat16, device="cuda")
    slots = torch.tensor([5, pages * P + 3, 17], dtype=torch.int64, device="cuda")
    ops.kv_store(key, key * 2, slots, arena)
    torch.cuda.synchronize()
    assert ops.device_status() == 1 << 4
    flat_k = arena[:, 0].reshape(-1, 8, 128)
    flat_v = arena[:, 1].reshape(-1, 8, 128)
    assert (flat_k[[5, 17]] == 1).all() and (flat_v[[5, 17]] == 2).all()
    written = torch.zeros(pages * P, dtype=torch.bool)
    written[[5, 17]] = True
    assert (flat_k[~written.cuda()] == 0).all() and (flat_v[~written.cuda()] == 0).all()
    assert ops.device_status() == 0  # read-and-clear
