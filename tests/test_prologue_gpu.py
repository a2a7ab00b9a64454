"""The fused attention prologue (QK-RMSNorm + RoPE + KV append) against the reference's torch ops.

The reference ops run on the same GPU (``oracle.attention.rmsnorm / rope`` with the model's bf16
cos/sin tables, ``cuda_graph_executor.py:25-28, 95-102``). RoPE rounding is reproduced step by step
and V rows are copied, so differences come only from the fp32 sum-of-squares order inside RMSNorm:
queries and keys may differ by one bf16 step in rare elements (checked: max-abs <= 2e-2, and at most
1% of elements differ at all); V rows must match bit for bit; nothing outside the appended rows may
change.
"""

from __future__ import annotations

import pytest
import torch

from oracle import attention as A
from oracle import paged as OP

pytestmark = pytest.mark.gpu

NH, NKV, HD, EPS = 32, 8, 128, 1e-6


def _inputs(seed, t, max_len):
    g = torch.Generator().manual_seed(seed)
    qkv = (torch.randn(t, (NH + 2 * NKV) * HD, generator=g) * 2).to(torch.bfloat16).cuda()
    qn = (1 + 0.1 * torch.randn(HD, generator=g)).to(torch.bfloat16).cuda()
    kn = (1 + 0.1 * torch.randn(HD, generator=g)).to(torch.bfloat16).cuda()
    cos, sin = A.cos_sin(torch.arange(max_len, device="cuda"), A.inv_freq(HD, 1e6, "cuda"),
                         torch.bfloat16)
    return qkv, qn, kn, cos, sin


def _reference(qkv, qn, kn, cos, sin, pos0):
    t = qkv.shape[0]
    q, k, v = qkv.split([NH * HD, NKV * HD, NKV * HD], dim=-1)
    rows = torch.arange(pos0, pos0 + t, device=qkv.device)
    c, s = cos[rows][:, None, :], sin[rows][:, None, :]
    q = A.rope(A.rmsnorm(q.view(t, NH, HD), qn, EPS), c, s)
    k = A.rope(A.rmsnorm(k.view(t, NKV, HD), kn, EPS), c, s)
    return q, k, v.view(t, NKV, HD)


def _close(got, ref, what):
    d = (got.float() - ref.float()).abs()
    assert d.max().item() <= 2e-2, f"{what}: max-abs {d.max().item():.4g}"
    frac = (d > 0).float().mean().item()
    assert frac <= 0.01, f"{what}: {frac:.4%} of elements differ"


@pytest.mark.parametrize("t,pos0", [(1, 0), (1, 4095), (5, 700), (512, 0), (1024, 0)])
def test_static_prologue_matches_reference_ops(t, pos0):
    from solort_b200 import ops

    max_len = 4096
    qkv, qn, kn, cos, sin = _inputs(t * 31 + pos0, t, max_len)
    kc = torch.full((max_len, NKV, HD), 7.0, dtype=torch.bfloat16, device="cuda")
    vc = kc.clone()
    pos = torch.tensor([pos0], dtype=torch.int64, device="cuda")
    q = ops.qk_norm_rope_append(qkv, qn, kn, EPS, cos, sin, pos, kc, vc,
                                num_qo_heads=NH, num_kv_heads=NKV)
    torch.cuda.synchronize()
    rq, rk, rv = _reference(qkv, qn, kn, cos, sin, pos0)
    _close(q, rq, "queries")
    _close(kc[pos0:pos0 + t], rk, "appended keys")
    assert torch.equal(vc[pos0:pos0 + t], rv), "appended values must be exact copies"
    outside = torch.ones(max_len, dtype=torch.bool)
    outside[pos0:pos0 + t] = False
    assert (kc[outside.cuda()] == 7.0).all() and (vc[outside.cuda()] == 7.0).all()
    assert ops.device_status() == 0


def test_prologue_skips_rows_past_the_cache():
    from solort_b200 import ops

    max_len = 64
    qkv, qn, kn, cos, sin = _inputs(3, 8, 128)
    kc = torch.zeros((max_len, NKV, HD), dtype=torch.bfloat16, device="cuda")
    vc = kc.clone()
    pos = torch.tensor([60], dtype=torch.int64, device="cuda")  # rows 60..67: four fit
    ops.qk_norm_rope_append(qkv, qn, kn, EPS, cos, sin, pos, kc, vc, num_qo_heads=NH,
                            num_kv_heads=NKV)
    torch.cuda.synchronize()
    _, rk, rv = _reference(qkv, qn, kn, cos, sin, 60)
    _close(kc[60:64], rk[:4], "keys that fit")
    assert torch.equal(vc[60:64], rv[:4])
    assert (kc[:60] == 0).all()


@pytest.mark.parametrize("P,t,pos0", [(16, 1, 1023), (16, 5, 30), (8, 40, 3), (64, 3, 127)])
def test_paged_prologue_writes_the_reference_slots(P, t, pos0):
    """Appends through a permuted block table land in the slots of ``kv_cache.py:136-149``."""
    from solort_b200 import ops

    n_pages = (pos0 + t + P - 1) // P + 4
    g = torch.Generator().manual_seed(P * 7 + t)
    table = torch.randperm(n_pages, generator=g)[: (pos0 + t + P - 1) // P].tolist()
    arena = torch.full((n_pages, 2, P, NKV, HD), 5.0, dtype=torch.bfloat16, device="cuda")
    qkv, qn, kn, cos, sin = _inputs(P + t, t, 2048)
    bt = torch.tensor(table, dtype=torch.int32, device="cuda")
    pos = torch.tensor([pos0], dtype=torch.int64, device="cuda")
    ops.qk_norm_rope_append(qkv, qn, kn, EPS, cos, sin, pos, arena[:, 0], arena[:, 1],
                            num_qo_heads=NH, num_kv_heads=NKV, block_table=bt)
    torch.cuda.synchronize()
    _, rk, rv = _reference(qkv, qn, kn, cos, sin, pos0)
    slots = OP.slot_mapping(table, list(range(pos0, pos0 + t)), P)
    flat = arena.view(n_pages, 2, P, NKV, HD).transpose(0, 1).reshape(2, n_pages * P, NKV, HD)
    _close(flat[0, slots], rk, "paged keys")
    assert torch.equal(flat[1, slots], rv)
    untouched = torch.ones(n_pages * P, dtype=torch.bool)
    untouched[slots] = False
    assert (flat[:, untouched.cuda()] == 5.0).all()
