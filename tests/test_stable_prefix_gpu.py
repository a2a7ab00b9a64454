"""SOLORT_DECODE_STABLE_PREFIX: keys below q_pos are requested before the previous kernel finishes.

The flag changes only when loads are issued, never what is computed, so flagged and unflagged calls
must agree bit for bit; and when the previous kernel is the prologue that appends this step's key
and value at q_pos (the runner's order), the appended row must still be read after that kernel: the
cache holds a large constant at the appended positions beforehand, so a stale read would move the
output far outside the tolerance against the fp32 oracle.
"""

from __future__ import annotations

import pytest
import torch

from oracle import attention as A

pytestmark = pytest.mark.gpu

NH, NKV, HD, EPS = 32, 8, 128, 1e-6


def _ops():
    from solort_b200 import ops

    return ops


@pytest.mark.parametrize("L,q_len", [(1, 1), (32, 1), (33, 1), (224, 1), (225, 1), (8192, 1),
                                     (3000, 4), (4097, 8)])
def test_flag_gives_the_same_bits_static(L, q_len):
    ops = _ops()
    q, k, v = A.make_attention_inputs(L + q_len, NH, NKV, HD, q_len, L, L - q_len)
    dq, dk, dv = q[None].cuda(), k.cuda(), v.cuda()
    qpos = torch.tensor([L - q_len], dtype=torch.int64, device="cuda")
    a = ops.gqa_decode(dq, dk, dv, qpos)
    b = ops.gqa_decode(dq, dk, dv, qpos, stable_prefix=True)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert ops.device_status() == 0


def test_flag_gives_the_same_bits_paged():
    ops = _ops()
    P, pages = 16, 96
    g = torch.Generator(device="cuda").manual_seed(5)
    arena = torch.randn(pages, 2, P, NKV, HD, generator=g, device="cuda").to(torch.bfloat16)
    perm = torch.randperm(pages, generator=torch.Generator().manual_seed(1)).to(torch.int32)
    bt = perm.view(1, pages).cuda()
    q = torch.randn(1, 4, NH, HD, generator=g, device="cuda").to(torch.bfloat16)
    qpos = torch.tensor([1000], dtype=torch.int64, device="cuda")
    a = ops.gqa_decode_paged(q, arena, bt, qpos, max_kv_len=1004)
    b = ops.gqa_decode_paged(q, arena, bt, qpos, max_kv_len=1004, stable_prefix=True)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


def test_appended_row_is_read_after_the_prologue_in_a_graph():
    """Prologue (append at pos) -> decode (flagged) for 6 layers in one graph, replayed at moving
    positions: equal to the unflagged graph and to the oracle over the appended cache."""
    ops = _ops()
    layers, max_len = 6, 2048
    g = torch.Generator().manual_seed(3)
    qkv = (torch.randn(layers, 1, (NH + 2 * NKV) * HD, generator=g) * 2).to(torch.bfloat16).cuda()
    qn = (1 + 0.1 * torch.randn(HD, generator=g)).to(torch.bfloat16).cuda()
    kn = (1 + 0.1 * torch.randn(HD, generator=g)).to(torch.bfloat16).cuda()
    cos, sin = A.cos_sin(torch.arange(max_len, device="cuda"), A.inv_freq(HD, 1e6, "cuda"),
                         torch.bfloat16)
    hist = torch.randn(layers, 2, max_len, NKV, HD, generator=g).to(torch.bfloat16).cuda()
    pos_buf = torch.zeros(1, dtype=torch.int64, device="cuda")
    ws = torch.zeros(ops.decode_workspace_bytes(1, 1, NH, NKV, max_len), dtype=torch.uint8,
                     device="cuda")

    def build(flag):
        kc = torch.empty(layers, max_len, NKV, HD, dtype=torch.bfloat16, device="cuda")
        vc = torch.empty_like(kc)
        out = torch.empty(layers, 1, 1, NH, HD, dtype=torch.bfloat16, device="cuda")

        def step():
            for li in range(layers):
                qq = ops.qk_norm_rope_append(qkv[li], qn, kn, EPS, cos, sin, pos_buf, kc[li],
                                             vc[li], num_qo_heads=NH, num_kv_heads=NKV)
                ops.gqa_decode(qq.view(1, 1, NH, HD), kc[li], vc[li], pos_buf, out=out[li],
                               workspace=ws, stable_prefix=flag)

        pos_buf.fill_(0)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
        return graph, kc, vc, out

    runs = {flag: build(flag) for flag in (False, True)}
    for pos in (0, 31, 32, 223, 224, 225, 1000, 2047):
        outs = {}
        for flag, (graph, kc, vc, out) in runs.items():
            kc.copy_(hist[:, 0])
            vc.copy_(hist[:, 1])
            kc[:, pos:].fill_(30.0)  # what a read before the append would see
            vc[:, pos:].fill_(30.0)
            pos_buf.fill_(pos)
            graph.replay()
            torch.cuda.synchronize()
            outs[flag] = out.clone()
        assert torch.equal(outs[True], outs[False]), f"pos {pos}"
        graph, kc, vc, out = runs[True]
        for li in (0, layers - 1):
            q_l = ops.qk_norm_rope_append(qkv[li], qn, kn, EPS, cos, sin, pos_buf,
                                          kc[li].clone(), vc[li].clone(), num_qo_heads=NH,
                                          num_kv_heads=NKV)
            ref, _ = A.attention_fp32(q_l.view(1, NH, HD).cpu(), kc[li, : pos + 1].cpu(),
                                      vc[li, : pos + 1].cpu(), HD**-0.5, pos)
            d = (out[li, 0, 0].float().cpu() - ref[0].float()).abs()
            assert d.max().item() <= 2e-2 and d.mean().item() <= 2e-3, (pos, li, d.max().item())
    assert ops.device_status() == 0
    for graph, *_ in runs.values():
        del graph
