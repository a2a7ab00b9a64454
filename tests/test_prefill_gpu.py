"""GPU parity of the tcgen05 prefill kernel against the CPU oracle (max-abs <= 2e-2,
mean-abs <= 2e-3 against fp32 softmax attention over the same bf16 inputs)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as A

pytestmark = pytest.mark.gpu

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _close(got, ref, what):
    d = (got.float().cpu() - ref.float().cpu()).abs()
    assert torch.isfinite(got.float()).all(), f"{what}: non-finite"
    assert d.max().item() <= MAX_ABS, f"{what}: max-abs {d.max().item():.4g}"
    assert d.mean().item() <= MEAN_ABS, f"{what}: mean-abs {d.mean().item():.4g}"


@pytest.mark.parametrize("T", [1, 17, 128, 200, 256, 511, 512, 1024])
@pytest.mark.parametrize("nh,nkv", [(32, 8), (16, 8)])
def test_prefill_causal_square(T, nh, nkv):
    from solort_b200 import ops

    q, k, v = A.make_attention_inputs(T + nh, nh, nkv, 128, T, T, 0)
    ref, _ = A.attention_fp32(q, k, v, 128 ** -0.5, 0)
    out = ops.gqa_prefill(q.cuda(), k.cuda(), v.cuda())
    torch.cuda.synchronize()
    _close(out, ref, f"prefill T={T} {nh}/{nkv}")
    assert ops.device_status() == 0


@pytest.mark.parametrize("q_len,kv_len", [(3, 7), (100, 300), (128, 1000), (257, 513)])
def test_prefill_bottom_right_over_cache(q_len, kv_len):
    """Chunked prefill / verify over a populated cache: bottom-right causal alignment
    (transformers_flashinfer.py:182-193)."""
    from solort_b200 import ops

    q, k, v = A.make_attention_inputs(q_len * 3 + kv_len, 32, 8, 128, q_len, kv_len, kv_len - q_len)
    ref, _ = A.attention_fp32(q, k, v, 128 ** -0.5, kv_len - q_len)
    out = ops.gqa_prefill(q.cuda(), k.cuda(), v.cuda())
    _close(out, ref, f"bottom-right q={q_len} kv={kv_len}")
    lit = A.sdpa_bottom_right(q.transpose(0, 1)[None].float(), k.transpose(0, 1)[None].float(),
                              v.transpose(0, 1)[None].float(), 128 ** -0.5, causal=True)[0]
    _close(out, lit, "vs the bridge's torch fallback")


@pytest.mark.parametrize("q_len,kv_len,nh,causal",
                         [(1900, 1900, 32, True), (1900, 1900, 16, True), (1500, 1800, 32, True),
                          (1000, 2000, 32, False)])
def test_prefill_persistent_items(q_len, kv_len, nh, causal):
    """More (query tile, head) items than SMs: each persistent CTA of the one-tile kernel walks
    several items (up to four at q_len 1900 with 32 heads on 148 SMs), with the Q and O buffers
    alternating between items and each output tile stored after the next item's first tile."""
    from solort_b200 import ops

    off = kv_len - q_len if causal else 10 ** 6
    q, k, v = A.make_attention_inputs(11 + q_len + nh, nh, 8, 128, q_len, kv_len,
                                      kv_len - q_len)
    ref, _ = A.attention_fp32(q, k, v, 128 ** -0.5, off)
    out = ops.gqa_prefill(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    torch.cuda.synchronize()
    _close(out, ref, f"persistent q={q_len} kv={kv_len} nh={nh} causal={causal}")
    assert ops.device_status() == 0


def test_prefill_persistent_head_major_views():
    """The persistent kernel over head-major storage ([heads, T, hd] tensors viewed as [T, heads,
    hd]): the tensor maps then take (dim, token, head) coordinates instead of (dim, head, token)."""
    from solort_b200 import ops

    T, nh, nkv = 1100, 32, 8  # 9 query tiles x 32 heads = 288 items on at most 148 CTAs
    q, k, v = A.make_attention_inputs(21, nh, nkv, 128, T, T, 0)
    qh = q.transpose(0, 1).contiguous().cuda().transpose(0, 1)
    kh = k.transpose(0, 1).contiguous().cuda().transpose(0, 1)
    vh = v.transpose(0, 1).contiguous().cuda().transpose(0, 1)
    assert qh.stride(1) > qh.stride(0)
    ref, _ = A.attention_fp32(q, k, v, 128 ** -0.5, 0)
    out = ops.gqa_prefill(qh, kh, vh)
    torch.cuda.synchronize()
    _close(out, ref, "persistent, head-major views")
    assert ops.device_status() == 0


@pytest.mark.parametrize("nh,nkv,T", [
    (64, 8, 700),      # group 8, one CTA per (query tile, head)
    (48, 16, 1100),    # group 3, persistent kernel (9 tiles x 48 heads = 432 items)
    (32, 2, 1500),     # group 16, persistent kernel
    (12, 12, 900),     # group 1 (multi-head), 12 heads
    (40, 8, 2300),     # group 5, two-tile kernel (9 pairs x 40 heads = 360 CTAs)
    (8, 1, 2100),      # group 8 over a single KV head, two-tile kernel with an odd tile count
])
def test_prefill_other_group_sizes(nh, nkv, T):
    """GQA groups other than Qwen3's, across the three prefill kernels: query head h reads KV head
    h / (nh / nkv) through the tensor maps, with no K/V expansion."""
    from solort_b200 import ops

    q, k, v = A.make_attention_inputs(T + 17 * nh + nkv, nh, nkv, 128, T, T, 0)
    ref, _ = A.attention_fp32(q, k, v, 128 ** -0.5, 0)
    out = ops.gqa_prefill(q.cuda(), k.cuda(), v.cuda())
    torch.cuda.synchronize()
    _close(out, ref, f"prefill nh={nh} nkv={nkv} T={T}")
    assert ops.device_status() == 0


def test_prefill_non_causal():
    from solort_b200 import ops

    q, k, v = A.make_attention_inputs(5, 32, 8, 128, 130, 390, 389)
    ref, _ = A.attention_fp32(q, k, v, 128 ** -0.5, 10 ** 6)
    out = ops.gqa_prefill(q.cuda(), k.cuda(), v.cuda(), causal=False)
    _close(out, ref, "non-causal")


def test_prefill_strided_qkv_view():
    """q/k/v as views into one fused QKV GEMM output, as the reference slices them
    (cuda_graph_executor.py:115-119)."""
    from solort_b200 import ops

    T, nh, nkv = 300, 32, 8
    q, k, v = A.make_attention_inputs(9, nh, nkv, 128, T, T, 0)
    qkv = torch.cat([q.reshape(T, -1), k.reshape(T, -1), v.reshape(T, -1)], -1).cuda()
    qv = qkv[:, : nh * 128].view(T, nh, 128)
    kv_ = qkv[:, nh * 128 : (nh + nkv) * 128].view(T, nkv, 128)
    vv = qkv[:, (nh + nkv) * 128 :].view(T, nkv, 128)
    ref, _ = A.attention_fp32(q, k, v, 128 ** -0.5, 0)
    _close(ops.gqa_prefill(qv, kv_, vv), ref, "strided views")


def test_prefill_golden_runner():
    """The reference runner's own prefill attention tensors (tests/golden/runner_attention.npz)."""
    from solort_b200 import ops

    d = np.load("tests/golden/runner_attention.npz")
    for li in range(2):
        q = torch.from_numpy(d[f"prefill.l{li}.q"]).to(torch.bfloat16).transpose(0, 1).contiguous()
        k = torch.from_numpy(d[f"prefill.l{li}.k"]).to(torch.bfloat16).transpose(0, 1).contiguous()
        v = torch.from_numpy(d[f"prefill.l{li}.v"]).to(torch.bfloat16).transpose(0, 1).contiguous()
        ref = torch.from_numpy(d[f"prefill.l{li}.out"]).transpose(0, 1)
        _close(ops.gqa_prefill(q.cuda(), k.cuda(), v.cuda()), ref, f"golden prefill l{li}")


# Prompts of 16 or more 128-row tiles take the two-tile ping-pong kernel.
@pytest.mark.parametrize("T,nh,nkv", [(2048, 16, 8), (2049, 16, 8), (2300, 32, 8), (4096, 8, 8)])
def test_prefill_ping_pong_causal(T, nh, nkv):
    from solort_b200 import ops

    q, k, v = A.make_attention_inputs(T * 3 + nh, nh, nkv, 128, T, T, 0)
    ref, _ = A.attention_fp32(q, k, v, 128 ** -0.5, 0)
    out = ops.gqa_prefill(q.cuda(), k.cuda(), v.cuda())
    torch.cuda.synchronize()
    _close(out, ref, f"ping-pong prefill T={T} {nh}/{nkv}")
    assert ops.device_status() == 0


@pytest.mark.parametrize("q_len,kv_len,causal", [(2100, 3000, True), (2048, 2500, False)])
def test_prefill_ping_pong_over_cache(q_len, kv_len, causal):
    from solort_b200 import ops

    q, k, v = A.make_attention_inputs(q_len + kv_len, 16, 8, 128, q_len, kv_len, kv_len - q_len)
    ref, _ = A.attention_fp32(q, k, v, 128 ** -0.5, (kv_len - q_len) if causal else 10 ** 7)
    out = ops.gqa_prefill(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    torch.cuda.synchronize()
    _close(out, ref, f"ping-pong q={q_len} kv={kv_len} causal={causal}")
    assert ops.device_status() == 0


def test_prefill_full_size_config3():
    """BASELINE config 3 at its largest size (T = 4096, 32 query / 8 KV heads), against the same
    fp32 attention evaluated on the device (too slow on the host at this size)."""
    from solort_b200 import ops

    T = 4096
    q, k, v = A.make_attention_inputs(4242, 32, 8, 128, T, T, 0)
    dq, dk, dv = q.cuda(), k.cuda(), v.cuda()
    out = ops.gqa_prefill(dq, dk, dv)
    ref, _ = A.attention_fp32(dq, dk, dv, 128 ** -0.5, 0)
    torch.cuda.synchronize()
    _close(out, ref, "prefill T=4096 32/8")
    assert ops.device_status() == 0
