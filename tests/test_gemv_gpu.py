"""The decode-step weight stream (``ops.gemv``) against an fp32 evaluation of the same bf16
operands: both accumulate in fp32 and round once to bf16, so results may differ only by the
accumulation order (checked: max-abs <= 1e-2 * max|ref| + 1e-3)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("t,n,k", [(1, 6144, 2560), (1, 2560, 4096), (5, 19456, 2560), (8, 37, 264),
                                   (3, 151936, 2560), (2, 100, 8), (1, 5, 40000), (3, 1000, 2568),
                                   (8, 2560, 9728), (1, 149, 1024)])
def test_gemv_matches_fp32(t, n, k):
    from solort_b200 import ops

    g = torch.Generator().manual_seed(t * 1000 + n + k)
    a = torch.randn(t, k, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).to(torch.bfloat16).cuda()
    ref = a.float() @ w.float().T
    y = ops.gemv(a, w)
    torch.cuda.synchronize()
    d = (y.float() - ref).abs().max().item()
    assert d <= 1e-2 * ref.abs().max().item() + 1e-3, f"{t}x{n}x{k}: {d}"
    assert ops.device_status() == 0


@pytest.mark.parametrize("t,n,k", [(1, 2560, 9728), (4, 2560, 9728), (7, 64, 136), (8, 2560, 9728)])
def test_gemv_fused_silu_gate_up(t, n, k):
    from solort_b200 import ops

    g = torch.Generator().manual_seed(t + n + k)
    gu = (2 * torch.randn(t, 2 * k, generator=g)).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).to(torch.bfloat16).cuda()
    gate, up = gu.split([k, k], dim=-1)
    act = F.silu(gate) * up  # the reference MLP's bf16 activation
    ref = act.float() @ w.float().T
    y = ops.gemv(gu, w, silu_gate_up=True)
    torch.cuda.synchronize()
    d = (y.float() - ref).abs().max().item()
    assert d <= 1e-2 * ref.abs().max().item() + 1e-3, f"{t}x{n}x{k}: {d}"


def test_gemv_is_deterministic():
    """Rows cut between warps are summed in a fixed order: repeated calls agree bit for bit."""
    from solort_b200 import ops

    g = torch.Generator().manual_seed(7)
    a = torch.randn(2, 9728, generator=g).to(torch.bfloat16).cuda()
    w = (torch.randn(2560, 9728, generator=g) / 100).to(torch.bfloat16).cuda()
    first = ops.gemv(a, w)
    for _ in range(5):
        assert torch.equal(ops.gemv(a, w), first)


@pytest.mark.parametrize("t,n,k", [(1, 6144, 2560), (2, 19456, 2560), (1, 151936, 2560), (3, 40, 264)])
def test_gemv_fused_residual_rmsnorm_is_add_rmsnorm_then_gemv(t, n, k):
    """Mode 2 reproduces add_rmsnorm + gemv bit for bit (same reduction order), writes the
    residual sum once, and matches the reference's fp32 _rmsnorm followed by the matmul."""
    from solort_b200 import ops

    g = torch.Generator().manual_seed(t * 7 + n + k)
    x = torch.randn(t, k, generator=g).to(torch.bfloat16).cuda()
    d = torch.randn(t, k, generator=g).to(torch.bfloat16).cuda()
    nw = (1 + 0.1 * torch.randn(k, generator=g)).to(torch.bfloat16).cuda()
    w = (torch.randn(n, k, generator=g) / k ** 0.5).to(torch.bfloat16).cuda()
    x_new, h = ops.add_rmsnorm(x, d, nw, 1e-6, x_out=torch.empty_like(x))
    want = ops.gemv(h, w)
    x_out = torch.full_like(x, float("nan"))
    y = ops.gemv(x, w, norm_weight=nw, delta=d, x_out=x_out, eps=1e-6)
    torch.cuda.synchronize()
    assert torch.equal(y, want)
    assert torch.equal(x_out, x_new)
    xs = (x.float() + d.float()).to(torch.bfloat16).float()
    hr = ((xs * torch.rsqrt(xs.pow(2).mean(-1, keepdim=True) + 1e-6)) * nw.float()).to(torch.bfloat16)
    ref = hr.float() @ w.float().T
    assert (y.float() - ref).abs().max().item() <= 1e-2 * ref.abs().max().item() + 1e-3

    # without delta: the norm of x itself, nothing written
    _, h0 = ops.add_rmsnorm(x, None, nw, 1e-6)
    assert torch.equal(ops.gemv(x, w, norm_weight=nw, eps=1e-6), ops.gemv(h0, w))


def test_gemv_fused_norm_rejects_aliased_residual():
    from solort_b200 import ops

    x = torch.randn(1, 256, device="cuda").to(torch.bfloat16)
    d = torch.randn(1, 256, device="cuda").to(torch.bfloat16)
    nw = torch.ones(256, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(64, 256, device="cuda").to(torch.bfloat16)
    with pytest.raises(RuntimeError):
        ops.gemv(x, w, norm_weight=nw, delta=d, x_out=x)

