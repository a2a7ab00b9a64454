"""CPU restatement of the reference's GQA attention (test infrastructure only).

Every function here is the checker for one CUDA entry point of ``solort_b200``. Citations are
``path:line`` inside the reference project (owen920831/SoloRT).

Two kinds of oracle live here:

* ``attention_fp32`` -- the parity oracle named by the engine's contract: the same bf16 Q/K/V
  upcast to fp32, fp32 scores and softmax, GQA by head grouping, and an absolute-position causal
  limit (query row ``i`` at position ``q_pos0 + i`` sees keys at positions ``<= q_pos0 + i``).
  That one rule covers the reference's decode mask (``cuda_graph_executor.py:168``), its verify
  mask (``:250``), its square causal prefill (``:127``) and the HF bridge's bottom-right causal
  alignment (``transformers_flashinfer.py:182-193``).
* ``decode_reference_grouped`` / ``prefill_reference`` / ``verify_reference`` /
  ``sdpa_bottom_right`` -- literal restatements of the reference's own torch code (bf16 scores in
  the grouped decode, SDPA with ``repeat_interleave`` in prefill and verify). They are pinned to
  the reference bit-for-bit by the golden fixtures and are what ``bench.py`` times as the
  reference's CPU path.
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

LOG2E = 1.4426950408889634


# --------------------------------------------------------------------------------------------
# Input pipeline: QK-RMSNorm and rotate-half RoPE exactly as the reference applies them.
# --------------------------------------------------------------------------------------------


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """RMSNorm in fp32, cast back (``cuda_graph_executor.py:25-28``)."""
    d = x.float()
    d = d * torch.rsqrt(d.pow(2).mean(-1, keepdim=True) + eps)
    return (d * w.float()).to(x.dtype)


def inv_freq(head_dim: int, theta: float, device: torch.device | str = "cpu") -> torch.Tensor:
    """``1 / theta ** (arange(0, hd, 2) / hd)`` (``cuda_graph_executor.py:64-66``)."""
    return 1.0 / (float(theta) ** (torch.arange(0, head_dim, 2, device=device).float() / head_dim))


def cos_sin(positions: torch.Tensor, freqs: torch.Tensor, dtype: torch.dtype):
    """cos/sin tables cast to the model dtype (``cuda_graph_executor.py:95-98``)."""
    f = positions[:, None].float() * freqs[None, :]
    emb = torch.cat([f, f], -1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE (``cuda_graph_executor.py:100-102``)."""
    d = x.shape[-1] // 2
    return x * cos + torch.cat([-x[..., d:], x[..., :d]], -1) * sin


def make_attention_inputs(
    seed: int,
    num_qo_heads: int,
    num_kv_heads: int,
    head_dim: int,
    n_q: int,
    n_kv: int,
    q_pos0: int,
    *,
    theta: float = 1e6,
    eps: float = 1e-6,
    dtype: torch.dtype = torch.bfloat16,
    device: str = "cpu",
):
    """Seeded synthetic attention inputs with the reference's input pipeline.

    Q, K, V ~ N(0, 1) in ``dtype``; per-head RMSNorm (unit weight, ``eps``) on Q and K; RoPE
    (``theta``) at positions ``q_pos0 .. q_pos0 + n_q - 1`` for Q and ``0 .. n_kv - 1`` for K.
    Layout is token-major NHD: ``q [n_q, nh, hd]``, ``k, v [n_kv, nkv, hd]``. This follows the
    per-layer steps of ``_decode_forward`` (``cuda_graph_executor.py:173-177``) on random
    projections instead of weights.
    """
    g = torch.Generator(device=device)
    g.manual_seed(int(seed))
    q = torch.randn(n_q, num_qo_heads, head_dim, generator=g, device=device).to(dtype)
    k = torch.randn(n_kv, num_kv_heads, head_dim, generator=g, device=device).to(dtype)
    v = torch.randn(n_kv, num_kv_heads, head_dim, generator=g, device=device).to(dtype)
    ones = torch.ones(head_dim, dtype=dtype, device=device)
    freqs = inv_freq(head_dim, theta, device)
    qc, qs = cos_sin(torch.arange(q_pos0, q_pos0 + n_q, device=device), freqs, dtype)
    kc, ks = cos_sin(torch.arange(0, n_kv, device=device), freqs, dtype)
    q = rope(rmsnorm(q, ones, eps), qc[:, None, :], qs[:, None, :])
    k = rope(rmsnorm(k, ones, eps), kc[:, None, :], ks[:, None, :])
    return q.contiguous(), k.contiguous(), v.contiguous()


# --------------------------------------------------------------------------------------------
# The parity oracle.
# --------------------------------------------------------------------------------------------


def attention_fp32(
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    scale: float,
    q_pos0: int,
    *,
    kv_pos0: int = 0,
    q_chunk: int = 256,
):
    """fp32 GQA attention with an absolute-position causal limit.

    ``q [n_q, nh, hd]``, ``k, v [n_kv, nkv, hd]`` (any float dtype, upcast to fp32). Query row
    ``i`` (position ``q_pos0 + i``) attends key ``j`` (position ``kv_pos0 + j``) iff
    ``kv_pos0 + j <= q_pos0 + i``. Query head ``h`` reads KV head ``h // (nh // nkv)``, which is
    ``repeat_interleave(groups, 0)`` in ``cuda_graph_executor.py:124-125`` and the
    ``[nkv, groups, hd]`` view in ``:180``.

    Returns ``(out fp32 [n_q, nh, hd], lse fp32 [n_q, nh])`` with the natural-log LSE of the
    scaled scores. Rows that see no key get ``out = 0`` and ``lse = -inf``.
    """
    n_q, nh, hd = q.shape
    n_kv, nkv, _ = k.shape
    groups = nh // nkv
    kf = k.float().permute(1, 0, 2)  # [nkv, n_kv, hd]
    vf = v.float().permute(1, 0, 2)
    dev = q.device
    kpos = kv_pos0 + torch.arange(n_kv, device=dev)
    outs, lses = [], []
    for s in range(0, n_q, q_chunk):
        e = min(n_q, s + q_chunk)
        qf = q[s:e].float().permute(1, 0, 2).reshape(nkv, groups * (e - s), hd)
        sc = torch.matmul(qf, kf.transpose(1, 2)).view(nkv, groups, e - s, n_kv) * scale
        qpos = q_pos0 + torch.arange(s, e, device=dev)
        visible = kpos[None, :] <= qpos[:, None]  # [rows, n_kv]
        sc = sc.masked_fill(~visible.view(1, 1, e - s, n_kv), float("-inf"))
        lse = torch.logsumexp(sc, -1)  # [nkv, g, rows]
        p = torch.exp(sc - lse[..., None])
        p = torch.nan_to_num(p, nan=0.0)
        o = torch.matmul(p.view(nkv, groups * (e - s), n_kv), vf).view(nkv, groups, e - s, hd)
        outs.append(o.permute(2, 0, 1, 3).reshape(e - s, nh, hd))
        lses.append(lse.permute(2, 0, 1).reshape(e - s, nh))
    return torch.cat(outs, 0), torch.cat(lses, 0)


def lse_merge(o_parts: torch.Tensor, lse_parts: torch.Tensor):
    """Merge partial attention results over disjoint key sets.

    ``o_parts [R, ..., hd]`` are per-part normalised outputs and ``lse_parts [R, ...]`` their
    natural-log LSEs. ``O = sum_r exp(lse_r - lse*) O_r / sum_r exp(lse_r - lse*)`` and
    ``lse = lse* + log(sum_r exp(lse_r - lse*))``. Parts with ``lse = -inf`` carry no weight.
    The reference has no split-KV path; this is the algebra the sharded decode relies on.
    """
    lse_parts = lse_parts.float()
    m = lse_parts.max(0).values
    m_safe = torch.where(torch.isinf(m), torch.zeros_like(m), m)
    w = torch.exp(lse_parts - m_safe[None])
    den = w.sum(0)
    out = (w[..., None] * o_parts.float()).sum(0) / den.clamp_min(1e-30)[..., None]
    lse = m_safe + torch.log(den)
    return out, lse


# --------------------------------------------------------------------------------------------
# Literal restatements of the reference's torch attention code.
# --------------------------------------------------------------------------------------------


def decode_reference_grouped(
    q: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, pos: int, bound: int, scale: float
) -> torch.Tensor:
    """The reference's grouped single-token decode attention, line for line.

    ``cuda_graph_executor.py:168`` builds ``nkeep = arange[:bound] > pos``; ``:180-184`` computes
    bf16 scores with two batched matmuls, masks, takes an fp32-internal softmax cast back to the
    model dtype, and multiplies by V. ``q [nh, hd]`` (one token), ``kc, vc [max_len, nkv, hd]``.
    Returns ``ctx [1, nh * hd]`` in the input dtype.
    """
    nh, hd = q.shape
    nkv = kc.shape[1]
    groups = nh // nkv
    arange = torch.arange(kc.shape[0], device=kc.device)
    nkeep = (arange[:bound] > pos).view(1, 1, bound)
    qg = q.reshape(nkv, groups, hd)
    kt = kc[:bound].permute(1, 2, 0)
    vb = vc[:bound].permute(1, 0, 2)
    sc = (torch.matmul(qg, kt) * scale).masked_fill(nkeep, float("-inf"))
    return torch.matmul(torch.softmax(sc, -1).to(q.dtype), vb).reshape(1, nh * hd)


def prefill_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float):
    """The reference's causal prefill attention (``cuda_graph_executor.py:117-130``).

    ``q [t, nh, hd]``, ``k, v [t, nkv, hd]``; KV expanded with ``repeat_interleave`` and fed to
    ``F.scaled_dot_product_attention(is_causal=True)``. Returns ``[t, nh * hd]``.
    """
    t, nh, hd = q.shape
    groups = nh // k.shape[1]
    qh, kh, vh = q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1)
    kk = kh.repeat_interleave(groups, 0)
    vv = vh.repeat_interleave(groups, 0)
    ctx = F.scaled_dot_product_attention(qh, kk, vv, is_causal=True, scale=scale)
    return ctx.transpose(0, 1).reshape(t, nh * hd)


def verify_reference(
    q: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, vpos0: int, scale: float
) -> torch.Tensor:
    """The reference's K+1-token verify attention (``cuda_graph_executor.py:245-263``).

    Query ``i`` sits at ``vpos0 + i`` and sees every key ``j <= vpos0 + i`` of the whole static
    buffer (``keep`` mask ``:250``); the buffer is expanded ``x groups`` and fed to masked SDPA
    (``:261-263``). ``q [k1, nh, hd]``, ``kc, vc [max_len, nkv, hd]``. Returns ``[k1, nh * hd]``.
    """
    k1, nh, hd = q.shape
    max_len, nkv, _ = kc.shape
    groups = nh // nkv
    pos = vpos0 + torch.arange(k1, device=q.device)
    arange = torch.arange(max_len, device=q.device)
    keep = (arange[None, :] <= pos[:, None]).view(1, k1, max_len)
    kk = kc.permute(1, 0, 2).repeat_interleave(groups, 0)
    vv = vc.permute(1, 0, 2).repeat_interleave(groups, 0)
    ctx = F.scaled_dot_product_attention(q.transpose(0, 1), kk, vv, attn_mask=keep, scale=scale)
    return ctx.transpose(0, 1).reshape(k1, nh * hd)


def sdpa_bottom_right(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    scaling: float,
    *,
    causal: bool,
) -> torch.Tensor:
    """The HF bridge's torch attention (``transformers_flashinfer.py:153-202``), without counters.

    ``query [b, h, q, d]``, ``key/value [b, hkv, kv, d]``; GQA by ``repeat_interleave``; when
    causal and ``q < kv`` the mask is bottom-right aligned (query ``i`` sees keys
    ``<= kv - q + i``). Returns ``[b, q, h, d]``.
    """
    if query.shape[1] != key.shape[1]:
        if query.shape[1] % key.shape[1] != 0:
            raise RuntimeError(
                f"cannot expand KV heads {key.shape[1]} to query heads {query.shape[1]}"
            )
        groups = query.shape[1] // key.shape[1]
        key = key.repeat_interleave(groups, dim=1)
        value = value.repeat_interleave(groups, dim=1)
    q_len, kv_len = query.shape[-2], key.shape[-2]
    attn_mask = None
    is_causal = False
    if causal:
        if q_len == kv_len:
            is_causal = True
        else:
            offset = kv_len - q_len
            qi = torch.arange(q_len, device=query.device).unsqueeze(1)
            ki = torch.arange(kv_len, device=query.device).unsqueeze(0)
            attn_mask = torch.zeros(q_len, kv_len, dtype=query.dtype, device=query.device)
            attn_mask = attn_mask.masked_fill(~(ki <= qi + offset), float("-inf"))
    out = F.scaled_dot_product_attention(
        query, key, value, attn_mask=attn_mask, is_causal=is_causal, scale=float(scaling)
    )
    return out.transpose(1, 2).contiguous()


def default_scale(head_dim: int) -> float:
    """``hd ** -0.5`` (``cuda_graph_executor.py:44``)."""
    return head_dim ** -0.5


def log2_scale(scale: float) -> float:
    return scale * LOG2E


__all__ = [
    "attention_fp32",
    "cos_sin",
    "decode_reference_grouped",
    "default_scale",
    "inv_freq",
    "lse_merge",
    "make_attention_inputs",
    "prefill_reference",
    "rmsnorm",
    "rope",
    "sdpa_bottom_right",
    "verify_reference",
    "math",
]
