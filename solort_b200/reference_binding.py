"""Binding of the engine into SoloRT's own CUDA-graph Qwen3 runner.

``EngineAttention`` is a mixin for ``_GraphQwen3Runner`` (``src/solort/model/
cuda_graph_executor.py:31-289``). It overrides exactly the three methods the runner's capture
helpers call -- ``_prefill_forward(bound)`` (``:104-135``, called by ``_capture_prefill :137-147``),
``_decode_forward(bound)`` (``:163-190``, called by ``_capture :195-207``) and
``_verify_forward()`` (``:245-268``, called by ``verify :270-289``) -- with the same signatures
and return values, and changes only the attention inside them:

* prefill ``:124-130`` (``repeat_interleave`` + causal SDPA) -> ``torch.ops.solort_attn.gqa_prefill``;
* decode ``:168,180-184`` (mask over the bucket, grouped bf16 matmuls, softmax) ->
  ``torch.ops.solort_attn.gqa_decode`` with the bucket as ``max_kv_len`` and the live position
  read from ``pos_buf`` on the device;
* verify ``:250,261-263`` (``repeat_interleave`` of the whole buffer + masked SDPA) ->
  ``torch.ops.solort_attn.gqa_decode`` with ``q_len = K + 1`` at ``vpos0``.

Everything else -- the norms, RoPE, the KV stores at ``:122-123,178-179,259-260``, projections,
MLP, buckets, graph capture, ``decode_gpu_argmax`` and the speculative executor's ``_spec_round``
-- is the base class's own code path, unchanged. The split-KV workspace is allocated in
``__init__``, before any capture. Use::

    from solort.model import cuda_graph_executor as cge
    from solort_b200.reference_binding import install
    install(cge)   # CudaGraphQwen3Executor / SpecCudaGraphQwen3Executor now build engine runners

or ``class Runner(EngineAttention, cge._GraphQwen3Runner)``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from solort_b200 import ops

BOUND_METHODS = ("_prefill_forward", "_decode_forward", "_verify_forward")


def _rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """The reference's ``_rmsnorm`` (``cuda_graph_executor.py:25-28``): fp32 math, cast back."""
    d = x.float()
    d = d * torch.rsqrt(d.pow(2).mean(-1, keepdim=True) + eps)
    return (d * w.float()).to(x.dtype)


class EngineAttention:
    """Mixin placed before ``_GraphQwen3Runner`` in the bases; see the module docstring."""

    MAX_VERIFY_ROWS = 32  # query rows per KV head of one decode CTA: (K + 1) * groups <= 32

    def __init__(self, model, max_len: int) -> None:
        super().__init__(model, max_len)
        need = max(ops.decode_workspace_bytes(1, q, self.nh, self.nkv, self.max_len,
                                              kv_capacity=self.max_len)
                   for q in (1, max(1, self.MAX_VERIFY_ROWS // self.groups)))
        self.attn_ws = torch.empty(max(need, 256), dtype=torch.uint8, device=self.dev)

    # the reference's per-layer pieces, shared by the three overrides
    def _qkv_rope(self, x, ly, t, cos, sin):
        h = _rmsnorm(x, ly["in_ln"], self.eps)
        q, k, v = (h @ ly["wqkv"].T).split([self.q_dim, self.kv_dim, self.kv_dim], dim=-1)
        q = q.view(t, self.nh, self.hd).transpose(0, 1)
        k = k.view(t, self.nkv, self.hd).transpose(0, 1)
        v = v.view(t, self.nkv, self.hd).transpose(0, 1)
        q = self._rope(_rmsnorm(q, ly["qn"], self.eps), cos, sin)
        k = self._rope(_rmsnorm(k, ly["kn"], self.eps), cos, sin)
        return q, k, v  # [heads, t, hd]

    def _out_mlp(self, x, ctx, ly):
        x = x + ctx @ ly["wo"].T
        h2 = _rmsnorm(x, ly["post_ln"], self.eps)
        gate, up = (h2 @ ly["wgu"].T).split([self.inter, self.inter], dim=-1)
        return x + (F.silu(gate) * up) @ ly["wd"].T

    def _prefill_forward(self, bound: int) -> torch.Tensor:
        t = bound
        cos, sin = self._cos_sin(torch.arange(t, device=self.dev))
        x = self.embed[self.pre_tok[:bound]].to(self.dt)
        for li, ly in enumerate(self.layers):
            q, k, v = self._qkv_rope(x, ly, t, cos, sin)
            self.kc[li, :t] = k.transpose(0, 1)
            self.vc[li, :t] = v.transpose(0, 1)
            ctx = torch.empty(t, self.nh, self.hd, dtype=self.dt, device=self.dev)
            torch.ops.solort_attn.gqa_prefill(q.transpose(0, 1), self.kc[li, :t], self.vc[li, :t],
                                              ctx, True, self.scale)
            x = self._out_mlp(x, ctx.view(t, self.q_dim), ly)
        return _rmsnorm(x, self.final_norm, self.eps)

    def _decode_forward(self, bound: int) -> torch.Tensor:
        cos, sin = self._cos_sin(self.pos_buf)
        x = self.embed[self.tok_buf].to(self.dt)
        for li, ly in enumerate(self.layers):
            q, k, v = self._qkv_rope(x, ly, 1, cos, sin)
            self.kc[li].index_copy_(0, self.pos_buf, k.transpose(0, 1))
            self.vc[li].index_copy_(0, self.pos_buf, v.transpose(0, 1))
            ctx = torch.empty(1, 1, self.nh, self.hd, dtype=self.dt, device=self.dev)
            torch.ops.solort_attn.gqa_decode(q.transpose(0, 1)[None], self.kc[li], self.vc[li],
                                             self.pos_buf, ctx, self.attn_ws, "NHD", self.scale,
                                             bound, None, 0, False)
            x = self._out_mlp(x, ctx.view(1, self.q_dim), ly)
        x = _rmsnorm(x, self.final_norm, self.eps)
        return (x @ self.lm_head.T).float()

    def _verify_forward(self) -> torch.Tensor:
        k1 = self.vtok.shape[0]
        if k1 * self.groups > self.MAX_VERIFY_ROWS:
            raise RuntimeError(f"verify supports at most {self.MAX_VERIFY_ROWS // self.groups} "
                               "tokens per round")
        pos = self.vpos0 + torch.arange(k1, device=self.dev)
        cos, sin = self._cos_sin(pos)
        x = self.embed[self.vtok].to(self.dt)
        for li, ly in enumerate(self.layers):
            q, k, v = self._qkv_rope(x, ly, k1, cos, sin)
            self.kc[li].index_copy_(0, pos, k.transpose(0, 1))
            self.vc[li].index_copy_(0, pos, v.transpose(0, 1))
            ctx = torch.empty(1, k1, self.nh, self.hd, dtype=self.dt, device=self.dev)
            torch.ops.solort_attn.gqa_decode(q.transpose(0, 1)[None], self.kc[li], self.vc[li],
                                             self.vpos0, ctx, self.attn_ws, "NHD", self.scale,
                                             self.max_len, None, 0, False)
            x = self._out_mlp(x, ctx.view(k1, self.q_dim), ly)
        return (_rmsnorm(x, self.final_norm, self.eps) @ self.lm_head.T).float()


def engine_runner_class(base: type) -> type:
    """``base`` (the reference's ``_GraphQwen3Runner`` or a class of the same shape) with the
    engine's attention mixed in."""
    return type("Engine" + base.__name__.lstrip("_"), (EngineAttention, base), {})


def install(module) -> type:
    """Point ``module._GraphQwen3Runner`` (the reference's ``cuda_graph_executor`` module) at the
    engine-backed subclass, so the executors' constructors (``cuda_graph_executor.py:310,424``)
    build it. Idempotent; returns the class in use."""
    base = module._GraphQwen3Runner
    if issubclass(base, EngineAttention):
        return base
    module._GraphQwen3Runner = engine_runner_class(base)
    return module._GraphQwen3Runner
