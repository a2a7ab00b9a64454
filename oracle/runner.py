"""Eager restatement of the reference's CUDA-graph Qwen3 runner (test infrastructure only).

Follows ``_GraphQwen3Runner`` (``src/solort/model/cuda_graph_executor.py:31-289``) step by step
-- fused QKV / gate-up weights (``:52-63``), QK-RMSNorm + RoPE (``:25-28, 95-102``), static KV
``[L, max_len, nkv, hd]`` (``:67-69``), the reference's own attention at the three sites
(``:124-130`` prefill SDPA with ``repeat_interleave``, ``:168, 180-184`` grouped bf16 decode,
``:250, 261-263`` masked verify SDPA) -- without graph capture. It is the checker for the
engine's runner: same weights in, greedy token streams compared. Pinned by
``tests/golden/runner_attention.npz`` (the reference runner's own token stream on a tiny model).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle.attention import attention_fp32, rmsnorm


class ReferenceQwen3Runner:
    """``attention="reference"`` (default) runs the reference's literal torch attention;
    ``attention="fp32"`` swaps in the parity oracle (fp32 softmax over the same bf16 inputs) at the
    same three sites, everything else unchanged."""

    def __init__(self, model, max_len: int, attention: str = "reference"):
        if attention not in ("reference", "fp32"):
            raise ValueError(attention)
        self.attention = attention
        c = model.config
        self.dev = next(model.parameters()).device
        self.dt = model.dtype
        self.L = int(c.num_hidden_layers)
        self.nh = int(c.num_attention_heads)
        self.nkv = int(c.num_key_value_heads)
        self.hd = int(getattr(c, "head_dim", c.hidden_size // c.num_attention_heads))
        self.groups = self.nh // self.nkv
        self.eps = float(c.rms_norm_eps)
        self.scale = self.hd ** -0.5
        self.max_len = int(max_len)
        self.embed = model.model.embed_tokens.weight
        self.final_norm = model.model.norm.weight
        self.lm_head = model.lm_head.weight
        self.q_dim, self.kv_dim = self.nh * self.hd, self.nkv * self.hd
        self.layers = []
        for i in range(self.L):
            a, mlp = model.model.layers[i].self_attn, model.model.layers[i].mlp
            self.inter = mlp.gate_proj.weight.shape[0]
            self.layers.append({
                "in_ln": model.model.layers[i].input_layernorm.weight,
                "post_ln": model.model.layers[i].post_attention_layernorm.weight,
                "wqkv": torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0).contiguous(),
                "wo": a.o_proj.weight, "qn": a.q_norm.weight, "kn": a.k_norm.weight,
                "wgu": torch.cat([mlp.gate_proj.weight, mlp.up_proj.weight], 0).contiguous(),
                "wd": mlp.down_proj.weight,
            })
        theta = float(getattr(c, "rope_theta", None) or c.rope_parameters["rope_theta"])
        self.inv_freq = 1.0 / (theta ** (torch.arange(0, self.hd, 2, device=self.dev).float() / self.hd))
        shape = (self.L, self.max_len, self.nkv, self.hd)
        self.kc = torch.zeros(shape, device=self.dev, dtype=self.dt)
        self.vc = torch.zeros(shape, device=self.dev, dtype=self.dt)
        self.arange = torch.arange(self.max_len, device=self.dev)
        self.buckets = sorted({b for b in (128, 256, 512, 1024, 2048, 4096) if b < self.max_len}
                              | {self.max_len})
        self.pre_buckets = sorted({b for b in (16, 32, 64, 128, 256, 512, 1024) if b <= self.max_len})

    def _cos_sin(self, positions):
        f = positions[:, None].float() * self.inv_freq[None, :]
        emb = torch.cat([f, f], -1)
        return emb.cos().to(self.dt), emb.sin().to(self.dt)

    @staticmethod
    def _rope(x, cos, sin):
        d = x.shape[-1] // 2
        return x * cos + torch.cat([-x[..., d:], x[..., :d]], -1) * sin

    def _mlp(self, x, ly):
        h2 = rmsnorm(x, ly["post_ln"], self.eps)
        gate, up = (h2 @ ly["wgu"].T).split([self.inter, self.inter], dim=-1)
        return x + (F.silu(gate) * up) @ ly["wd"].T

    def prefill(self, ids: torch.Tensor) -> torch.Tensor:
        """``cuda_graph_executor.py:104-135, 149-161``: pad to the prefill bucket, causal forward,
        logits of the last real position."""
        plen = int(ids.shape[0])
        t = next(b for b in self.pre_buckets if b >= plen)
        tok = torch.zeros(t, dtype=torch.long, device=self.dev)
        tok[:plen] = ids
        cos, sin = self._cos_sin(torch.arange(t, device=self.dev))
        x = self.embed[tok].to(self.dt)
        for li, ly in enumerate(self.layers):
            h = rmsnorm(x, ly["in_ln"], self.eps)
            q, k, v = (h @ ly["wqkv"].T).split([self.q_dim, self.kv_dim, self.kv_dim], dim=-1)
            q = q.view(t, self.nh, self.hd).transpose(0, 1)
            k = k.view(t, self.nkv, self.hd).transpose(0, 1)
            v = v.view(t, self.nkv, self.hd).transpose(0, 1)
            q = self._rope(rmsnorm(q, ly["qn"], self.eps), cos, sin)
            k = self._rope(rmsnorm(k, ly["kn"], self.eps), cos, sin)
            self.kc[li, :t] = k.transpose(0, 1)
            self.vc[li, :t] = v.transpose(0, 1)
            if self.attention == "fp32":
                o, _ = attention_fp32(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1),
                                      self.scale, 0)
                ctx = o.to(self.dt).transpose(0, 1)
            else:
                kk = k.repeat_interleave(self.groups, 0)
                vv = v.repeat_interleave(self.groups, 0)
                ctx = F.scaled_dot_product_attention(q, kk, vv, is_causal=True, scale=self.scale)
            x = x + ctx.transpose(0, 1).reshape(t, self.q_dim) @ ly["wo"].T
            x = self._mlp(x, ly)
        hid = rmsnorm(x, self.final_norm, self.eps)
        return (hid[plen - 1: plen] @ self.lm_head.T).float()

    def decode(self, token: int, pos: int) -> torch.Tensor:
        """``cuda_graph_executor.py:163-193``: one token at ``pos`` over bucket ``bound``."""
        bound = next(b for b in self.buckets if b > pos)
        pos_t = torch.tensor([pos], dtype=torch.long, device=self.dev)
        cos, sin = self._cos_sin(pos_t)
        x = self.embed[torch.tensor([token], device=self.dev)].to(self.dt)
        nkeep = (self.arange[:bound] > pos_t).view(1, 1, bound)
        for li, ly in enumerate(self.layers):
            h = rmsnorm(x, ly["in_ln"], self.eps)
            q, k, v = (h @ ly["wqkv"].T).split([self.q_dim, self.kv_dim, self.kv_dim], dim=-1)
            q = q.view(1, self.nh, self.hd).transpose(0, 1)
            k = k.view(1, self.nkv, self.hd).transpose(0, 1)
            v = v.view(1, self.nkv, self.hd).transpose(0, 1)
            q = self._rope(rmsnorm(q, ly["qn"], self.eps), cos, sin)
            k = self._rope(rmsnorm(k, ly["kn"], self.eps), cos, sin)
            self.kc[li].index_copy_(0, pos_t, k.transpose(0, 1))
            self.vc[li].index_copy_(0, pos_t, v.transpose(0, 1))
            if self.attention == "fp32":
                o, _ = attention_fp32(q.transpose(0, 1), self.kc[li, :bound], self.vc[li, :bound],
                                      self.scale, pos)
                ctx = o.to(self.dt).reshape(1, self.q_dim)
            else:
                qg = q.reshape(self.nkv, self.groups, self.hd)
                kt = self.kc[li, :bound].permute(1, 2, 0)
                vb = self.vc[li, :bound].permute(1, 0, 2)
                sc = (torch.matmul(qg, kt) * self.scale).masked_fill(nkeep, float("-inf"))
                ctx = torch.matmul(torch.softmax(sc, -1).to(self.dt), vb).reshape(1, self.q_dim)
            x = x + ctx @ ly["wo"].T
            x = self._mlp(x, ly)
        x = rmsnorm(x, self.final_norm, self.eps)
        return (x @ self.lm_head.T).float()

    def verify(self, tokens: torch.Tensor, pos_start: int) -> torch.Tensor:
        """``cuda_graph_executor.py:245-268``: K+1 tokens at ``pos_start..``, logits [K+1, V]."""
        k1 = int(tokens.shape[0])
        pos = pos_start + torch.arange(k1, device=self.dev)
        cos, sin = self._cos_sin(pos)
        x = self.embed[tokens.to(self.dev)].to(self.dt)
        keep = (self.arange[None, :] <= pos[:, None]).view(1, k1, self.max_len)
        for li, ly in enumerate(self.layers):
            h = rmsnorm(x, ly["in_ln"], self.eps)
            q, k, v = (h @ ly["wqkv"].T).split([self.q_dim, self.kv_dim, self.kv_dim], dim=-1)
            q = q.view(k1, self.nh, self.hd).transpose(0, 1)
            k = k.view(k1, self.nkv, self.hd).transpose(0, 1)
            v = v.view(k1, self.nkv, self.hd).transpose(0, 1)
            q = self._rope(rmsnorm(q, ly["qn"], self.eps), cos, sin)
            k = self._rope(rmsnorm(k, ly["kn"], self.eps), cos, sin)
            self.kc[li].index_copy_(0, pos, k.transpose(0, 1))
            self.vc[li].index_copy_(0, pos, v.transpose(0, 1))
            if self.attention == "fp32":
                o, _ = attention_fp32(q.transpose(0, 1), self.kc[li], self.vc[li], self.scale,
                                      pos_start)
                ctx = o.to(self.dt).transpose(0, 1)
            else:
                kk = self.kc[li].permute(1, 0, 2).repeat_interleave(self.groups, 0)
                vv = self.vc[li].permute(1, 0, 2).repeat_interleave(self.groups, 0)
                ctx = F.scaled_dot_product_attention(q, kk, vv, attn_mask=keep, scale=self.scale)
            x = x + ctx.transpose(0, 1).reshape(k1, self.q_dim) @ ly["wo"].T
            x = self._mlp(x, ly)
        return (rmsnorm(x, self.final_norm, self.eps) @ self.lm_head.T).float()

    def greedy(self, prompt: torch.Tensor, steps: int) -> list[int]:
        """Prefill, then ``steps`` greedy decode tokens (the executor's greedy loop,
        ``cuda_graph_executor.py:332-380``)."""
        toks = [int(self.prefill(prompt).argmax(-1).item())]
        pos = int(prompt.shape[0])
        for _ in range(steps):
            toks.append(int(self.decode(toks[-1], pos).argmax(-1).item()))
            pos += 1
        return toks
