"""Restatement of the reference's CUDA-graph Qwen3 runner (test infrastructure only).

``ReferenceQwen3Runner`` follows ``_GraphQwen3Runner`` (``src/solort/model/cuda_graph_executor.py:
31-289``) method for method -- fused QKV / gate-up weights (``:52-63``), QK-RMSNorm + RoPE
(``:25-28, 95-102``), static KV ``[L, max_len, nkv, hd]`` (``:67-69``), the static buffers
``tok_buf / pos_buf / pre_tok / vtok / vpos0`` (``:70-71, 83-93``), ``_prefill_forward(bound)``
(``:104-135``), ``_decode_forward(bound)`` (``:163-190``), ``_verify_forward()`` (``:245-268``)
and the public ``prefill / decode / decode_argmax / decode_gpu / decode_gpu_argmax / verify``
(``:149-161, 209-243, 270-289``) -- with the reference's own attention at the three sites
(``:124-130`` prefill SDPA with ``repeat_interleave``, ``:168, 180-184`` grouped bf16 decode,
``:250, 261-263`` masked verify SDPA). With ``graphs=True`` (CUDA, literal attention) it captures
and replays CUDA graphs exactly as the reference does (``:137-147, 195-214, 270-289``); otherwise
the same forwards run eagerly. ``attention="fp32"`` swaps in the parity oracle (fp32 softmax over
the same bf16 inputs) at the three sites, everything else unchanged.

Because the method structure is the reference's, the engine's binding mixin
(``solort_b200.reference_binding.EngineAttention``) binds to this class the same way it binds to
the reference's, which is how the GPU tests run the binding where the reference package is not
installed. ``reference_spec_round`` restates ``SpecCudaGraphQwen3Executor._spec_round``
(``:463-482``). Pinned by ``tests/golden/runner_attention.npz`` (the reference runner's own
attention tensors and token stream on a tiny model).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from oracle.attention import attention_fp32, rmsnorm


class ReferenceQwen3Runner:
    """``attention="reference"`` (default) runs the reference's literal torch attention;
    ``attention="fp32"`` swaps in the parity oracle at the same three sites."""

    def __init__(self, model, max_len: int, attention: str = "reference", graphs: bool = False):
        if attention not in ("reference", "fp32"):
            raise ValueError(attention)
        self.attention = attention
        c = model.config
        self.dev = next(model.parameters()).device
        self.graphs = bool(graphs) and self.dev.type == "cuda"
        if self.graphs and attention != "reference":
            raise ValueError("graph capture needs the literal attention (device-side positions)")
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
        self.tok_buf = torch.zeros(1, dtype=torch.long, device=self.dev)
        self.pos_buf = torch.zeros(1, dtype=torch.long, device=self.dev)
        self.arange = torch.arange(self.max_len, device=self.dev)
        self.buckets = sorted({b for b in (128, 256, 512, 1024, 2048, 4096) if b < self.max_len}
                              | {self.max_len})
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self._logits: dict[int, torch.Tensor] = {}
        self._tok: dict[int, torch.Tensor] = {}
        self.pre_buckets = sorted({b for b in (16, 32, 64, 128, 256, 512, 1024) if b <= self.max_len})
        self.pre_tok = torch.zeros(self.max_len, dtype=torch.long, device=self.dev)
        self._pre_graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self._pre_hidden: dict[int, torch.Tensor] = {}
        self.verify_graph = None
        self.vtok: torch.Tensor | None = None
        self.vpos0: torch.Tensor | None = None
        self._vlogits: torch.Tensor | None = None

    # ---- shared pieces (:95-102) ----
    def _cos_sin(self, positions):
        f = positions[:, None].float() * self.inv_freq[None, :]
        emb = torch.cat([f, f], -1)
        return emb.cos().to(self.dt), emb.sin().to(self.dt)

    def _rope(self, x, cos, sin):
        d = x.shape[-1] // 2
        return x * cos + torch.cat([-x[..., d:], x[..., :d]], -1) * sin

    def _qkv(self, x, ly, t, cos, sin):
        h = rmsnorm(x, ly["in_ln"], self.eps)
        q, k, v = (h @ ly["wqkv"].T).split([self.q_dim, self.kv_dim, self.kv_dim], dim=-1)
        q = q.view(t, self.nh, self.hd).transpose(0, 1)
        k = k.view(t, self.nkv, self.hd).transpose(0, 1)
        v = v.view(t, self.nkv, self.hd).transpose(0, 1)
        q = self._rope(rmsnorm(q, ly["qn"], self.eps), cos, sin)
        k = self._rope(rmsnorm(k, ly["kn"], self.eps), cos, sin)
        return q, k, v

    def _mlp(self, x, ly):
        h2 = rmsnorm(x, ly["post_ln"], self.eps)
        gate, up = (h2 @ ly["wgu"].T).split([self.inter, self.inter], dim=-1)
        return x + (F.silu(gate) * up) @ ly["wd"].T

    # ---- prefill (:104-161) ----
    def _prefill_forward(self, bound: int) -> torch.Tensor:
        t = bound
        cos, sin = self._cos_sin(torch.arange(t, device=self.dev))
        x = self.embed[self.pre_tok[:bound]].to(self.dt)
        for li, ly in enumerate(self.layers):
            q, k, v = self._qkv(x, ly, t, cos, sin)
            self.kc[li, :t] = k.transpose(0, 1)
            self.vc[li, :t] = v.transpose(0, 1)
            if self.attention == "fp32":
                o, _ = attention_fp32(q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1),
                                      self.scale, 0)
                ctx = o.to(self.dt).reshape(t, self.q_dim)
            else:
                kk = k.repeat_interleave(self.groups, 0)
                vv = v.repeat_interleave(self.groups, 0)
                ctx = (F.scaled_dot_product_attention(q, kk, vv, is_causal=True, scale=self.scale)
                       .transpose(0, 1).reshape(t, self.q_dim))
            x = x + ctx @ ly["wo"].T
            x = self._mlp(x, ly)
        return rmsnorm(x, self.final_norm, self.eps)

    def _capture_prefill(self, bound: int) -> None:
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(2):
                hid = self._prefill_forward(bound)
        torch.cuda.current_stream().wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            hid = self._prefill_forward(bound)
        self._pre_graphs[bound], self._pre_hidden[bound] = graph, hid

    def prefill(self, ids: torch.Tensor) -> torch.Tensor:
        """Pad to the prefill bucket, causal forward, logits of the last real position."""
        plen = int(ids.shape[0])
        bound = next(b for b in self.pre_buckets if b >= plen)
        self.pre_tok[:plen].copy_(ids)
        self.pre_tok[plen:bound].zero_()
        if self.graphs:
            if bound not in self._pre_graphs:
                self._capture_prefill(bound)
            self._pre_graphs[bound].replay()
            hid = self._pre_hidden[bound]
        else:
            hid = self._prefill_forward(bound)
        return (hid[plen - 1: plen] @ self.lm_head.T).float()

    # ---- decode (:163-243) ----
    def _decode_forward(self, bound: int) -> torch.Tensor:
        cos, sin = self._cos_sin(self.pos_buf)
        x = self.embed[self.tok_buf].to(self.dt)
        nkeep = (self.arange[:bound] > self.pos_buf).view(1, 1, bound)
        for li, ly in enumerate(self.layers):
            q, k, v = self._qkv(x, ly, 1, cos, sin)
            self.kc[li].index_copy_(0, self.pos_buf, k.transpose(0, 1))
            self.vc[li].index_copy_(0, self.pos_buf, v.transpose(0, 1))
            if self.attention == "fp32":
                o, _ = attention_fp32(q.transpose(0, 1), self.kc[li, :bound], self.vc[li, :bound],
                                      self.scale, int(self.pos_buf.item()))
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

    def _bucket_for(self, pos: int) -> int:
        return next(b for b in self.buckets if b > pos)

    def _capture(self, bound: int) -> None:
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(3):
                lg = self._decode_forward(bound)
                tk = lg.argmax(-1)
        torch.cuda.current_stream().wait_stream(stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            lg = self._decode_forward(bound)
            tk = lg.argmax(-1)
        self._graphs[bound], self._logits[bound], self._tok[bound] = graph, lg, tk

    def _run_decode(self, pos: int):
        """The reference's ``_replay`` (``:209-214``), or the eager forward; returns
        ``(logits, argmax)``."""
        bound = self._bucket_for(pos)
        if self.graphs:
            if bound not in self._graphs:
                self._capture(bound)
            self._graphs[bound].replay()
            return self._logits[bound], self._tok[bound]
        lg = self._decode_forward(bound)
        return lg, lg.argmax(-1)

    def decode(self, token: int, pos: int) -> torch.Tensor:
        self.tok_buf.fill_(int(token))
        self.pos_buf.fill_(int(pos))
        return self._run_decode(pos)[0]

    def decode_argmax(self, token: int, pos: int) -> int:
        self.tok_buf.fill_(int(token))
        self.pos_buf.fill_(int(pos))
        return int(self._run_decode(pos)[1].item())

    def decode_gpu(self, tok_t: torch.Tensor, pos: int) -> torch.Tensor:
        self.tok_buf.copy_(tok_t.view(1))
        self.pos_buf.fill_(int(pos))
        return self._run_decode(pos)[0].argmax(-1)

    def decode_gpu_argmax(self, tok_t: torch.Tensor, pos: int) -> torch.Tensor:
        self.tok_buf.copy_(tok_t.view(1))
        self.pos_buf.fill_(int(pos))
        return self._run_decode(pos)[1].clone()

    # ---- verify (:245-289) ----
    def _verify_forward(self) -> torch.Tensor:
        k1 = self.vtok.shape[0]
        pos = self.vpos0 + torch.arange(k1, device=self.dev)
        cos, sin = self._cos_sin(pos)
        x = self.embed[self.vtok].to(self.dt)
        keep = (self.arange[None, :] <= pos[:, None]).view(1, k1, self.max_len)
        for li, ly in enumerate(self.layers):
            q, k, v = self._qkv(x, ly, k1, cos, sin)
            self.kc[li].index_copy_(0, pos, k.transpose(0, 1))
            self.vc[li].index_copy_(0, pos, v.transpose(0, 1))
            if self.attention == "fp32":
                o, _ = attention_fp32(q.transpose(0, 1), self.kc[li], self.vc[li], self.scale,
                                      int(self.vpos0.item()))
                ctx = o.to(self.dt).reshape(k1, self.q_dim)
            else:
                kk = self.kc[li].permute(1, 0, 2).repeat_interleave(self.groups, 0)
                vv = self.vc[li].permute(1, 0, 2).repeat_interleave(self.groups, 0)
                ctx = (F.scaled_dot_product_attention(q, kk, vv, attn_mask=keep, scale=self.scale)
                       .transpose(0, 1).reshape(k1, self.q_dim))
            x = x + ctx @ ly["wo"].T
            x = self._mlp(x, ly)
        return (rmsnorm(x, self.final_norm, self.eps) @ self.lm_head.T).float()

    def verify(self, tok_t: torch.Tensor, pos_start: int) -> torch.Tensor:
        """Score ``K + 1`` tokens at ``pos_start ..``; logits ``[K + 1, vocab]``."""
        tok_t = tok_t.to(self.dev)
        if self.vtok is None or self.vtok.shape[0] != tok_t.shape[0]:
            self.vtok = torch.zeros(tok_t.shape[0], dtype=torch.long, device=self.dev)
            self.vpos0 = torch.zeros(1, dtype=torch.long, device=self.dev)
            self.verify_graph = None
        self.vtok.copy_(tok_t)
        self.vpos0.fill_(int(pos_start))
        if not self.graphs:
            return self._verify_forward()
        if self.verify_graph is None:
            stream = torch.cuda.Stream()
            stream.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(stream):
                for _ in range(3):
                    self._vlogits = self._verify_forward()
            torch.cuda.current_stream().wait_stream(stream)
            self.verify_graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.verify_graph):
                self._vlogits = self._verify_forward()
            self.vtok.copy_(tok_t)
            self.vpos0.fill_(int(pos_start))
        self.verify_graph.replay()
        return self._vlogits

    def greedy(self, prompt: torch.Tensor, steps: int) -> list[int]:
        """Prefill, then ``steps`` greedy decode tokens (the executor's greedy loop,
        ``cuda_graph_executor.py:332-380``)."""
        toks = [int(self.prefill(prompt).argmax(-1).item())]
        pos = int(prompt.shape[0])
        for _ in range(steps):
            toks.append(self.decode_argmax(toks[-1], pos))
            pos += 1
        return toks


def reference_spec_round(target, draft, last_token: int, n: int, k: int) -> list[int]:
    """``SpecCudaGraphQwen3Executor._spec_round`` (``cuda_graph_executor.py:463-482``) on two
    runners with the reference's surface: the draft proposes ``k`` tokens by GPU-resident
    ``decode_gpu`` calls from position ``n``, the target verifies ``[last_token, drafts]`` at
    ``n .. n + k`` in one call, ``a`` = the length of the prefix of drafts equal to the target's
    argmax (``cumprod`` of the matches), and the round emits the accepted drafts plus the
    target's token after them; when all ``k`` are accepted the draft also decodes its last
    proposal at ``n + k`` so its KV stays continuous."""
    with torch.no_grad():
        t_gpu = torch.tensor([int(last_token)], dtype=torch.long, device=target.dev)
        drafts = []
        cur, pos = t_gpu, n
        for _ in range(k):
            cur = draft.decode_gpu(cur, pos)
            drafts.append(cur)
            pos += 1
        draft_vec = torch.cat(drafts)
        tg = target.verify(torch.cat([t_gpu, draft_vec]), n).argmax(-1)
        a = int((tg[:k] == draft_vec).cumprod(0).sum().item())
        if a == k:
            out = torch.cat([draft_vec, tg[k:k + 1]]).tolist()
            draft.decode_gpu(draft_vec[k - 1:k], n + k)
        else:
            out = torch.cat([draft_vec[:a], tg[a:a + 1]]).tolist()
    return out


def reference_speculative_greedy(target, draft, prompt: torch.Tensor, steps: int,
                                 k: int = 4) -> tuple[list[int], list[int]]:
    """The speculative executor's greedy loop (``cuda_graph_executor.py:426-461``): both runners
    prefill, the target's prefill argmax is the first token, then ``reference_spec_round`` until
    ``steps`` more tokens exist; near ``max_len`` the target decodes single tokens. Returns the
    tokens (``steps + 1``) and each round's accepted draft count."""
    toks = [int(target.prefill(prompt).argmax(-1).item())]
    draft.prefill(prompt)
    pos = int(prompt.shape[0])
    accepted = []
    while len(toks) < steps + 1:
        if pos + k + 2 >= min(target.max_len, draft.max_len):
            toks.append(target.decode_argmax(toks[-1], pos))
            pos += 1
            continue
        new = reference_spec_round(target, draft, toks[-1], pos, k)
        accepted.append(len(new) - 1)
        toks += new
        pos += len(new)
    return toks[:steps + 1], accepted
