"""CUDA-graph Qwen3 runner whose three attention sites run on the engine.

Same public surface and control flow as the reference's ``_GraphQwen3Runner``
(``src/solort/model/cuda_graph_executor.py:31-289``), so ``CudaGraphQwen3Executor`` and
``SpecCudaGraphQwen3Executor`` (``:292-482``) can use it unchanged: ``prefill``, ``decode``,
``decode_argmax``, ``decode_gpu``, ``decode_gpu_argmax``, ``verify``; bucketed decode graphs
routed by position (``:73-77, 192-214``), bucketed prefill graphs (``:83-85, 137-161``), one
lazily captured verify graph (``:270-289``); static KV ``[L, max_len, nkv, hd]`` (``:67-69``).

What changes is the attention at the three inline sites:
* prefill (``:124-130``, ``repeat_interleave`` + causal SDPA) -> ``ops.gqa_prefill`` (tcgen05);
* decode (``:168, 180-184``, grouped bf16 matmuls over the bucket) -> ``ops.gqa_decode`` reading
  the live position from ``pos_buf`` on the device (split-KV, fp32 softmax);
* verify (``:250, 261-263``, ``repeat_interleave`` of the whole buffer + masked SDPA) ->
  ``ops.gqa_decode`` with ``q_len = K + 1`` (per-row causal limit, no expansion).
With ``prologue="fused"`` (the default) the per-head QK-RMSNorm, RoPE and KV append of each
layer (``:176-179, 120-123, 257-260``) run as one ``ops.qk_norm_rope_append`` launch reading the
model's bf16 cos/sin tables; with ``glue="fused"`` (the default) each residual add and the RMSNorm
after it run as one ``ops.add_rmsnorm`` launch and F.silu(gate) * up as one ``ops.silu_mul``;
``"torch"`` keeps the reference's torch ops at either place. With ``proj="gemv"`` (the default)
the decode step's projections and lm_head (one token row, where a weight stream beats cuBLAS) run
as ``ops.gemv`` launches that also carry the layer glue: each residual add + RMSNorm runs in the
staging of the projection after it (qkv, gate_up, lm_head) and SiLU(gate) * up in the down
projection's, so a decoder layer is six launches (qkv, prologue, attention, o, gate_up, down;
plus the split-KV merge when the attention splits). The residual stream alternates between two
buffers because the fused norm writes x + delta while other CTAs still read x. Verify's K + 1 rows,
prefill's projections and the argmax use the reference's torch calls.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from solort_b200 import ops


def _rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    d = x.float()
    d = d * torch.rsqrt(d.pow(2).mean(-1, keepdim=True) + eps)
    return (d * w.float()).to(x.dtype)


class GraphQwen3Runner:
    MAX_VERIFY_TOKENS = 8
    GEMV_MAX_ROWS = 1  # weight-streaming projections for one token row; cuBLAS from two rows on

    def __init__(self, model, max_len: int, prologue: str = "fused", glue: str = "fused",
                 proj: str = "gemv", single_decode_graph: bool = False) -> None:
        if prologue not in ("fused", "torch") or glue not in ("fused", "torch") or \
                proj not in ("gemv", "torch"):
            raise ValueError((prologue, glue, proj))
        self.prologue, self.glue, self.proj = prologue, glue, proj
        c = model.config
        self.dev = next(model.parameters()).device
        if self.dev.type != "cuda":
            raise RuntimeError("GraphQwen3Runner requires CUDA")
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
        # the reference's bf16 cos/sin rows for every position, read by the fused prologue
        self.cos_tab, self.sin_tab = self._cos_sin(torch.arange(int(max_len), device=self.dev))
        self.zero_pos = torch.zeros(1, dtype=torch.long, device=self.dev)
        shape = (self.L, self.max_len, self.nkv, self.hd)
        self.kc = torch.zeros(shape, device=self.dev, dtype=self.dt)
        self.vc = torch.zeros(shape, device=self.dev, dtype=self.dt)
        self.tok_buf = torch.zeros(1, dtype=torch.long, device=self.dev)
        self.pos_buf = torch.zeros(1, dtype=torch.long, device=self.dev)
        # The engine reads the live length from pos_buf, so one graph sized for max_len serves
        # every position (single_decode_graph); the buckets remain the default because a bound far
        # above the live length makes most splits of the decode grid empty.
        self.buckets = [self.max_len] if single_decode_graph else sorted(
            {b for b in (128, 256, 512, 1024, 2048, 4096) if b < self.max_len} | {self.max_len})
        self._graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self._logits: dict[int, torch.Tensor] = {}
        self._tok: dict[int, torch.Tensor] = {}
        self.pre_buckets = sorted({b for b in (16, 32, 64, 128, 256, 512, 1024) if b <= self.max_len})
        self.pre_tok = torch.zeros(self.max_len, dtype=torch.long, device=self.dev)
        self._pre_graphs: dict[int, torch.cuda.CUDAGraph] = {}
        self._pre_hidden: dict[int, torch.Tensor] = {}
        self.verify_graph: torch.cuda.CUDAGraph | None = None
        self.vtok: torch.Tensor | None = None
        self.vpos0: torch.Tensor | None = None
        self._vlogits: torch.Tensor | None = None
        # one split-KV workspace, sized for the largest decode / verify call, allocated before any
        # graph capture and shared by every layer (calls are stream-ordered)
        nbytes = max(
            ops.decode_workspace_bytes(1, q, self.nh, self.nkv, self.max_len, kv_capacity=self.max_len)
            for q in (1, min(self.MAX_VERIFY_TOKENS, 32 // self.groups))
        )
        self.attn_ws = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=self.dev)

    # ---- shared pieces (same math as the reference) ----
    def _cos_sin(self, positions: torch.Tensor):
        f = positions[:, None].float() * self.inv_freq[None, :]
        emb = torch.cat([f, f], -1)
        return emb.cos().to(self.dt), emb.sin().to(self.dt)

    @staticmethod
    def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        d = x.shape[-1] // 2
        return x * cos + torch.cat([-x[..., d:], x[..., :d]], -1) * sin

    def _qkv(self, h: torch.Tensor, ly: dict, t: int, cos, sin):
        q, k, v = (h @ ly["wqkv"].T).split([self.q_dim, self.kv_dim, self.kv_dim], dim=-1)
        q = q.view(t, self.nh, self.hd).transpose(0, 1)
        k = k.view(t, self.nkv, self.hd).transpose(0, 1)
        v = v.view(t, self.nkv, self.hd).transpose(0, 1)
        q = self._rope(_rmsnorm(q, ly["qn"], self.eps), cos, sin)
        k = self._rope(_rmsnorm(k, ly["kn"], self.eps), cos, sin)
        return q, k, v  # [heads, t, hd]

    def _mm(self, a: torch.Tensor, w: torch.Tensor, silu_gate_up: bool = False) -> torch.Tensor:
        """``act(a) @ w.T``: the weight-streaming kernel for the decode / verify step's few rows
        (``proj="gemv"``), the torch matmul otherwise (prefill's GEMM-shaped calls)."""
        if self.proj == "gemv" and a.shape[0] <= self.GEMV_MAX_ROWS:
            return ops.gemv(a, w, silu_gate_up=silu_gate_up)
        if silu_gate_up:
            a = ops.silu_mul(a) if self.glue == "fused" else self._silu_up(a)
        return a @ w.T

    def _silu_up(self, gu: torch.Tensor) -> torch.Tensor:
        gate, up = gu.split([self.inter, self.inter], dim=-1)
        return F.silu(gate) * up

    def _attn_inputs(self, h: torch.Tensor, ly: dict, li: int, t: int, pos_t: torch.Tensor,
                     pos_rows: torch.Tensor, cos, sin) -> torch.Tensor:
        """Queries ``[t, nh, hd]`` of layer ``li`` from its normed input ``h`` for tokens at
        ``pos_t[0] ..``, with the tokens' K / V appended to ``kc[li]``/``vc[li]`` (``pos_rows``: the
        same positions as a vector)."""
        if self.prologue == "fused":
            qkv = self._mm(h, ly["wqkv"])
            return ops.qk_norm_rope_append(qkv, ly["qn"], ly["kn"], self.eps, self.cos_tab,
                                           self.sin_tab, pos_t, self.kc[li], self.vc[li],
                                           num_qo_heads=self.nh, num_kv_heads=self.nkv)
        q, k, v = self._qkv(h, ly, t, cos, sin)
        self.kc[li].index_copy_(0, pos_rows, k.transpose(0, 1))
        self.vc[li].index_copy_(0, pos_rows, v.transpose(0, 1))
        return q.transpose(0, 1)

    def _mlp(self, x: torch.Tensor, ly: dict) -> torch.Tensor:
        h2 = _rmsnorm(x, ly["post_ln"], self.eps)
        gate, up = (h2 @ ly["wgu"].T).split([self.inter, self.inter], dim=-1)
        return x + (F.silu(gate) * up) @ ly["wd"].T

    def _layer_stack(self, x: torch.Tensor, t: int, pos_t: torch.Tensor, pos_rows: torch.Tensor,
                     cos, sin, attend, lm_head: bool = False) -> torch.Tensor:
        """The decoder layers over hidden states ``x [t, hidden]`` (updated in place with the fused
        glue), ``attend(li, q [t, nh, hd]) -> ctx``; returns the final-normed states, or with
        ``lm_head`` the logits. The fused glue folds each residual add into the next RMSNorm and
        SiLU(gate) * up into one launch; with one token row both ride inside the projections."""
        if (self.glue == "fused" and self.prologue == "fused" and self.proj == "gemv"
                and t <= self.GEMV_MAX_ROWS):
            return self._streamed_stack(x, t, pos_t, attend, lm_head)
        if self.glue == "fused":
            _, h = ops.add_rmsnorm(x, None, self.layers[0]["in_ln"], self.eps)
            for li, ly in enumerate(self.layers):
                q = self._attn_inputs(h, ly, li, t, pos_t, pos_rows, cos, sin)
                o = self._mm(attend(li, q).reshape(t, self.q_dim), ly["wo"])
                _, h2 = ops.add_rmsnorm(x, o, ly["post_ln"], self.eps, x_out=x)
                dn = self._mm(self._mm(h2, ly["wgu"]), ly["wd"], silu_gate_up=True)
                nxt = self.layers[li + 1]["in_ln"] if li + 1 < self.L else self.final_norm
                _, h = ops.add_rmsnorm(x, dn, nxt, self.eps, x_out=x)
        else:
            for li, ly in enumerate(self.layers):
                q = self._attn_inputs(_rmsnorm(x, ly["in_ln"], self.eps), ly, li, t, pos_t,
                                      pos_rows, cos, sin)
                x = x + attend(li, q).reshape(t, self.q_dim) @ ly["wo"].T
                x = self._mlp(x, ly)
            h = _rmsnorm(x, self.final_norm, self.eps)
        return self._mm(h, self.lm_head) if lm_head else h

    def _streamed_stack(self, x: torch.Tensor, t: int, pos_t: torch.Tensor, attend,
                        lm_head: bool) -> torch.Tensor:
        """One-token-row decoder layers as weight streams with the glue inside: x + delta and its
        RMSNorm in the qkv / gate_up / lm_head staging, SiLU(gate) * up in the down projection."""
        xs = (x, torch.empty_like(x))
        cur, delta, norm = 0, None, self.layers[0]["in_ln"]

        def normed_proj(w, nw):
            nonlocal cur
            if delta is None:
                return ops.gemv(xs[cur], w, norm_weight=nw, eps=self.eps)
            y = ops.gemv(xs[cur], w, norm_weight=nw, delta=delta, x_out=xs[1 - cur], eps=self.eps)
            cur = 1 - cur
            return y

        for li, ly in enumerate(self.layers):
            qkv = normed_proj(ly["wqkv"], norm)
            q = ops.qk_norm_rope_append(qkv, ly["qn"], ly["kn"], self.eps, self.cos_tab,
                                        self.sin_tab, pos_t, self.kc[li], self.vc[li],
                                        num_qo_heads=self.nh, num_kv_heads=self.nkv)
            delta = ops.gemv(attend(li, q).reshape(t, self.q_dim), ly["wo"])
            gu = normed_proj(ly["wgu"], ly["post_ln"])
            delta = ops.gemv(gu, ly["wd"], silu_gate_up=True)
            norm = self.layers[li + 1]["in_ln"] if li + 1 < self.L else self.final_norm
        if lm_head:
            return normed_proj(self.lm_head, self.final_norm)
        _, h = ops.add_rmsnorm(xs[cur], delta, self.final_norm, self.eps,
                               x_out=xs[1 - cur])
        return h

    # ---- prefill ----
    def _prefill_forward(self, bound: int) -> torch.Tensor:
        t = bound
        rows = torch.arange(t, device=self.dev)
        cos, sin = (None, None) if self.prologue == "fused" else self._cos_sin(rows)
        x = self.embed[self.pre_tok[:bound]].to(self.dt).contiguous()

        def attend(li, q):
            return ops.gqa_prefill(q, self.kc[li, :t], self.vc[li, :t], causal=True, scale=self.scale)

        return self._layer_stack(x, t, self.zero_pos, rows, cos, sin, attend)

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
        plen = int(ids.shape[0])
        bound = next(b for b in self.pre_buckets if b >= plen)
        self.pre_tok[:plen].copy_(ids)
        self.pre_tok[plen:bound].zero_()
        if bound not in self._pre_graphs:
            self._capture_prefill(bound)
        self._pre_graphs[bound].replay()
        return self._mm(self._pre_hidden[bound][plen - 1: plen], self.lm_head).float()

    # ---- decode ----
    def _decode_forward(self, bound: int) -> torch.Tensor:
        cos, sin = (None, None) if self.prologue == "fused" else self._cos_sin(self.pos_buf)
        x = self.embed[self.tok_buf].to(self.dt).contiguous()

        def attend(li, q):
            return ops.gqa_decode(q.reshape(1, 1, self.nh, self.hd), self.kc[li], self.vc[li],
                                  self.pos_buf, scale=self.scale, max_kv_len=bound,
                                  workspace=self.attn_ws, stable_prefix=True)

        return self._layer_stack(x, 1, self.pos_buf, self.pos_buf, cos, sin, attend,
                                 lm_head=True).float()

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

    def _replay(self, pos: int) -> int:
        if pos >= self.max_len:
            raise RuntimeError("decode position exceeds graph_max_len")
        bound = self._bucket_for(pos)
        if bound not in self._graphs:
            self._capture(bound)
        self._graphs[bound].replay()
        return bound

    def decode(self, token: int, pos: int) -> torch.Tensor:
        self.tok_buf.fill_(int(token))
        self.pos_buf.fill_(int(pos))
        return self._logits[self._replay(pos)]

    def decode_argmax(self, token: int, pos: int) -> int:
        self.tok_buf.fill_(int(token))
        self.pos_buf.fill_(int(pos))
        return int(self._tok[self._replay(pos)].item())

    def decode_gpu(self, tok_t: torch.Tensor, pos: int) -> torch.Tensor:
        self.tok_buf.copy_(tok_t.view(1))
        self.pos_buf.fill_(int(pos))
        return self._logits[self._replay(pos)].argmax(-1)

    def decode_gpu_argmax(self, tok_t: torch.Tensor, pos: int) -> torch.Tensor:
        self.tok_buf.copy_(tok_t.view(1))
        self.pos_buf.fill_(int(pos))
        return self._tok[self._replay(pos)].clone()

    # ---- verify ----
    def _verify_forward(self) -> torch.Tensor:
        k1 = self.vtok.shape[0]
        pos = self.vpos0 + torch.arange(k1, device=self.dev)
        cos, sin = (None, None) if self.prologue == "fused" else self._cos_sin(pos)
        x = self.embed[self.vtok].to(self.dt).contiguous()

        def attend(li, q):
            return ops.gqa_decode(q.reshape(1, k1, self.nh, self.hd), self.kc[li], self.vc[li],
                                  self.vpos0, scale=self.scale, workspace=self.attn_ws,
                                  stable_prefix=True)

        return self._layer_stack(x, k1, self.vpos0, pos, cos, sin, attend, lm_head=True).float()

    def verify(self, tok_t: torch.Tensor, pos_start: int) -> torch.Tensor:
        if self.verify_graph is None:
            k1 = int(tok_t.shape[0])
            if k1 * self.groups > 32:
                raise RuntimeError(f"verify supports at most {32 // self.groups} tokens")
            self.vtok = torch.zeros(k1, dtype=torch.long, device=self.dev)
            self.vpos0 = torch.zeros(1, dtype=torch.long, device=self.dev)
            self.vtok.copy_(tok_t)
            self.vpos0.fill_(int(pos_start))
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
        """Prefill then ``steps`` greedy tokens through the decode graphs."""
        toks = [int(self.prefill(prompt).argmax(-1).item())]
        pos = int(prompt.shape[0])
        for _ in range(steps):
            toks.append(self.decode_argmax(toks[-1], pos))
            pos += 1
        return toks


def accept_drafts(proposals: list[int], target_next: list[int]) -> list[int]:
    """Greedy speculative acceptance (the rule of ``SpecCudaGraphQwen3Executor._spec_round``,
    ``src/solort/model/cuda_graph_executor.py:476-481``): ``target_next[i]`` is the target's argmax
    after ``i`` drafts (``len(proposals) + 1`` entries). The drafts are taken while they equal the
    target's choice; the target's token after the last accepted draft closes the round. Returns the
    round's new tokens, ``accepted + 1`` of them."""
    k = len(proposals)
    if len(target_next) != k + 1:
        raise ValueError(f"need {k + 1} target tokens for {k} drafts, got {len(target_next)}")
    accepted = 0
    while accepted < k and proposals[accepted] == target_next[accepted]:
        accepted += 1
    return list(proposals[:accepted]) + [target_next[accepted]]


def spec_round(target: GraphQwen3Runner, draft: GraphQwen3Runner, last_token: int, pos: int,
               k: int) -> list[int]:
    """One speculative round (``cuda_graph_executor.py:463-482``): ``last_token`` sits at ``pos``;
    the draft runner proposes ``k`` tokens by back-to-back GPU-resident decode replays, the target
    scores ``[last_token, drafts]`` at ``pos .. pos + k`` in one verify replay (which also writes
    their KV), and ``accept_drafts`` picks the new tokens. When every draft is accepted the draft
    runner also decodes its last proposal at ``pos + k``, so its KV covers every position the next
    round starts after. One host synchronisation per round."""
    last = torch.tensor([int(last_token)], dtype=torch.long, device=target.dev)
    proposals, cur = [], last
    for i in range(k):
        cur = draft.decode_gpu(cur, pos + i)
        proposals.append(cur)
    prop = torch.cat(proposals)
    tgt = target.verify(torch.cat([last, prop]), pos).argmax(-1)
    host = torch.cat([prop, tgt]).tolist()
    new = accept_drafts(host[:k], host[k:])
    if len(new) == k + 1:
        draft.decode_gpu(prop[k - 1:k], pos + k)
    return new


def speculative_greedy(target: GraphQwen3Runner, draft: GraphQwen3Runner, prompt: torch.Tensor,
                       steps: int, k: int = 4) -> tuple[list[int], list[int]]:
    """Greedy generation with a draft model, as the reference's speculative executor runs it: both
    runners prefill the prompt, the target's prefill argmax is the first token, then speculative
    rounds until ``steps`` more tokens exist; near ``max_len`` (where a round would not fit) the
    target decodes single tokens (``:450-452``). Returns the tokens (``steps + 1``, like
    ``GraphQwen3Runner.greedy``) and each round's accepted draft count."""
    toks = [int(target.prefill(prompt).argmax(-1).item())]
    draft.prefill(prompt)
    pos = int(prompt.shape[0])  # position of toks[-1]
    accepted = []
    while len(toks) < steps + 1:
        if pos + k + 2 >= min(target.max_len, draft.max_len):
            toks.append(target.decode_argmax(toks[-1], pos))
            pos += 1
            continue
        new = spec_round(target, draft, toks[-1], pos, k)
        accepted.append(len(new) - 1)
        toks += new
        pos += len(new)
    return toks[:steps + 1], accepted
