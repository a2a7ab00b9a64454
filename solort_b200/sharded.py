"""Sequence-sharded long-context decode across GPUs (one process per GPU).

The reference is single-GPU; this is the engine's one sharded path. Rank ``r`` of ``R`` holds the
keys ``[r * S, (r + 1) * S)`` of the sequence in its own HBM. Per layer:

1. ``gqa_decode_partial`` over the local shard (split-KV decode + merge of its own splits) writes
   the rank's partial ``O`` (fp32, ``[rows, 128]``) and natural-log ``LSE`` (``[rows]``) into one
   packed buffer ``[rows * 129]``; local key ``t`` sits at position ``r * S + t``
   (``kv_pos_offset``), so causal limits stay exact at shard boundaries.
2. ``torch.distributed.all_gather_into_tensor`` (NCCL over NVLink / NVSwitch) brings every
   rank's packed partial into this GPU's memory: ``R * rows * 129 * 4`` bytes (16.5 KB per rank
   for 32 heads). No kernel reads peer memory, and every TMA load targets only its own CTA.
3. ``lse_merge`` combines the ``R`` partials into the bf16 output on every rank.

All buffers are allocated at construction, one set per layer, so a whole decode step (with its
NCCL calls) can be captured in one CUDA graph. The partial / merge functions are injectable so
the rank logic can also run on CPU ranks (``gloo``) against the oracle in tests.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

HEAD_DIM = 128


class ShardedDecode:
    def __init__(self, rank: int, world: int, *, num_qo_heads: int, layers: int,
                 device: torch.device, batch: int = 1, q_len: int = 1, group=None,
                 partial_fn=None, merge_fn=None, kv_layout: str = "HND"):
        if partial_fn is None or merge_fn is None:
            from solort_b200 import ops

            partial_fn = partial_fn or ops.gqa_decode_partial
            merge_fn = merge_fn or ops.lse_merge
        self.rank, self.world, self.group = rank, world, group
        self.partial_fn, self.merge_fn = partial_fn, merge_fn
        self.kv_layout = kv_layout
        self.shape = (batch, q_len, num_qo_heads)
        self.rows = batch * q_len * num_qo_heads
        self.width = self.rows * (HEAD_DIM + 1)
        self.send = torch.empty(layers, self.width, dtype=torch.float32, device=device)
        self.recv = torch.empty(layers, world * self.width, dtype=torch.float32, device=device)

    def _views(self, li: int):
        B, T, H = self.shape
        buf = self.send[li]
        o = buf[: self.rows * HEAD_DIM].view(B, T, H, HEAD_DIM)
        lse = buf[self.rows * HEAD_DIM:].view(B, T, H)
        parts = self.recv[li].view(self.world, self.width)
        o_parts = parts[:, : self.rows * HEAD_DIM].view(self.world, B, T, H, HEAD_DIM)
        lse_parts = parts[:, self.rows * HEAD_DIM:].view(self.world, B, T, H)
        return buf, o, lse, o_parts, lse_parts

    def layer(self, li: int, q: torch.Tensor, k_shard: torch.Tensor, v_shard: torch.Tensor,
              q_pos: torch.Tensor, kv_pos_offset: int, out: torch.Tensor,
              workspace: torch.Tensor | None = None) -> torch.Tensor:
        """Attention of ``q [B, q_len, nh, 128]`` over the whole sharded sequence of layer ``li``;
        ``k_shard``/``v_shard`` are this rank's keys, first one at ``kv_pos_offset``."""
        buf, o, lse, o_parts, lse_parts = self._views(li)
        self.partial_fn(q, k_shard, v_shard, q_pos, kv_pos_offset=kv_pos_offset,
                        kv_layout=self.kv_layout, out_f32=o, lse_out=lse, workspace=workspace)
        if self.world > 1:
            dist.all_gather_into_tensor(self.recv[li], buf, group=self.group)
        else:
            self.recv[li].copy_(buf)
        return self.merge_fn(o_parts, lse_parts, out=out)

    def close(self) -> None:
        self.send = self.recv = None
