"""Sequence-sharded long-context decode across GPUs (one process per GPU).

The reference is single-GPU; this is the engine's one sharded path. Rank ``r`` of ``R`` holds the
keys ``[r * S, (r + 1) * S)`` of the sequence in its own HBM; local key ``t`` sits at position
``r * S + t`` (``kv_pos_offset``), so causal limits stay exact at shard boundaries. Per layer each
rank computes its partial ``O`` (fp32 ``[rows, 128]``) and natural-log ``LSE`` (``[rows]``), the
partials reach every rank, and each rank merges the ``R`` of them into the bf16 output.

Two exchanges:

* ``exchange="p2p"`` (the GPU path ``bench.py`` runs): ``gqa_decode_exchange`` -- the split-KV
  decode whose merge kernel stores the rank's partial rows straight into its slot on every rank
  over NVLink, as 64-bit words that each carry a float and an arrival mark -- then
  ``exchange_merge``, which polls its slots (bounded) until every word is marked, merges and zeroes
  them. The slots live in ``PeerExchange`` buffers: plain allocations exported by CUDA IPC and
  mapped point to point by every peer. No collective library, fence or flag, and no load from peer
  memory.
* ``exchange="nccl"``: ``gqa_decode_partial`` into a packed ``[rows * 129]`` buffer,
  ``torch.distributed.all_gather_into_tensor`` (NCCL over NVLink / NVSwitch), then ``lse_merge``.
  The partial / merge functions are injectable so this rank logic also runs on CPU ranks
  (``gloo``) against the oracle in tests.

Everything is allocated at construction, one slot set per layer, so a whole decode step can be
captured in one CUDA graph: a layer's slots are written again only in the next step, after every
rank has finished reading them (each rank's next-step send for that layer follows, in stream order,
its receipt of the other ranks' partials for all later layers of this step).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

HEAD_DIM = 128
SLOT_FLOATS_PER_ROW = HEAD_DIM + 1  # O row + its LSE


def exchange_layout(rank: int, world: int, rows: int, layers: int) -> dict:
    """Byte layout of one rank's exchange buffer: ``[layers][world]`` slots of ``rows * 129``
    64-bit words (each a float plus its arrival mark), padded to 256 bytes so every slot is
    16-byte aligned. Slot ``(li, src)`` receives rank ``src``'s partial for layer ``li``. Returns
    the sizes and the slot offset function."""
    slot_bytes = -(-rows * SLOT_FLOATS_PER_ROW * 8 // 256) * 256

    def slot(li: int, src: int) -> int:
        return (li * world + src) * slot_bytes

    return {"slot_bytes": slot_bytes, "total_bytes": layers * world * slot_bytes, "slot": slot}


class PeerExchange:
    """This rank's receive buffer plus the mappings of every peer's, for ``layers`` slot sets."""

    def __init__(self, rank: int, world: int, rows: int, layers: int, group=None, *,
                 emulated_bases: list[int] | None = None):
        from solort_b200 import _lib

        if not 1 <= world <= _lib.MAX_RANKS:
            raise RuntimeError(f"the peer exchange supports 1..{_lib.MAX_RANKS} ranks, got {world}")
        self.lib = _lib.load()
        self.rank, self.world, self.rows, self.layers, self.group = rank, world, rows, layers, group
        self.layout = exchange_layout(rank, world, rows, layers)
        if emulated_bases is not None:
            # All ranks in this process on one GPU (see emulate()): nothing to map.
            self.base, self.own = list(emulated_bases), emulated_bases[rank]
            self.opened, self.owns_buffer = [], False
            self.send_args = [self._send_args(li) for li in range(layers)]
            return
        self.owns_buffer = True
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES)()
        _lib.check(self.lib.solort_attn_exchange_buffer_create(self.layout["total_bytes"],
                                                               ctypes.byref(ptr), handle),
                   "solort_attn_exchange_buffer_create")
        self.own = ptr.value
        handles = [bytes(handle)]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
        self.base = [0] * world
        self.opened = []
        for p in range(world):
            if p == rank:
                self.base[p] = self.own
                continue
            peer = ctypes.c_void_p()
            hb = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES).from_buffer_copy(handles[p])
            _lib.check(self.lib.solort_attn_exchange_buffer_open(hb, ctypes.byref(peer)),
                       "solort_attn_exchange_buffer_open")
            self.base[p] = peer.value
            self.opened.append(peer.value)
        if world > 1:
            dist.barrier(group=group)  # every buffer is mapped everywhere before anyone writes
        self.send_args = [self._send_args(li) for li in range(layers)]

    def _send_args(self, li: int):
        from solort_b200 import _lib

        x = _lib.SolortExchangeArgs()
        x.num_ranks, x.rank = self.world, self.rank
        for p in range(self.world):
            x.slot_in_rank[p] = self.base[p] + self.layout["slot"](li, self.rank)
        return x

    def recv(self, li: int) -> tuple[int, int]:
        """This rank's receive slots for layer ``li``: (address, stride in 64-bit words), rank
        ``s``'s slot at ``address + s * stride`` words."""
        return self.own + self.layout["slot"](li, 0), self.layout["slot_bytes"] // 8

    @classmethod
    def emulate(cls, world: int, rows: int, layers: int) -> list["PeerExchange"]:
        """``world`` ranks' exchanges inside this process on the current GPU, for tests: every
        rank's buffer is local memory, and a caller that runs all ranks' sends before any rank's
        merge never has a kernel waiting on one that has not finished."""
        from solort_b200 import _lib

        lib = _lib.load()
        lay = exchange_layout(0, world, rows, layers)
        bases = []
        for _ in range(world):
            ptr = ctypes.c_void_p()
            handle = (ctypes.c_ubyte * _lib.IPC_HANDLE_BYTES)()
            _lib.check(lib.solort_attn_exchange_buffer_create(lay["total_bytes"], ctypes.byref(ptr),
                                                              handle),
                       "solort_attn_exchange_buffer_create")
            bases.append(ptr.value)
        xs = [cls(r, world, rows, layers, emulated_bases=bases) for r in range(world)]
        for x in xs:
            x.owns_buffer = True  # each emulated rank frees its own buffer on close()
        return xs

    def close(self) -> None:
        if self.own is None:
            return
        if self.opened:
            dist.barrier(group=self.group)  # nobody stores into a buffer that is going away
        for p in self.opened:
            self.lib.solort_attn_exchange_buffer_close(ctypes.c_void_p(p))
        if self.owns_buffer:
            self.lib.solort_attn_exchange_buffer_destroy(ctypes.c_void_p(self.own))
        self.own, self.opened = None, []


class ShardedDecode:
    def __init__(self, rank: int, world: int, *, num_qo_heads: int, layers: int,
                 device: torch.device, batch: int = 1, q_len: int = 1, group=None,
                 partial_fn=None, merge_fn=None, kv_layout: str = "HND", exchange: str = "nccl"):
        if exchange not in ("nccl", "p2p"):
            raise ValueError(exchange)
        self.rank, self.world, self.group = rank, world, group
        self.exchange = exchange
        self.kv_layout = kv_layout
        self.shape = (batch, q_len, num_qo_heads)
        self.rows = batch * q_len * num_qo_heads
        self.width = self.rows * (HEAD_DIM + 1)
        self.px = None
        if exchange == "p2p":
            self.px = PeerExchange(rank, world, self.rows, layers, group=group)
            return
        if partial_fn is None or merge_fn is None:
            from solort_b200 import ops

            partial_fn = partial_fn or ops.gqa_decode_partial
            merge_fn = merge_fn or ops.lse_merge
        self.partial_fn, self.merge_fn = partial_fn, merge_fn
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
              workspace: torch.Tensor | None = None, stable_prefix: bool = False) -> torch.Tensor:
        """Attention of ``q [B, q_len, nh, 128]`` over the whole sharded sequence of layer ``li``;
        ``k_shard``/``v_shard`` are this rank's keys, first one at ``kv_pos_offset``
        (``stable_prefix`` as in ``ops.gqa_decode``, peer exchange only)."""
        if self.px is not None:
            from solort_b200 import ops

            ops.gqa_decode_exchange(q, k_shard, v_shard, q_pos, self.px.send_args[li],
                                    kv_pos_offset=kv_pos_offset, kv_layout=self.kv_layout,
                                    workspace=workspace, stable_prefix=stable_prefix)
            return ops.exchange_merge(*self.px.recv(li), self.world, out)
        buf, o, lse, o_parts, lse_parts = self._views(li)
        self.partial_fn(q, k_shard, v_shard, q_pos, kv_pos_offset=kv_pos_offset,
                        kv_layout=self.kv_layout, out_f32=o, lse_out=lse, workspace=workspace)
        if self.world > 1:
            dist.all_gather_into_tensor(self.recv[li], buf, group=self.group)
        else:
            self.recv[li].copy_(buf)
        return self.merge_fn(o_parts, lse_parts, out=out)

    def prepared_layer(self, li: int, q: torch.Tensor, k_shard: torch.Tensor,
                       v_shard: torch.Tensor, q_pos: torch.Tensor, kv_pos_offset: int,
                       out: torch.Tensor, workspace: torch.Tensor, stable_prefix: bool = False):
        """``layer`` with its arguments packed once (peer exchange only): a callable that launches
        the layer's two kernels on the current stream."""
        from solort_b200 import ops

        if self.px is None:
            raise RuntimeError("prepared layers need exchange='p2p'")
        return ops.ShardedDecodeCall(q, k_shard, v_shard, q_pos, self.px.send_args[li],
                                     *self.px.recv(li), self.world, kv_pos_offset=kv_pos_offset,
                                     kv_layout=self.kv_layout, out=out, workspace=workspace,
                                     stable_prefix=stable_prefix)

    def close(self) -> None:
        if self.px is not None:
            self.px.close()
            self.px = None
        self.send = self.recv = None
