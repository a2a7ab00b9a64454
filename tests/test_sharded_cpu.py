"""Sequence-sharded decode host logic on CPU ranks (gloo, world size 2), and host-side failure
detection. The CUDA kernels are replaced by the oracle here (test infrastructure); the GPU path
runs the same class with the real kernels and NCCL in bench.py / the multi-GPU runs."""

from __future__ import annotations

import datetime
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

NH, NKV, HD = 32, 8, 128


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_partial(q, k, v, q_pos, *, kv_pos_offset, kv_layout, out_f32, lse_out, workspace=None):
    from oracle import attention as A

    assert kv_layout == "HND"
    o, lse = A.attention_fp32(q[0], k.transpose(0, 1), v.transpose(0, 1), HD ** -0.5,
                              int(q_pos[0]), kv_pos0=kv_pos_offset)
    out_f32[0].copy_(o)
    lse_out[0].copy_(lse)


def _oracle_merge(o_parts, lse_parts, *, out):
    from oracle import attention as A

    o, _ = A.lse_merge(o_parts, lse_parts)
    out.copy_(o)
    return out


def _worker(rank, world, port, L, q_len, result_q, fail_rank):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=10))
        from oracle import attention as A
        from solort_b200.sharded import ShardedDecode

        q, k, v = A.make_attention_inputs(17, NH, NKV, HD, q_len, L, L - q_len)
        shard = L // world
        ks = k[rank * shard:(rank + 1) * shard].float().transpose(0, 1).contiguous()
        vs = v[rank * shard:(rank + 1) * shard].float().transpose(0, 1).contiguous()
        sd = ShardedDecode(rank, world, num_qo_heads=NH, layers=2, device=torch.device("cpu"),
                           q_len=q_len, partial_fn=_oracle_partial, merge_fn=_oracle_merge)
        out = torch.empty(1, q_len, NH, HD)
        qpos = torch.tensor([L - q_len])
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        try:
            sd.layer(1, q.float()[None], ks, vs, qpos, rank * shard, out)
        except Exception as exc:  # the survivor must see an error, not hang
            result_q.put((rank, "collective_error", type(exc).__name__))
            return
        ref, _ = A.attention_fp32(q, k, v, HD ** -0.5, L - q_len)
        err = (out[0] - ref).abs().max().item()
        result_q.put((rank, "ok", err))
        dist.destroy_process_group()
    except Exception:
        result_q.put((rank, "raised", traceback.format_exc(limit=1)))


def _run(world, L, q_len, fail_rank=-1, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, L, q_len, q, fail_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, status, info = q.get(timeout=timeout)
        results[r] = (status, info)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


@pytest.mark.parametrize("q_len", [1, 4])
def test_sharded_decode_two_ranks_matches_full_attention(q_len):
    res = _run(2, 512, q_len)
    for r in (0, 1):
        status, err = res[r]
        assert status == "ok", res
        assert err < 1e-4, res


def test_rank_failure_before_collective_is_reported_not_hung():
    res = _run(2, 256, 1, fail_rank=1)
    assert res[1][0] == "raised"
    assert res[0][0] == "collective_error", res


@pytest.mark.parametrize("world,rows,layers", [(1, 32, 36), (2, 32, 36), (8, 32, 36), (3, 5, 4)])
def test_exchange_layout_slots_are_aligned_and_disjoint(world, rows, layers):
    """The peer-exchange buffer: every slot 16-byte aligned (vector stores), slots never overlap,
    and all of them fit in the allocation."""
    from solort_b200.sharded import SLOT_FLOATS_PER_ROW, exchange_layout

    lay = exchange_layout(0, world, rows, layers)
    assert lay["slot_bytes"] >= rows * SLOT_FLOATS_PER_ROW * 8
    spans = []
    for li in range(layers):
        for src in range(world):
            s = lay["slot"](li, src)
            assert s % 16 == 0
            spans.append((s, s + rows * SLOT_FLOATS_PER_ROW * 8))
    spans.sort()
    for (a0, a1), (b0, _) in zip(spans, spans[1:]):
        assert a1 <= b0
    assert spans[-1][1] <= lay["total_bytes"]
