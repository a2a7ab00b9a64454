"""The peer-memory exchange of the sequence-sharded decode, with R ranks emulated on one GPU.

Each emulated rank owns a shard of the keys and an exchange buffer in this GPU's memory. All R
ranks' sends (``gqa_decode_exchange``: decode over the shard, then stores of the rank's partial
into its slot on every rank as self-marking 64-bit words) run before any rank's ``exchange_merge``,
so every word a merge waits for is already there: no kernel ever waits on one that has not
finished. The merged output of every rank must match the oracle's attention over the whole sequence
(max-abs <= 2e-2, mean-abs <= 2e-3), on two rounds in a row (the merges zero the slots for the
next round).
"""

from __future__ import annotations

import time

import pytest
import torch

from oracle import attention as A

pytestmark = pytest.mark.gpu


def _close(got, ref, what):
    d = (got.float().cpu() - ref.float().cpu()).abs()
    assert torch.isfinite(got.float()).all(), what
    assert d.max().item() <= 2e-2, f"{what}: max-abs {d.max().item():.4g}"
    assert d.mean().item() <= 2e-3, f"{what}: mean-abs {d.mean().item():.4g}"


@pytest.mark.parametrize("R,L", [(1, 4096), (2, 8192), (4, 8192), (8, 2048), (3, 3000)])
def test_emulated_exchange_matches_full_attention(R, L):
    from solort_b200 import ops
    from solort_b200.sharded import PeerExchange

    S = -(-L // R)
    q, k, v = A.make_attention_inputs(R * 10 + L, 32, 8, 128, 1, S * R, L - 1)
    ref, _ = A.attention_fp32(q, k[:L], v[:L], 128**-0.5, L - 1)
    xs = PeerExchange.emulate(R, rows=32, layers=2)
    try:
        dq = q[None].cuda()
        qpos = torch.tensor([L - 1], dtype=torch.int64, device="cuda")
        shards = [(k[r * S:(r + 1) * S].cuda(), v[r * S:(r + 1) * S].cuda()) for r in range(R)]
        for rnd in range(2):
            for li in range(2):
                for r in range(R):
                    ops.gqa_decode_exchange(dq, *shards[r], qpos, xs[r].send_args[li],
                                            kv_pos_offset=r * S, max_kv_len=S)
                outs = [ops.exchange_merge(*xs[r].recv(li), R,
                                           torch.full_like(dq, float("nan")))
                        for r in range(R)]
                torch.cuda.synchronize()
                for r in range(R):
                    _close(outs[r][0], ref, f"R={R} rank {r} layer {li} round {rnd}")
        assert ops.device_status() == 0
    finally:
        for x in xs:
            x.close()


def test_exchange_merge_gives_up_on_a_missing_peer():
    """Rank 1 never sends: the merge's bounded wait expires, the device status reports it (bit 3)
    and the context stays usable."""
    from solort_b200 import ops
    from solort_b200.sharded import PeerExchange

    L = 1024
    q, k, v = A.make_attention_inputs(7, 32, 8, 128, 1, L, L - 1)
    xs = PeerExchange.emulate(2, rows=32, layers=1)
    try:
        dq = q[None].cuda()
        qpos = torch.tensor([L - 1], dtype=torch.int64, device="cuda")
        ops.gqa_decode_exchange(dq, k.cuda(), v.cuda(), qpos, xs[0].send_args[0])
        out = torch.full_like(dq, 3.0)
        t0 = time.monotonic()
        ops.exchange_merge(*xs[0].recv(0), 2, out)
        torch.cuda.synchronize()
        assert time.monotonic() - t0 < 30
        assert ops.device_status() & 8
        assert (out == 3.0).all(), "a row whose peer never arrived must not be written"
        ops.gqa_decode(dq, k.cuda(), v.cuda(), qpos)  # the context still works
        torch.cuda.synchronize()
        assert ops.device_status() == 0
    finally:
        for x in xs:
            x.close()
