"""The torch custom-op layer (``torch.ops.solort_attn.*``) without a GPU: every op is registered
with the schema the engine documents (outputs and workspaces marked as mutated), each fake
implementation accepts well-formed fake CUDA tensors and rejects malformed ones under
``FakeTensorMode``, and no CPU kernel exists (CPU tensors raise instead of falling back)."""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

from solort_b200 import ops, torch_ops  # noqa: F401

BF, F32, I32, I64 = torch.bfloat16, torch.float32, torch.int32, torch.int64


def test_every_op_is_registered_with_mutated_outputs():
    mutated = {
        "gqa_decode": {"out", "workspace"},
        "gqa_decode_paged": {"out", "workspace"},
        "gqa_prefill": {"out"},
        "gqa_decode_partial": {"out_f32", "lse_out", "workspace"},
        "lse_merge": {"out"},
        "kv_store": {"kv_pages"},
    }
    assert set(torch_ops.OPS) == set(mutated)
    for name, expect in mutated.items():
        schema = getattr(torch.ops.solort_attn, name).default._schema
        got = {a.name for a in schema.arguments if a.alias_info is not None and a.alias_info.is_write}
        assert got == expect, (name, got)
        assert len(schema.returns) == 0, name


def _t(*shape, dtype=BF):
    return torch.empty(*shape, dtype=dtype, device="cuda")


def test_fake_impls_trace_well_formed_calls():
    with FakeTensorMode():
        q = _t(1, 5, 32, 128)
        kv = _t(4096, 8, 128)
        ws = _t(1 << 20, dtype=torch.uint8)
        pos = _t(1, dtype=I64)
        torch.ops.solort_attn.gqa_decode(q, kv, kv, pos, _t(1, 5, 32, 128), ws, "NHD", None, 1024)
        torch.ops.solort_attn.gqa_decode(q, _t(8, 4096, 128), _t(8, 4096, 128), pos,
                                         _t(1, 5, 32, 128), ws, "HND")
        pages = _t(64, 2, 16, 8, 128)
        bt = _t(1, 64, dtype=I32)
        torch.ops.solort_attn.gqa_decode_paged(q, pages, bt, pos, _t(1, 5, 32, 128), ws, 1024)
        torch.ops.solort_attn.gqa_prefill(_t(512, 32, 128), _t(512, 8, 128), _t(512, 8, 128),
                                          _t(512, 32, 128), True, None)
        torch.ops.solort_attn.gqa_decode_partial(_t(1, 1, 32, 128), kv, kv, pos,
                                                 _t(1, 1, 32, 128, dtype=F32),
                                                 _t(1, 1, 32, dtype=F32), ws, 4096)
        torch.ops.solort_attn.lse_merge(_t(4, 1, 1, 32, 128, dtype=F32), _t(4, 1, 1, 32, dtype=F32),
                                        _t(1, 1, 32, 128))
        torch.ops.solort_attn.kv_store(_t(3, 8, 128), _t(3, 8, 128), _t(3, dtype=I64), pages)


@pytest.mark.parametrize("case", ["out_shape", "pos_dtype", "paged_rank", "bt_dtype", "merge_out",
                                  "prefill_noncausal_len", "store_slots", "kv_layout"])
def test_fake_impls_reject_malformed_calls(case):
    with FakeTensorMode():
        q = _t(1, 1, 32, 128)
        kv = _t(4096, 8, 128)
        ws = _t(0, dtype=torch.uint8)
        pos = _t(1, dtype=I64)
        pages = _t(64, 2, 16, 8, 128)
        with pytest.raises(RuntimeError):
            if case == "out_shape":
                torch.ops.solort_attn.gqa_decode(q, kv, kv, pos, _t(1, 2, 32, 128), ws)
            elif case == "pos_dtype":
                torch.ops.solort_attn.gqa_decode(q, kv, kv, _t(1, dtype=I32), _t(1, 1, 32, 128), ws)
            elif case == "paged_rank":
                torch.ops.solort_attn.gqa_decode_paged(q, _t(64, 16, 8, 128), _t(1, 64, dtype=I32),
                                                       pos, _t(1, 1, 32, 128), ws, 1024)
            elif case == "bt_dtype":
                torch.ops.solort_attn.gqa_decode_paged(q, pages, _t(1, 64, dtype=I64), pos,
                                                       _t(1, 1, 32, 128), ws, 1024)
            elif case == "merge_out":
                torch.ops.solort_attn.lse_merge(_t(4, 1, 1, 32, 128, dtype=F32),
                                                _t(4, 1, 1, 32, dtype=F32), _t(1, 1, 32, 128, dtype=F32))
            elif case == "prefill_noncausal_len":
                torch.ops.solort_attn.gqa_prefill(_t(600, 32, 128), _t(512, 8, 128), _t(512, 8, 128),
                                                  _t(600, 32, 128), True, None)
            elif case == "store_slots":
                torch.ops.solort_attn.kv_store(_t(3, 8, 128), _t(3, 8, 128), _t(2, dtype=I64), pages)
            elif case == "kv_layout":
                torch.ops.solort_attn.gqa_decode(q, kv, kv, pos, _t(1, 1, 32, 128), ws, "THD")


def test_no_cpu_kernel_is_registered():
    q = torch.zeros(1, 1, 32, 128, dtype=BF)
    kv = torch.zeros(64, 8, 128, dtype=BF)
    pos = torch.zeros(1, dtype=I64)
    with pytest.raises(NotImplementedError):
        torch.ops.solort_attn.gqa_decode(q, kv, kv, pos, torch.empty_like(q),
                                         torch.empty(0, dtype=torch.uint8))
