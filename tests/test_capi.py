"""The C-ABI library loads, exports every symbol the header declares, and its ctypes mirrors have
the header's layout. No GPU work: these run on CPU."""

from __future__ import annotations

import ctypes
import os
import re
import subprocess
import tempfile

import pytest
import torch

from solort_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADERS = [os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include"))
           if f.endswith(".h")]


def declared_symbols() -> set[str]:
    syms = set()
    for h in HEADERS:
        syms |= set(re.findall(r"SOLORT_API\s+[\w\s\*]+?\b(solort_\w+)\s*\(", open(h).read()))
    return syms


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    declared = declared_symbols()
    assert declared, "no SOLORT_API declarations found"
    for sym in sorted(declared):
        assert hasattr(lib, sym), f"{sym} declared in include/ but not exported"
    for sym in _lib.EXPORTED_SYMBOLS:
        assert sym in declared, f"{sym} bound in _lib but not declared in include/"
    assert set(_lib.EXPORTED_SYMBOLS) == declared


def test_only_c_abi_symbols_are_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    text_syms = [ln.split()[-1] for ln in out.splitlines() if " T " in ln]
    assert text_syms and all(s.startswith("solort_attn_") for s in text_syms), text_syms


def test_abi_version_and_status_strings():
    lib = _lib.load()
    assert lib.solort_attn_abi_version() >= 1
    for code in _lib.STATUS_NAMES:
        assert lib.solort_attn_status_string(code)
    assert b"unknown" in lib.solort_attn_status_string(12345)


def _c_layout(struct: str, fields: list[str]) -> dict[str, int]:
    src = ["#include <stdio.h>", "#include <stddef.h>", '#include "solort_attn.h"', "int main(void){",
           f'printf("sizeof %zu\\n", sizeof({struct}));']
    src += [f'printf("{f} %zu\\n", offsetof({struct}, {f}));' for f in fields]
    src.append("return 0;}")
    with tempfile.TemporaryDirectory() as d:
        c, exe = os.path.join(d, "t.c"), os.path.join(d, "t")
        open(c, "w").write("\n".join(src))
        subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), c, "-o", exe], check=True)
        out = subprocess.run([exe], capture_output=True, text=True, check=True).stdout
    return {ln.split()[0]: int(ln.split()[1]) for ln in out.splitlines()}


STRUCTS = [(_lib.SolortDecodeArgs, "SolortDecodeArgs"), (_lib.SolortMergeArgs, "SolortMergeArgs"),
           (_lib.SolortExchangeArgs, "SolortExchangeArgs"),
           (_lib.SolortExchangeMergeArgs, "SolortExchangeMergeArgs"),
           (_lib.SolortPrologueArgs, "SolortPrologueArgs"),
           (_lib.SolortAddRmsNormArgs, "SolortAddRmsNormArgs"),
           (_lib.SolortSiluMulArgs, "SolortSiluMulArgs"),
           (_lib.SolortGemvArgs, "SolortGemvArgs"),
           (_lib.SolortKVStoreArgs, "SolortKVStoreArgs")]


@pytest.mark.parametrize("cls,name", STRUCTS + ([(_lib.SolortPrefillArgs, "SolortPrefillArgs")]
                                                if "SolortPrefillArgs" in open(HEADERS[0]).read()
                                                else []))
def test_ctypes_struct_matches_header(cls, name):
    fields = [f[0] for f in cls._fields_]
    c = _c_layout(name, fields)
    assert c["sizeof"] == ctypes.sizeof(cls)
    for f in fields:
        assert c[f] == getattr(cls, f).offset, f


def test_no_cpu_fallback():
    """The product path refuses CPU tensors instead of computing them some other way."""
    from solort_b200 import ops

    q = torch.zeros(1, 1, 32, 128, dtype=torch.bfloat16)
    k = torch.zeros(16, 8, 128, dtype=torch.bfloat16)
    pos = torch.zeros(1, dtype=torch.int64)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.gqa_decode(q, k, k, pos)


def test_entry_points_report_no_device_without_gpu():
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _lib.load()
    a = _lib.SolortDecodeArgs()
    a.batch, a.q_len, a.num_qo_heads, a.num_kv_heads, a.head_dim = 1, 1, 32, 8, 128
    a.max_kv_len, a.kv_capacity = 1024, 1024
    need = ctypes.c_size_t(0)
    assert lib.solort_attn_decode_workspace_size(ctypes.byref(a), ctypes.byref(need)) == -6
    a.head_dim = 64
    assert lib.solort_attn_decode_workspace_size(ctypes.byref(a), ctypes.byref(need)) == -2
