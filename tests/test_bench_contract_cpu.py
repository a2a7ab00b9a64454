"""The benchmark's JSON contract on the CPU: the reference arm (the reference's grouped decode,
restated in oracle/, on the host cores) prints one line with every key the driver reads, and the
C header's constants match the Python binding's."""

from __future__ import annotations

import json
import os
import re
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
         "--warmup", "1", "--ctx", "1024", "--cpu-sample-s", "1"],
        capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "impl",
                "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["value"] > 0 and line["steps"] == 1
    assert line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] >= 1
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]


def test_header_constants_match_the_binding():
    from solort_b200 import _lib

    text = open(os.path.join(ROOT, "include", "solort_attn.h")).read()
    assert int(re.search(r"#define SOLORT_DECODE_STABLE_PREFIX (\d+)u", text).group(1)) == \
        _lib.DECODE_STABLE_PREFIX
    assert int(re.search(r"#define SOLORT_MAX_RANKS (\d+)", text).group(1)) == _lib.MAX_RANKS
    abi = int(re.search(r"#define SOLORT_ATTN_ABI_VERSION (\d+)", text).group(1))
    assert _lib.load().solort_attn_abi_version() == abi


def test_roofline_traffic_comes_from_committed_ncu_summaries():
    """Every workload with a committed ncu capture yields its per-launch DRAM bytes from the
    summary's `traffic_per_launch_bytes:` line, and the figure is close to the algorithmic bytes
    of one launch (K + V read once: 4096 bytes per key for 32/8 heads at head_dim 128)."""
    sys.path.insert(0, ROOT)
    import bench

    assert bench.TRAFFIC_PROFILES
    for (workload, keys), rel in bench.TRAFFIC_PROFILES.items():
        assert os.path.exists(os.path.join(ROOT, rel)), rel
        traffic, src = bench._profiled_traffic(workload, keys)
        assert src == rel and isinstance(traffic, int)
        algorithmic = 4096 * keys
        assert algorithmic <= traffic <= 1.05 * algorithmic, (rel, traffic, algorithmic)
    assert bench._profiled_traffic("decode", 12345) == (None, None)
