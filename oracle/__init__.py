"""CPU oracle for the SoloRT GQA attention hot path.

TEST INFRASTRUCTURE ONLY. Nothing in the product (``solort_b200``) imports this package. Only
``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline / reference arm of ``bench.py`` use
it, and only as the checker or as the timed stand-in for the reference's CPU path, never as a
fallback for the CUDA kernels.

The oracle restates, in plain torch on the CPU, the attention the reference computes on its fast
path (``src/solort/model/cuda_graph_executor.py``) and in its HF bridge fallback
(``src/solort/backends/transformers_flashinfer.py``), plus the paged-KV addressing of
``src/solort/cache/kv_cache.py``. Each function cites the reference lines it follows.

Pinning: ``tests/golden/make_golden.py`` imports the reference itself (in the build container, where
it is mounted) and records its outputs as fixtures under ``tests/golden/``;
``tests/test_oracle_golden.py`` checks every oracle function against them.
"""

from oracle.attention import (  # noqa: F401
    attention_fp32,
    decode_reference_grouped,
    inv_freq,
    cos_sin,
    lse_merge,
    make_attention_inputs,
    prefill_reference,
    rmsnorm,
    rope,
    sdpa_bottom_right,
    verify_reference,
)
from oracle.paged import (  # noqa: F401
    gather_layer_tokens,
    last_page_len,
    metadata_for,
    pages_required,
    slot_mapping,
    store_layer_tokens,
)
