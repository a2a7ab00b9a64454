"""B200-native (sm_100a) grouped-query attention engine for SoloRT's Qwen3 fast path.

The CUDA kernels live in the in-tree ``libsolort_attn.so`` behind the C ABI of
``include/solort_attn.h``; ``solort_b200.ops`` exposes them to torch.
"""

__version__ = "0.1.0"
