"""apex_b200 -- B200-native (sm_100a) attention hot path of spotta85/apex.

Per-head QK RMSNorm + RoPE fused into grouped-query attention over a bf16 KV cache, for
single-token decode (split-KV, HBM-bound) and causal / sliding-window prefill (tcgen05 tensor
cores), behind the reference's operator interface.  See ``apex_b200.ops`` for the Python
operator API, ``include/apex_cuda.h`` for the C ABI and ``apex_b200/csrc`` for the C++
backend and the kernels.
"""
from . import configs  # noqa: F401

__all__ = ["configs", "ops", "build", "dist"]
