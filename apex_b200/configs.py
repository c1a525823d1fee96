"""The five benchmark configurations of the attention hot path (shapes, seeds, masks).

Every configuration uses 16 query heads, 8 KV heads (GQA group 2) and head_dim 256, bf16
activations and a bf16 KV cache, per-head RMSNorm (eps 1e-6) on Q and K followed by
rotate-half RoPE over the full head_dim, softmax scale 1/sqrt(head_dim), and no norm on V.
The reference model's attention geometry (q_heads, kv_heads, head_dim, rope_pairs, rope_base,
window) is the ``AttentionShape`` of docs/B6_3_attention.md:365-384.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

# Synthetic-input streams: element (b, pos, head, d) of a tensor is a pure function of
# (seed, stream, index) with index = ((b * POS_STRIDE + pos) * heads + head) * head_dim + d.
POS_STRIDE = 1 << 20
STREAM_Q, STREAM_K, STREAM_V, STREAM_QW, STREAM_KW, STREAM_LENS = 1, 2, 3, 4, 5, 6


@dataclass(frozen=True)
class AttnConfig:
    name: str
    kind: str                     # "decode" or "prefill"
    batch: int
    seed: int
    rope_theta: float
    window: int = 0               # 0 = global causal
    seq_len: int = 0              # prefill: tokens per sequence
    chunk: int = 0                # prefill: tokens per call (== seq_len for one call)
    context: int = 0              # decode: keys per sequence including the new token
    lens_range: tuple = ()        # decode, ragged: (lo, hi) inclusive
    q_heads: int = 16
    kv_heads: int = 8
    head_dim: int = 256
    eps: float = 1e-6
    qk_norm: bool = True
    v_norm: bool = False
    partial_rope: int = 0         # pairs rotated when not all of them (the global layers' 64 of 256)
    note: str = field(default="", compare=False)

    @property
    def scale(self) -> float:
        return 1.0 / math.sqrt(self.head_dim)

    @property
    def rope_pairs(self) -> int:
        return self.partial_rope or self.head_dim // 2


CONFIGS = {
    "c1_decode": AttnConfig(
        "c1_decode", "decode", batch=1, seed=0, rope_theta=1e4, context=1024,
        note="single-layer decode, L=1024, no mask"),
    "c2_prefill_window": AttnConfig(
        "c2_prefill_window", "prefill", batch=1, seed=1, rope_theta=1e4, window=1024,
        seq_len=2048, chunk=2048, note="causal prefill, sliding window 1024"),
    "c3_ragged_decode": AttnConfig(
        "c3_ragged_decode", "decode", batch=64, seed=2, rope_theta=1e6,
        lens_range=(512, 8192), note="64 sequences, context uniform in [512, 8192]"),
    "c4_chunked_prefill": AttnConfig(
        "c4_chunked_prefill", "prefill", batch=4, seed=3, rope_theta=1e6, seq_len=32768,
        chunk=4096, note="4 x 32768 tokens in 4096-token chunks, global causal"),
    "c5_long_decode_b1": AttnConfig(
        "c5_long_decode_b1", "decode", batch=1, seed=4, rope_theta=1e6, context=131072,
        note="one 131072-key decode; KV split across GPUs"),
    "c5_long_decode_b8": AttnConfig(
        "c5_long_decode_b8", "decode", batch=8, seed=4, rope_theta=1e6, context=131072,
        note="eight 131072-key decodes; KV split across GPUs"),
    # the reference model's global ("full attention") layers: 16 q / 2 kv heads of head_dim 512, RoPE on
    # the first 64 of 256 pairs, theta 1e6, weightless RMSNorm of V (docs/B6_3_attention.md:46-60)
    "global_decode": AttnConfig(
        "global_decode", "decode", batch=8, seed=11, rope_theta=1e6, context=32768, q_heads=16, kv_heads=2,
        head_dim=512, v_norm=True, partial_rope=64,
        note="global-layer decode: 8 x 32768 keys, 2 kv heads of 512, GQA group 8"),
    "global_prefill": AttnConfig(
        "global_prefill", "prefill", batch=1, seed=12, rope_theta=1e6, seq_len=4096, chunk=4096, q_heads=16,
        kv_heads=2, head_dim=512, v_norm=True, partial_rope=64,
        note="global-layer prefill: one 4096-token chunk, 2 kv heads of 512, GQA group 8, global causal"),
    # not an attention configuration: the NVFP4 projections either side of one decode step
    "proj_decode": AttnConfig(
        "proj_decode", "proj", batch=1, seed=9, rope_theta=1e4,
        note="q/k/v and o_proj + post-attention norm of one decode token, sliding-layer shapes"),
    # the same four projections over one 4096-token prefill chunk (the chunk of c4), bf16 activations
    "proj_prefill": AttnConfig(
        "proj_prefill", "proj", batch=1, seed=10, rope_theta=1e4, seq_len=4096, chunk=4096,
        note="q/k/v and o_proj + post-attention norm of one 4096-token chunk, sliding-layer shapes"),
}


def decode_bytes(cfg: AttnConfig, lens) -> int:
    """Algorithmic HBM bytes of one decode step: K and V rows read (bf16) + q in + o out."""
    kv = sum(2 * cfg.kv_heads * int(L) * cfg.head_dim * 2 for L in lens)
    qo = 2 * len(lens) * cfg.q_heads * cfg.head_dim * 2
    return kv + qo


def visible_pairs(pos0: int, tokens: int, window: int) -> int:
    """Number of (query, key) pairs a causal (optionally windowed) prefill attends."""
    total = 0
    for t in range(tokens):
        pos = pos0 + t
        first = pos + 1 - window if (window and pos + 1 > window) else 0
        total += pos - first + 1
    return total


def prefill_flops(cfg: AttnConfig, pos0: int, tokens: int) -> int:
    """QK^T + PV FLOPs of one prefill call: 4 * Hq * d * visible pairs."""
    return 4 * cfg.q_heads * cfg.head_dim * visible_pairs(pos0, tokens, cfg.window)
