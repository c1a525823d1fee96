"""Operator API of the attention hot path, over the C ABI, on torch device tensors.

The names and argument meaning mirror the reference's operator layer:

* ``head_norm_rope``   apex::headNormRope (src/ops.h:88-122): same arguments in the same order,
                       with tensors in place of (Buffer*, byte offset) pairs -- pass a view
                       (e.g. ``cache.k[..., pos0:, :]``) where the reference passes an offset.
* ``attention``        apex::attention (docs/B6_3_attention.md:424-431) on an f32 KvCache.
* ``attention_decode`` / ``attention_prefill``: the bf16 path -- the steps of
                       apex::attentionBlock between its projections (docs/B6_3_attention.md:
                       444-454) fused per call over a bf16 KV cache.

Tensors must be CUDA, contiguous where stated, and of the stated dtype; every call enqueues on
the current torch stream.  Errors raise :class:`apex_b200._native.ApexError`; nothing falls
back to another implementation.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import ctypes

import torch

from . import _native
from ._native import AttnParams, check


@dataclass(frozen=True)
class AttentionShape:
    """The reference's AttentionShape (docs/B6_3_attention.md:365-372) + bf16-path knobs."""
    q_heads: int
    kv_heads: int
    head_dim: int
    rope_pairs: int
    rope_base: float
    window: int = 0
    scale: float = 1.0
    eps: float = 1e-6
    qk_norm: bool = True
    v_norm: bool = False
    ring: bool = False            # decode: the cache is a ring of `capacity` slots (position % capacity)

    def c(self) -> AttnParams:
        return AttnParams(self.q_heads, self.kv_heads, self.head_dim, self.rope_pairs,
                          self.rope_base, self.window, self.scale, self.eps, int(self.qk_norm),
                          int(self.v_norm), int(self.ring))

    @staticmethod
    def from_config(cfg) -> "AttentionShape":
        return AttentionShape(cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.rope_pairs,
                              cfg.rope_theta, cfg.window, cfg.scale, cfg.eps, cfg.qk_norm,
                              cfg.v_norm)


@dataclass
class KvCache:
    """One layer's cache (docs/B6_3_attention.md:394-398): k, v [kv_heads][capacity][hd], or
    [B][kv_heads][capacity][hd] for the batched bf16 path."""
    k: torch.Tensor
    v: torch.Tensor

    @property
    def capacity(self) -> int:
        return self.k.shape[-2]


def _ptr(t):
    return None if t is None else ctypes_ptr(t)


def ctypes_ptr(t: torch.Tensor):
    if not t.is_cuda:
        raise ValueError("apex_b200 ops take CUDA tensors")
    return t.data_ptr()


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _need(t: torch.Tensor, dtype, name: str, contiguous: bool = True):
    if t.dtype != dtype:
        raise TypeError(f"{name}: expected {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name}: must be contiguous")
    if not t.is_cuda:
        raise ValueError(f"{name}: must be a CUDA tensor")


# ---------------------------------------------------------------------------- f32 drop-ins

def head_norm_rope(input: torch.Tensor, weights, has_weights: bool, output: torch.Tensor,
                   tokens: int, heads: int, head_dim: int, rope_pairs: int, rope_base: float,
                   abs_pos: int, out_token_stride: int, out_head_stride: int, eps: float) -> None:
    """apex::headNormRope (src/ops.h:88-122).  f32 input [tokens, heads, head_dim] -> output
    element (t, h, d) at output.flat[t*out_token_stride + h*out_head_stride + d] (output may
    be a view starting where the reference's output_offset points).  bf16 tensors select the
    bf16 kernel.  weights: bf16 [head_dim] (torch.bfloat16 or int16 raw bits) or None."""
    lib = _native.load()
    fn = lib.apex_head_norm_rope_f32 if input.dtype == torch.float32 else lib.apex_head_norm_rope_bf16
    if input.dtype not in (torch.float32, torch.bfloat16) or output.dtype != input.dtype:
        raise TypeError("head_norm_rope: input and output must both be float32 or both bfloat16")
    if not input.is_contiguous():
        raise ValueError("head_norm_rope: input must be contiguous")
    w = None
    if has_weights:
        if weights is None:
            raise ValueError("head_norm_rope: has_weights without weights")
        w = weights.data_ptr()
    check(fn(ctypes_ptr(input), w, ctypes_ptr(output), tokens, heads, head_dim, int(has_weights),
             rope_pairs, rope_base, abs_pos, out_token_stride, out_head_stride, eps, _stream()))


def attention(q: torch.Tensor, cache: KvCache, output: torch.Tensor, shape: AttentionShape,
              tokens: int, pos0: int) -> None:
    """apex::attention (docs/B6_3_attention.md:424-431): f32 q, out [tokens, q_heads, hd];
    cache.k / cache.v f32 [kv_heads, capacity, hd]; softmax scale = shape.scale (the
    reference's value is 1.0)."""
    for t, n in ((q, "q"), (cache.k, "cache.k"), (cache.v, "cache.v"), (output, "output")):
        _need(t, torch.float32, n)
    lib = _native.load()
    check(lib.apex_attention_f32_scaled(q.data_ptr(), cache.k.data_ptr(), cache.v.data_ptr(),
                                        output.data_ptr(), tokens, shape.q_heads, shape.kv_heads,
                                        shape.head_dim, cache.capacity, pos0, shape.window,
                                        shape.scale, _stream()))


# ---------------------------------------------------------------------------- bf16 hot path

class DecodeWorkspace:
    """Device workspace of attention_decode for up to `batch` sequences of `max_seq_len` keys.
    Allocated once (its counters zeroed once); every decode call leaves them zero again."""

    def __init__(self, shape: AttentionShape, batch: int, max_seq_len: int, device=None):
        p = shape.c()
        lib = _native.load()
        self.nbytes = int(lib.apex_attn_decode_workspace_bytes(p, batch, max_seq_len))
        self.buffer = torch.empty(max(self.nbytes, 16), dtype=torch.uint8, device=device or "cuda")
        check(lib.apex_attn_decode_workspace_init(self.buffer.data_ptr(), self.nbytes, _stream()))
        self.batch, self.max_seq_len = batch, max_seq_len


def _check_decode(shape, q_raw, k_new, v_new, cache, seq_lens, B):
    Hq, Hkv, D = shape.q_heads, shape.kv_heads, shape.head_dim
    _need(q_raw, torch.bfloat16, "q_raw")
    _need(k_new, torch.bfloat16, "k_new")
    _need(v_new, torch.bfloat16, "v_new")
    _need(cache.k, torch.bfloat16, "cache.k")
    _need(cache.v, torch.bfloat16, "cache.v")
    _need(seq_lens, torch.int32, "seq_lens")
    if q_raw.numel() != B * Hq * D or k_new.numel() != B * Hkv * D or v_new.numel() != B * Hkv * D:
        raise ValueError("attention_decode: q_raw [B,Hq,D], k_new/v_new [B,Hkv,D] expected")
    if cache.k.shape != cache.v.shape or cache.k.numel() != B * Hkv * cache.capacity * D:
        raise ValueError("attention_decode: caches must be [B, Hkv, capacity, D]")
    if seq_lens.numel() != B:
        raise ValueError("attention_decode: seq_lens must have B entries")


def attention_decode(shape: AttentionShape, q_raw, k_new, v_new, q_norm_w, k_norm_w,
                     cache: KvCache, seq_lens: torch.Tensor, max_seq_len: int, out: torch.Tensor,
                     workspace: DecodeWorkspace) -> torch.Tensor:
    """One fused decode step (apex_attn_decode_bf16).  q_raw [B,Hq,D], k_new/v_new [B,Hkv,D]
    bf16 (raw projections); cache [B,Hkv,cap,D] bf16; seq_lens int32 [B] (keys incl. the new
    token, which is appended at position seq_lens[b]-1); out [B,Hq,D] bf16."""
    B = seq_lens.numel()
    _check_decode(shape, q_raw, k_new, v_new, cache, seq_lens, B)
    _need(out, torch.bfloat16, "out")
    lib = _native.load()
    check(lib.apex_attn_decode_bf16(shape.c(), q_raw.data_ptr(), k_new.data_ptr(), v_new.data_ptr(),
                                    _ptr(q_norm_w), _ptr(k_norm_w), cache.k.data_ptr(),
                                    cache.v.data_ptr(), cache.capacity, seq_lens.data_ptr(), B,
                                    max_seq_len, out.data_ptr(), workspace.buffer.data_ptr(),
                                    workspace.nbytes, _stream()))
    return out


def attention_decode_partial(shape: AttentionShape, q_raw, k_new, v_new, q_norm_w, k_norm_w,
                             cache: KvCache, seq_lens: torch.Tensor, max_seq_len: int,
                             kv_begin: int, kv_end: int, partial: torch.Tensor,
                             workspace: DecodeWorkspace) -> torch.Tensor:
    """KV-split decode step on keys [kv_begin, kv_end) held locally
    (apex_attn_decode_partial_bf16); partial f32 [B, Hq, D+2] = (o, m log2, l)."""
    B = seq_lens.numel()
    _check_decode(shape, q_raw, k_new, v_new, cache, seq_lens, B)
    _need(partial, torch.float32, "partial")
    if partial.numel() != B * shape.q_heads * (shape.head_dim + 2):
        raise ValueError("attention_decode_partial: partial must be [B, Hq, D+2]")
    lib = _native.load()
    check(lib.apex_attn_decode_partial_bf16(shape.c(), q_raw.data_ptr(), k_new.data_ptr(),
                                            v_new.data_ptr(), _ptr(q_norm_w), _ptr(k_norm_w),
                                            cache.k.data_ptr(), cache.v.data_ptr(), cache.capacity,
                                            seq_lens.data_ptr(), B, max_seq_len, kv_begin, kv_end,
                                            partial.data_ptr(), workspace.buffer.data_ptr(),
                                            workspace.nbytes, _stream()))
    return partial


def attention_decode_kvsplit(shape: AttentionShape, q_raw, k_new, v_new, q_norm_w, k_norm_w,
                             cache: KvCache, seq_lens: torch.Tensor, max_seq_len: int,
                             kv_begin: int, kv_end: int, exchange, out: torch.Tensor,
                             workspace: DecodeWorkspace) -> torch.Tensor:
    """KV-split decode step on keys [kv_begin, kv_end) held locally, merged with the other ranks
    inside the kernel through NVLink peer memory (apex_attn_decode_kvsplit_bf16); `exchange` is
    the _native.PeerExchange that apex_b200.dist.PeerExchangeBuffers built.  out [B,Hq,D] bf16
    holds the full result on every rank."""
    B = seq_lens.numel()
    _check_decode(shape, q_raw, k_new, v_new, cache, seq_lens, B)
    _need(out, torch.bfloat16, "out")
    lib = _native.load()
    check(lib.apex_attn_decode_kvsplit_bf16(shape.c(), q_raw.data_ptr(), k_new.data_ptr(),
                                            v_new.data_ptr(), _ptr(q_norm_w), _ptr(k_norm_w),
                                            cache.k.data_ptr(), cache.v.data_ptr(), cache.capacity,
                                            seq_lens.data_ptr(), B, max_seq_len, kv_begin, kv_end,
                                            ctypes.byref(exchange), out.data_ptr(),
                                            workspace.buffer.data_ptr(), workspace.nbytes, _stream()))
    return out


def kv_ring_store(linear: KvCache, ring: KvCache, length: int) -> KvCache:
    """Copy the last min(length, ring capacity) positions of a linear bf16 cache [B, Hkv, cap, D]
    into a ring cache [B, Hkv, R, D] (position p at slot p % R), apex_kv_ring_store."""
    for t, n in ((linear.k, "linear.k"), (linear.v, "linear.v"), (ring.k, "ring.k"), (ring.v, "ring.v")):
        _need(t, torch.bfloat16, n)
    B, H, _, D = linear.k.shape
    if ring.k.shape[0] != B or ring.k.shape[1] != H or ring.k.shape[3] != D:
        raise ValueError("kv_ring_store: ring must be [B, Hkv, R, D] like the linear cache")
    check(_native.load().apex_kv_ring_store(linear.k.data_ptr(), linear.v.data_ptr(), ring.k.data_ptr(),
                                            ring.v.data_ptr(), B, H, D, linear.capacity, ring.capacity, length,
                                            _stream()))
    return ring


def merge_partials(partials: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """LSE merge of partial sets [R, rows, D+2] f32 -> out [rows, D] bf16."""
    _need(partials, torch.float32, "partials")
    _need(out, torch.bfloat16, "out")
    R, rows, rec = partials.shape
    D = rec - 2
    if out.numel() != rows * D:
        raise ValueError("merge_partials: out must be [rows, D]")
    check(_native.load().apex_attn_merge_partials(partials.data_ptr(), R, rows, D, out.data_ptr(),
                                                  _stream()))
    return out


class PrefillWorkspace:
    def __init__(self, shape: AttentionShape, batch: int, tokens: int, device=None):
        lib = _native.load()
        self.nbytes = int(lib.apex_attn_prefill_workspace_bytes(shape.c(), batch, tokens))
        self.buffer = torch.empty(max(self.nbytes, 16), dtype=torch.uint8, device=device or "cuda")


def attention_prefill(shape: AttentionShape, q_raw, k_raw, v_raw, q_norm_w, k_norm_w,
                      cache: KvCache, pos0: int, out: torch.Tensor,
                      workspace: PrefillWorkspace) -> torch.Tensor:
    """Fused prefill (apex_attn_prefill_bf16): q_raw [B,T,Hq,D], k_raw/v_raw [B,T,Hkv,D] bf16;
    appends K/V at pos0.. of cache [B,Hkv,cap,D]; out [B,T,Hq,D] bf16."""
    B, T = q_raw.shape[0], q_raw.shape[1]
    Hq, Hkv, D = shape.q_heads, shape.kv_heads, shape.head_dim
    for t, n in ((q_raw, "q_raw"), (k_raw, "k_raw"), (v_raw, "v_raw"), (cache.k, "cache.k"),
                 (cache.v, "cache.v"), (out, "out")):
        _need(t, torch.bfloat16, n)
    if q_raw.numel() != B * T * Hq * D or k_raw.numel() != B * T * Hkv * D or \
            v_raw.numel() != B * T * Hkv * D or out.numel() != B * T * Hq * D:
        raise ValueError("attention_prefill: shape mismatch")
    if cache.k.numel() != B * Hkv * cache.capacity * D:
        raise ValueError("attention_prefill: caches must be [B, Hkv, capacity, D]")
    check(_native.load().apex_attn_prefill_bf16(shape.c(), q_raw.data_ptr(), k_raw.data_ptr(),
                                                v_raw.data_ptr(), _ptr(q_norm_w), _ptr(k_norm_w),
                                                cache.k.data_ptr(), cache.v.data_ptr(),
                                                cache.capacity, B, T, pos0, out.data_ptr(),
                                                workspace.buffer.data_ptr(), workspace.nbytes,
                                                _stream()))
    return out


def attention_prefill_prep(shape: AttentionShape, q_raw, k_raw, v_raw, q_norm_w, k_norm_w,
                           cache: KvCache, pos0: int, workspace: "PrefillWorkspace") -> None:
    """First stage of attention_prefill (apex_attn_prefill_prep_bf16): norm + RoPE, K/V
    appended to the cache, normalised q into the workspace."""
    B, T = q_raw.shape[0], q_raw.shape[1]
    check(_native.load().apex_attn_prefill_prep_bf16(shape.c(), q_raw.data_ptr(), k_raw.data_ptr(),
                                                     v_raw.data_ptr(), _ptr(q_norm_w), _ptr(k_norm_w),
                                                     cache.k.data_ptr(), cache.v.data_ptr(),
                                                     cache.capacity, B, T, pos0, workspace.buffer.data_ptr(),
                                                     workspace.nbytes, _stream()))


def attention_prefill_attend(shape: AttentionShape, workspace: "PrefillWorkspace", cache: KvCache,
                             batch: int, tokens: int, pos0: int, out: torch.Tensor) -> None:
    """Second stage of attention_prefill (apex_attn_prefill_attend_bf16): tcgen05 attention of
    the workspace's normalised q over cache positions [0, pos0 + T) -> out [B, T, Hq, D]."""
    check(_native.load().apex_attn_prefill_attend_bf16(shape.c(), workspace.buffer.data_ptr(), workspace.nbytes,
                                                       cache.k.data_ptr(), cache.v.data_ptr(), cache.capacity,
                                                       batch, tokens, pos0, out.data_ptr(), _stream()))


def device_status() -> None:
    """Raise if a kernel's bounded wait gave up or it skipped an out-of-bounds length."""
    check(_native.load().apex_cuda_device_status(_stream()))


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)


# ---------------------------------------------------------------------------- projections and norm

@dataclass
class Nvfp4Matrix:
    """The reference's Nvfp4Matrix (src/ops.h:8-16): codes uint32 [w_rows, hidden_dim/8] and E4M3
    scales uint8 [w_rows, hidden_dim/16], as CUDA tensors (views into one weight buffer work)."""
    codes: torch.Tensor
    scales: torch.Tensor

    @property
    def w_rows(self) -> int:
        return self.codes.shape[0]

    @property
    def hidden_dim(self) -> int:
        return self.codes.shape[1] * 8


def _check_matrix(W: Nvfp4Matrix):
    if W.codes.dtype not in (torch.int32, torch.uint32) or W.scales.dtype != torch.uint8:
        raise TypeError("Nvfp4Matrix: codes int32/uint32, scales uint8")
    if W.scales.shape[0] != W.w_rows or W.scales.shape[1] * 16 != W.hidden_dim:
        raise ValueError("Nvfp4Matrix: scales must be [w_rows, hidden_dim/16]")
    for t in (W.codes, W.scales):
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError("Nvfp4Matrix: CUDA, contiguous tensors")


def matmul_nvfp4(input: torch.Tensor, W: Nvfp4Matrix, output: torch.Tensor, tokens: int) -> torch.Tensor:
    """apex::matmulNvfp4 (src/ops.h:34-46): output[t] = W . input[t].  input [tokens, hidden_dim] f32
    or bf16; output [tokens, w_rows] f32 or bf16."""
    _check_matrix(W)
    if input.dtype not in (torch.float32, torch.bfloat16) or output.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("matmul_nvfp4: input and output float32 or bfloat16")
    if input.numel() != tokens * W.hidden_dim or output.numel() != tokens * W.w_rows:
        raise ValueError("matmul_nvfp4: input [tokens, hidden_dim], output [tokens, w_rows]")
    check(_native.load().apex_matmul_nvfp4(ctypes_ptr(input), int(input.dtype == torch.bfloat16), W.codes.data_ptr(),
                                           W.scales.data_ptr(), ctypes_ptr(output), int(output.dtype == torch.bfloat16),
                                           W.hidden_dim, W.w_rows, tokens, _stream()))
    return output


def matmul_nvfp4_multi(input: torch.Tensor, Ws, outputs, tokens: int):
    """Up to four matmul_nvfp4 of the same input in one launch (q, k and v of a layer): outputs[m]
    [tokens, Ws[m].w_rows] = Ws[m] . input[t], all outputs of one dtype (float32 or bfloat16)."""
    Ws, outputs = list(Ws), list(outputs)
    if not 1 <= len(Ws) <= 4 or len(outputs) != len(Ws):
        raise ValueError("matmul_nvfp4_multi: one to four matrices, one output each")
    if input.dtype not in (torch.float32, torch.bfloat16):
        raise TypeError("matmul_nvfp4_multi: input float32 or bfloat16")
    out_dtype = outputs[0].dtype
    if out_dtype not in (torch.float32, torch.bfloat16) or any(o.dtype != out_dtype for o in outputs):
        raise TypeError("matmul_nvfp4_multi: outputs all float32 or all bfloat16")
    n = Ws[0].hidden_dim
    for W, o in zip(Ws, outputs):
        _check_matrix(W)
        if W.hidden_dim != n or o.numel() != tokens * W.w_rows:
            raise ValueError("matmul_nvfp4_multi: same hidden_dim for every matrix, outputs [tokens, w_rows]")
    if input.numel() != tokens * n:
        raise ValueError("matmul_nvfp4_multi: input [tokens, hidden_dim]")
    k = len(Ws)
    codes = (ctypes.c_void_p * k)(*[W.codes.data_ptr() for W in Ws])
    scales = (ctypes.c_void_p * k)(*[W.scales.data_ptr() for W in Ws])
    outs = (ctypes.c_void_p * k)(*[ctypes_ptr(o) for o in outputs])
    rows = (ctypes.c_uint32 * k)(*[W.w_rows for W in Ws])
    check(_native.load().apex_matmul_nvfp4_multi(ctypes_ptr(input), int(input.dtype == torch.bfloat16), k, codes,
                                                 scales, outs, rows, int(out_dtype == torch.bfloat16), n, tokens,
                                                 _stream()))
    return outputs


def rms_norm(input: torch.Tensor, weights: torch.Tensor, result: torch.Tensor, rows: int, hidden_dim: int,
             eps: float) -> torch.Tensor:
    """apex::rmsNorm (src/ops.h:18-27): f32 rows [rows, hidden_dim], weights bf16 [hidden_dim]."""
    _need(input, torch.float32, "input")
    _need(result, torch.float32, "result")
    if input.numel() != rows * hidden_dim or result.numel() != rows * hidden_dim or weights.numel() != hidden_dim:
        raise ValueError("rms_norm: shape mismatch")
    check(_native.load().apex_rms_norm_f32(input.data_ptr(), weights.data_ptr(), result.data_ptr(), rows, hidden_dim,
                                           eps, _stream()))
    return result


class ProjNormWorkspace:
    """Device workspace of matmul_nvfp4_rms_norm for up to `tokens` tokens of a w_rows-row matrix."""

    def __init__(self, w_rows: int, tokens: int, device=None):
        lib = _native.load()
        self.nbytes = int(lib.apex_matmul_nvfp4_rms_norm_workspace_bytes(w_rows, tokens))
        self.buffer = torch.zeros(self.nbytes, dtype=torch.uint8, device=device or "cuda")


def matmul_nvfp4_rms_norm(input: torch.Tensor, W: Nvfp4Matrix, norm_weight: torch.Tensor, output: torch.Tensor,
                          tokens: int, eps: float, workspace: ProjNormWorkspace, residual=None,
                          residual_out=None) -> torch.Tensor:
    """o_proj followed by the post-attention RMSNorm, fused (apex_matmul_nvfp4_rms_norm): output[t] =
    rmsnorm(W . input[t], norm_weight); residual_out[t] = residual[t] + output[t] when given."""
    _check_matrix(W)
    _need(output, torch.float32, "output")
    if input.numel() != tokens * W.hidden_dim or output.numel() != tokens * W.w_rows:
        raise ValueError("matmul_nvfp4_rms_norm: input [tokens, hidden_dim], output [tokens, w_rows]")
    check(_native.load().apex_matmul_nvfp4_rms_norm(
        ctypes_ptr(input), int(input.dtype == torch.bfloat16), W.codes.data_ptr(), W.scales.data_ptr(),
        norm_weight.data_ptr(), _ptr(residual), ctypes_ptr(output), _ptr(residual_out), W.hidden_dim, W.w_rows, tokens,
        eps, workspace.buffer.data_ptr(), workspace.nbytes, _stream()))
    return output
