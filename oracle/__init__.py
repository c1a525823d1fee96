"""CPU oracle for the attention hot path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` (as the checker) and ``bench.py``'s
``cpu_baseline`` / ``--impl reference`` legs may import this package.  The product
(``apex_b200``) never does.

Two libraries sit behind this module:

* ``liboracle.so`` -- the C restatement in ``apex_oracle.c`` (always built);
* ``libapexref.so`` -- the reference's own CPU code (``src/tests/cpu_ref.h`` and the
  ``ropeCpu`` / ``attentionRowCpu`` block of ``docs/B6_3_attention.md`` section 5),
  compiled in place by ``oracle/build.py`` when the reference tree is present.

Inputs are numpy arrays: f32 arrays for activations (holding bf16 values for the bf16
configurations) and uint16 arrays for bf16 norm weights, as in the reference.
"""
from __future__ import annotations

import ctypes
import math
import pathlib

import numpy as np

from . import build as _build

_F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_U16P = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
_I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_U32P = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_U8P = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u32, _f32, _i, _sz, _u64 = ctypes.c_uint32, ctypes.c_float, ctypes.c_int, ctypes.c_size_t, ctypes.c_uint64

_lib = None
_ref = None


def _nullable(ptype):
    """ndpointer that also accepts None (passed as NULL)."""
    class _P(ptype):
        @classmethod
        def from_param(cls, obj):
            if obj is None:
                return None
            return super().from_param(obj)
    return _P


_U16P_N = _nullable(_U16P)
_I32P_N = _nullable(_I32P)


def lib():
    """The restatement (liboracle.so), built on first use."""
    global _lib
    if _lib is None:
        path = _build.build_oracle()
        L = ctypes.CDLL(str(path))
        L.orc_fill_normal_bf16.argtypes = [_U16P, _sz, _u64, _u64, _u64, _f32, _f32]
        L.orc_fill_uniform_int.argtypes = [_I32P, _sz, _u64, _u64, ctypes.c_int32, ctypes.c_int32]
        L.orc_rms_norm.argtypes = [_F32P, _U16P_N, _F32P, _sz, _f32]
        L.orc_rope.argtypes = [_F32P, _sz, _sz, _f32, _u32]
        L.orc_head_norm_rope_f32.argtypes = [_F32P, _U16P_N, _F32P] + [_u32] * 5 + [_f32] + [_u32] * 3 + [_f32]
        L.orc_attention_row.argtypes = [_F32P, _F32P, _F32P, _F32P, _sz, _sz, _sz, ctypes.c_double]
        L.orc_attention_f32.argtypes = [_F32P] * 4 + [_u32] * 7 + [_f32]
        L.orc_kv_append.argtypes = [_F32P, _U16P_N, _i, _u32, _f32, _f32, _F32P] + [_u32] * 5 + [_i]
        L.orc_prefill.argtypes = ([_F32P] * 3 + [_U16P_N, _U16P_N, _i, _i, _u32, _f32, _f32, _f32, _u32,
                                  _F32P, _F32P] + [_u32] * 6 + [_I32P_N, _u32, _F32P, _i])
        L.orc_decode.argtypes = ([_F32P] * 3 + [_U16P_N, _U16P_N, _i, _i, _u32, _f32, _f32, _f32, _u32,
                                 _F32P, _F32P, _u32, _I32P] + [_u32] * 4 + [_F32P, _i])
        L.orc_partial_row.argtypes = [_F32P, _F32P, _F32P, _sz, _sz, _sz, ctypes.c_double, _F32P]
        L.orc_merge_partials.argtypes = [_F32P, _u32, _sz, _F32P]
        L.orc_matvec_nvfp4.argtypes = [_U32P, _U8P, _F32P, _F32P, _sz, _sz, _sz]
        L.orc_rms_norm_rows.argtypes = [_F32P, _U16P_N, _F32P, _sz, _sz, _f32]
        L.orc_fill_u32.argtypes = [_U32P, _sz, _u64, _u64]
        L.orc_e2m1.argtypes = [_u32]
        L.orc_e2m1.restype = _f32
        L.orc_e4m3.argtypes = [ctypes.c_uint8]
        L.orc_e4m3.restype = _f32
        L.orc_set_threads.argtypes = [_i]
        L.orc_max_threads.restype = _i
        _lib = L
    return _lib


def ref_lib():
    """The reference's own CPU code (libapexref.so), or None when it was never built."""
    global _ref
    if _ref is None:
        path = _build.build_reference()
        if path is None or not pathlib.Path(path).exists():
            return None
        R = ctypes.CDLL(str(path))
        R.ref_rms_norm.argtypes = [_F32P, _U16P_N, _F32P, _sz, _f32]
        R.ref_rope.argtypes = [_F32P, _sz, _sz, _f32, _u32]
        R.ref_attention_row.argtypes = [_F32P, _F32P, _F32P, _F32P, _sz, _sz, _sz]
        R.ref_diff.argtypes = [_F32P, _F32P, _sz, ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_double)]
        R.ref_head_norm_rope_f32.argtypes = [_F32P, _U16P_N, _F32P] + [_u32] * 5 + [_f32] + [_u32] * 3 + [_f32]
        R.ref_attention.argtypes = [_F32P] * 4 + [_u32] * 7 + [_f32, _I32P_N, _u32]
        R.ref_matvec_nvfp4.argtypes = [_U32P, _U8P, _F32P, _F32P, _sz, _sz, _sz]
        R.ref_rms_norm_rows.argtypes = [_F32P, _U16P_N, _F32P, _sz, _sz, _f32]
        _ref = R
    return _ref


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))
    try:
        import os
        os.environ["OMP_NUM_THREADS"] = str(n)
    except Exception:
        pass


def max_threads() -> int:
    return int(lib().orc_max_threads())


# ------------------------------------------------------------------ bf16 helpers (numpy)

def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round to nearest even (finite inputs)."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    b = b + np.uint32(0x7FFF) + ((b >> 16) & np.uint32(1))
    return (b >> 16).astype(np.uint16)


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(x))


# ------------------------------------------------------------------ synthetic inputs

def normal_bf16(n: int, seed: int, stream: int, offset: int = 0, mean: float = 0.0,
                std: float = 1.0) -> np.ndarray:
    out = np.empty(int(n), dtype=np.uint16)
    lib().orc_fill_normal_bf16(out, out.size, seed, stream, offset, mean, std)
    return out


def uniform_int(n: int, seed: int, stream: int, lo: int, hi: int) -> np.ndarray:
    out = np.empty(int(n), dtype=np.int32)
    lib().orc_fill_uniform_int(out, out.size, seed, stream, lo, hi)
    return out


# ------------------------------------------------------------------ restatement wrappers

def _c(a, dtype=np.float32):
    return np.ascontiguousarray(a, dtype=dtype)


def head_norm_rope_f32(inp, weight, out, tokens, heads, head_dim, has_weight, rope_pairs,
                       rope_base, abs_pos, out_token_stride, out_head_stride, eps, *, ref=False):
    """In-out on ``out`` (a flat f32 array), like the reference kernel."""
    L = ref_lib() if ref else lib()
    fn = L.ref_head_norm_rope_f32 if ref else L.orc_head_norm_rope_f32
    fn(_c(inp).ravel(), None if weight is None else _c(weight, np.uint16), out, tokens, heads,
       head_dim, int(has_weight), rope_pairs, rope_base, abs_pos, out_token_stride,
       out_head_stride, eps)
    return out


def attention_f32(q, K, V, tokens, q_heads, kv_heads, head_dim, capacity, pos0, window,
                  scale=1.0, *, ref=False, rows=None):
    q, K, V = _c(q).ravel(), _c(K).ravel(), _c(V).ravel()
    if ref:
        n_rows = tokens if rows is None else len(rows)
        out = np.zeros(n_rows * q_heads * head_dim, np.float32)
        ref_lib().ref_attention(q, K, V, out, tokens, q_heads, kv_heads, head_dim, capacity,
                                pos0, window, scale, None if rows is None else _c(rows, np.int32),
                                n_rows)
        return out
    if rows is not None:
        raise ValueError("rows is only supported by the reference shim")
    out = np.zeros(tokens * q_heads * head_dim, np.float32)
    lib().orc_attention_f32(q, K, V, out, tokens, q_heads, kv_heads, head_dim, capacity, pos0,
                            window, scale)
    return out


def kv_append(raw, w, norm, rope_pairs, rope_base, eps, cache, cap, pos0, T, H, D, round_bf16=0):
    lib().orc_kv_append(_c(raw).ravel(), None if w is None else _c(w, np.uint16), int(norm),
                        rope_pairs, rope_base, eps, cache, cap, pos0, T, H, D, int(round_bf16))


def prefill(q_raw, k_raw, v_raw, q_w, k_w, *, qk_norm, v_norm, rope_pairs, rope_base, eps, scale,
            window, Kc, Vc, cap, pos0, T, Hq, Hkv, D, rows=None, round_bf16=0):
    """One sequence; returns [n_rows, Hq, D]; appends K/V into Kc/Vc ([Hkv][cap][D], flat)."""
    n_rows = T if rows is None else len(rows)
    out = np.zeros(n_rows * Hq * D, np.float32)
    lib().orc_prefill(_c(q_raw).ravel(), _c(k_raw).ravel(), _c(v_raw).ravel(),
                      None if q_w is None else _c(q_w, np.uint16),
                      None if k_w is None else _c(k_w, np.uint16), int(qk_norm), int(v_norm),
                      rope_pairs, rope_base, eps, scale, window, Kc, Vc, cap, pos0, T, Hq, Hkv, D,
                      None if rows is None else _c(rows, np.int32), n_rows, out, int(round_bf16))
    return out.reshape(n_rows, Hq, D)


def decode(q_raw, k_new, v_new, q_w, k_w, *, qk_norm, v_norm, rope_pairs, rope_base, eps, scale,
           window, Kc, Vc, cap, lens, B, Hq, Hkv, D, round_bf16=0):
    out = np.zeros(B * Hq * D, np.float32)
    lib().orc_decode(_c(q_raw).ravel(), _c(k_new).ravel(), _c(v_new).ravel(),
                     None if q_w is None else _c(q_w, np.uint16),
                     None if k_w is None else _c(k_w, np.uint16), int(qk_norm), int(v_norm),
                     rope_pairs, rope_base, eps, scale, window, Kc, Vc, cap, _c(lens, np.int32),
                     B, Hq, Hkv, D, out, int(round_bf16))
    return out.reshape(B, Hq, D)


def partial_row(q, K, V, D, lo, hi, scale):
    out = np.zeros(D + 2, np.float32)
    lib().orc_partial_row(_c(q).ravel(), _c(K).ravel(), _c(V).ravel(), D, lo, hi, scale, out)
    return out


def merge_partials(parts, D):
    parts = _c(parts).reshape(-1, D + 2)
    out = np.zeros(D, np.float32)
    lib().orc_merge_partials(parts.ravel(), parts.shape[0], D, out)
    return out


def diff(a, b):
    """max |a-b| and rel-L2 (src/tests/cpu_ref.h:28-46 semantics); inf on non-finite."""
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    if not (np.isfinite(a).all() and np.isfinite(b).all()):
        return math.inf, math.inf
    e = a - b
    den = float(np.dot(b, b))
    num = float(np.dot(e, e))
    return float(np.abs(e).max(initial=0.0)), math.sqrt(num / den) if den > 0 else math.sqrt(num)


# ------------------------------------------------------------------ NVFP4 projections, RMSNorm rows

def fill_u32(n: int, seed: int, stream: int) -> np.ndarray:
    out = np.empty(int(n), dtype=np.uint32)
    lib().orc_fill_u32(out, out.size, seed, stream)
    return out


def nvfp4_matrix(rows: int, n: int, seed: int, scale_lo: int = 0x20, scale_hi: int = 0x40):
    """Synthetic NVFP4 matrix [rows][n]: uniform codes and E4M3 scales in [scale_lo, scale_hi]
    (positive, finite; 0x20..0x40 is 2^-3 .. 2)."""
    codes = fill_u32(rows * n // 8, seed, 7).reshape(rows, n // 8)
    scales = uniform_int(rows * n // 16, seed, 8, scale_lo, scale_hi).astype(np.uint8).reshape(rows, n // 16)
    return codes, scales


def matvec_nvfp4(codes, scales, inp, tokens, rows, n, *, ref=False):
    out = np.zeros(tokens * rows, np.float32)
    L = ref_lib() if ref else lib()
    fn = L.ref_matvec_nvfp4 if ref else L.orc_matvec_nvfp4
    fn(_c(codes, np.uint32).ravel(), _c(scales, np.uint8).ravel(), _c(inp).ravel(), out, tokens, rows, n)
    return out.reshape(tokens, rows)


def rms_norm_rows(inp, w, rows, n, eps, *, ref=False):
    out = np.zeros(rows * n, np.float32)
    L = ref_lib() if ref else lib()
    fn = L.ref_rms_norm_rows if ref else L.orc_rms_norm_rows
    fn(_c(inp).ravel(), None if w is None else _c(w, np.uint16), out, rows, n, eps)
    return out.reshape(rows, n)
