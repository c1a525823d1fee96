"""ctypes binding of the C ABI in include/apex_cuda.h (apex_b200/lib/libapex_cuda.so).

The library is the only compute path: if it is missing, or a call fails, this module raises
(there is no fallback).  Build it with ``python -m apex_b200.build``.
"""
from __future__ import annotations

import ctypes
import pathlib

LIB_PATH = pathlib.Path(__file__).resolve().parent / "lib" / "libapex_cuda.so"

APEX_OK = 0
APEX_ERR_INVALID_ARGUMENT = 1
APEX_ERR_UNSUPPORTED = 2
APEX_ERR_CUDA = 3
APEX_ERR_WORKSPACE = 4
APEX_ERR_DEVICE_TIMEOUT = 5
APEX_ERR_FORMAT = 6

_ERR_NAMES = {1: "invalid argument", 2: "unsupported", 3: "CUDA error", 4: "workspace", 5: "device timeout",
              6: "format"}

# Every entry point declared in include/apex_cuda.h.
EXPORTED = (
    "apex_cuda_last_error", "apex_cuda_abi_version", "apex_cuda_device_status",
    "apex_head_norm_rope_f32", "apex_attention_f32", "apex_attention_f32_scaled",
    "apex_head_norm_rope_bf16", "apex_attn_decode_workspace_bytes",
    "apex_attn_decode_workspace_init", "apex_attn_decode_bf16", "apex_attn_decode_partial_bf16",
    "apex_attn_merge_partials", "apex_attn_prefill_workspace_bytes", "apex_attn_prefill_bf16",
    "apex_attn_prefill_prep_bf16", "apex_attn_prefill_attend_bf16", "apex_attn_decode_bf16_noalloc",
    "apex_attn_peer_exchange_bytes", "apex_attn_decode_kvsplit_bf16", "apex_device_alloc",
    "apex_device_free", "apex_ipc_get_handle", "apex_ipc_open_handle", "apex_ipc_close_handle",
    "apex_kv_ring_store", "apex_matmul_nvfp4_f32", "apex_matmul_nvfp4", "apex_matmul_nvfp4_multi", "apex_rms_norm_f32", "apex_matmul_nvfp4_rms_norm_workspace_bytes",
    "apex_matmul_nvfp4_rms_norm",
    # include/apex_loader.h
    "apex_model_open", "apex_model_close", "apex_model_summary_get", "apex_model_tensor", "apex_model_expert_piece",
    "apex_model_verify", "apex_model_upload_core", "apex_model_load_expert",
)


class ApexError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(f"[{_ERR_NAMES.get(code, code)}] {message}")
        self.code = code


class AttnParams(ctypes.Structure):
    """apex_attn_params (include/apex_cuda.h)."""
    _fields_ = [("q_heads", ctypes.c_uint32), ("kv_heads", ctypes.c_uint32),
                ("head_dim", ctypes.c_uint32), ("rope_pairs", ctypes.c_uint32),
                ("rope_base", ctypes.c_float), ("window", ctypes.c_uint32),
                ("scale", ctypes.c_float), ("eps", ctypes.c_float),
                ("qk_norm", ctypes.c_uint32), ("v_norm", ctypes.c_uint32), ("ring", ctypes.c_uint32)]


MAX_PEERS = 8


class PeerExchange(ctypes.Structure):
    """apex_peer_exchange (include/apex_cuda.h): every rank's exchange buffers as mapped here."""
    _fields_ = [("rank", ctypes.c_uint32), ("world", ctypes.c_uint32),
                ("gather", ctypes.c_void_p * MAX_PEERS), ("flags", ctypes.c_void_p * MAX_PEERS),
                ("seq", ctypes.c_void_p), ("wait_ns", ctypes.c_uint64)]


class ModelSummary(ctypes.Structure):
    """apex_model_summary (include/apex_loader.h)."""
    _fields_ = [("core_size", ctypes.c_uint64), ("alignment", ctypes.c_uint64), ("expert_slot_size", ctypes.c_uint64)] + \
        [(n, ctypes.c_uint32) for n in ("core_tensors", "layer_files", "num_hidden_layers", "hidden_size",
                                        "num_attention_heads", "num_key_value_heads", "head_dim", "global_head_dim",
                                        "num_global_key_value_heads", "sliding_window", "num_experts",
                                        "quant_group_size", "quant_bits")] + \
        [(n, ctypes.c_float) for n in ("rms_norm_eps", "rope_theta_sliding", "rope_theta_full",
                                       "partial_rotary_factor_full")]


_lib = None
_vp, _u32, _f32, _sz, _i32 = ctypes.c_void_p, ctypes.c_uint32, ctypes.c_float, ctypes.c_size_t, ctypes.c_int
_PP = ctypes.POINTER(AttnParams)
_PX = ctypes.POINTER(PeerExchange)
_PSZ = ctypes.POINTER(ctypes.c_size_t)


def load(path: str | pathlib.Path | None = None):
    """Load (once) and return the native library; raises if it was never built."""
    global _lib
    if _lib is not None:
        return _lib
    p = pathlib.Path(path) if path else LIB_PATH
    if not p.exists():
        raise ImportError(f"apex_b200 native library not built: {p} (run python -m apex_b200.build)")
    L = ctypes.CDLL(str(p))
    L.apex_cuda_last_error.restype = ctypes.c_char_p
    L.apex_cuda_abi_version.restype = _i32
    L.apex_cuda_device_status.argtypes = [_vp]
    L.apex_head_norm_rope_f32.argtypes = [_vp, _vp, _vp] + [_u32] * 5 + [_f32] + [_u32] * 3 + [_f32, _vp]
    L.apex_head_norm_rope_bf16.argtypes = L.apex_head_norm_rope_f32.argtypes
    L.apex_attention_f32.argtypes = [_vp] * 4 + [_u32] * 7 + [_vp]
    L.apex_attention_f32_scaled.argtypes = [_vp] * 4 + [_u32] * 7 + [_f32, _vp]
    L.apex_attn_decode_workspace_bytes.argtypes = [_PP, _u32, _u32]
    L.apex_attn_decode_workspace_bytes.restype = _sz
    L.apex_attn_decode_workspace_init.argtypes = [_vp, _sz, _vp]
    L.apex_attn_decode_bf16.argtypes = ([_PP] + [_vp] * 7 + [_u32, _vp, _u32, _u32, _vp, _vp, _sz, _vp])
    L.apex_attn_decode_bf16_noalloc.argtypes = ([_PP] + [_vp] * 7 + [_u32, _vp, _u32, _u32, _vp, _vp])
    L.apex_attn_decode_partial_bf16.argtypes = ([_PP] + [_vp] * 7 + [_u32, _vp, _u32, _u32, _u32, _u32,
                                                                       _vp, _vp, _sz, _vp])
    L.apex_attn_merge_partials.argtypes = [_vp, _u32, _u32, _u32, _vp, _vp]
    L.apex_attn_peer_exchange_bytes.argtypes = [_PP, _u32, _u32, _PSZ, _PSZ, _PSZ]
    L.apex_attn_decode_kvsplit_bf16.argtypes = ([_PP] + [_vp] * 7 + [_u32, _vp, _u32, _u32, _u32, _u32, _PX,
                                                                       _vp, _vp, _sz, _vp])
    L.apex_device_alloc.argtypes = [_sz, ctypes.POINTER(_vp)]
    L.apex_device_free.argtypes = [_vp]
    L.apex_ipc_get_handle.argtypes = [_vp, _vp]
    L.apex_ipc_open_handle.argtypes = [_vp, ctypes.POINTER(_vp)]
    L.apex_ipc_close_handle.argtypes = [_vp]
    L.apex_attn_prefill_workspace_bytes.argtypes = [_PP, _u32, _u32]
    L.apex_attn_prefill_workspace_bytes.restype = _sz
    L.apex_attn_prefill_bf16.argtypes = ([_PP] + [_vp] * 7 + [_u32, _u32, _u32, _u32, _vp, _vp, _sz, _vp])
    L.apex_attn_prefill_prep_bf16.argtypes = ([_PP] + [_vp] * 7 + [_u32, _u32, _u32, _u32, _vp, _sz, _vp])
    L.apex_attn_prefill_attend_bf16.argtypes = ([_PP, _vp, _sz, _vp, _vp] + [_u32, _u32, _u32, _u32, _vp, _vp])
    L.apex_kv_ring_store.argtypes = [_vp] * 4 + [_u32] * 6 + [_vp]
    L.apex_matmul_nvfp4_f32.argtypes = [_vp] * 4 + [_u32] * 3 + [_vp]
    L.apex_matmul_nvfp4.argtypes = [_vp, _i32, _vp, _vp, _vp, _i32, _u32, _u32, _u32, _vp]
    L.apex_matmul_nvfp4_multi.argtypes = [_vp, _i32, _u32, _vp, _vp, _vp, _vp, _i32, _u32, _u32, _vp]
    L.apex_rms_norm_f32.argtypes = [_vp, _vp, _vp, _u32, _u32, _f32, _vp]
    L.apex_matmul_nvfp4_rms_norm_workspace_bytes.argtypes = [_u32, _u32]
    L.apex_matmul_nvfp4_rms_norm_workspace_bytes.restype = _sz
    L.apex_matmul_nvfp4_rms_norm.argtypes = [_vp, _i32, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _f32, _vp, _sz,
                                             _vp]
    _PU64 = ctypes.POINTER(ctypes.c_uint64)
    L.apex_model_open.argtypes = [ctypes.c_char_p, ctypes.POINTER(_vp)]
    L.apex_model_close.argtypes = [_vp]
    L.apex_model_close.restype = None
    L.apex_model_summary_get.argtypes = [_vp, ctypes.POINTER(ModelSummary)]
    L.apex_model_tensor.argtypes = [_vp, ctypes.c_char_p, _PU64, _PU64]
    L.apex_model_expert_piece.argtypes = [_vp, ctypes.c_char_p, _PU64, _PU64]
    L.apex_model_verify.argtypes = [_vp]
    L.apex_model_upload_core.argtypes = [_vp, _vp, _sz, _i32, _vp, ctypes.POINTER(ctypes.c_double)]
    L.apex_model_load_expert.argtypes = [_vp, _u32, _u32, _vp, _sz, _i32, _vp]
    for fn in EXPORTED:
        if fn not in ("apex_cuda_last_error", "apex_attn_decode_workspace_bytes",
                      "apex_attn_prefill_workspace_bytes", "apex_model_close",
                      "apex_matmul_nvfp4_rms_norm_workspace_bytes"):
            getattr(L, fn).restype = _i32
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != APEX_OK:
        msg = load().apex_cuda_last_error()
        raise ApexError(rc, msg.decode() if msg else "")
