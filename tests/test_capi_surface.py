"""CPU tests of the C ABI library: it loads, exports every entry point include/*.h declares, and
rejects bad arguments before touching a GPU."""
from __future__ import annotations

import ctypes
import pathlib
import re
import subprocess

import pytest

from apex_b200 import _native
from apex_b200._native import AttnParams

ROOT = pathlib.Path(__file__).resolve().parents[1]
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared():
    names = set()
    for h in HEADERS:
        names |= set(re.findall(r"APEX_API\s+[\w\s\*]*?\b(apex_\w+)\s*\(", h.read_text()))
    return sorted(names)


def test_header_declares_what_the_binding_knows():
    assert declared() == sorted(_native.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    out = subprocess.run(["nm", "-D", "--defined-only", str(_native.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    syms = {line.split()[-1] for line in out.splitlines() if line.strip()}
    for name in declared():
        assert name in syms, name
        assert getattr(lib, name) is not None
    assert lib.apex_cuda_abi_version() == 103


def _params(**kw):
    base = dict(q_heads=16, kv_heads=8, head_dim=256, rope_pairs=128, rope_base=1e4, window=0,
                scale=1 / 16, eps=1e-6, qk_norm=1, v_norm=0)
    base.update(kw)
    return AttnParams(**base)


def test_workspace_sizes_are_host_computable():
    lib = _native.load()
    p = _params()
    # normalised q (bf16, head-major) + 256 bytes of scheduler state
    assert lib.apex_attn_prefill_workspace_bytes(ctypes.byref(p), 1, 2048) == 2048 * 16 * 256 * 2 + 256
    # head_dim 512 (the global layers): the normalised q alone
    g = _params(q_heads=16, kv_heads=2, head_dim=512, rope_pairs=64)
    assert lib.apex_attn_prefill_workspace_bytes(ctypes.byref(g), 2, 1000) == 2 * 16 * 1000 * 512 * 2
    small = lib.apex_attn_decode_workspace_bytes(ctypes.byref(p), 1, 1024)
    big = lib.apex_attn_decode_workspace_bytes(ctypes.byref(p), 64, 8192)
    assert 0 < small < big


def test_peer_exchange_sizes_follow_the_documented_layout():
    """gather [2][world][batch*q_heads][head_dim+2] 8-byte (step, value) words, flags
    [world][batch*kv_heads] and seq [batch*kv_heads] uint32; at most 8 ranks."""
    lib = _native.load()
    p = _params()
    sizes = [ctypes.c_size_t() for _ in range(3)]
    for batch, world in ((1, 1), (8, 2), (8, 8)):
        _native.check(lib.apex_attn_peer_exchange_bytes(ctypes.byref(p), batch, world, *map(ctypes.byref, sizes)))
        gather, flags, seq = (s.value for s in sizes)
        assert gather == 2 * world * batch * 16 * (256 + 2) * 8
        assert flags == world * batch * 8 * 4 and seq == batch * 8 * 4
        assert gather % 16 == 0  # every record starts on a 16-byte boundary (16-byte stores)
    assert lib.apex_attn_peer_exchange_bytes(ctypes.byref(p), 1, 9, *map(ctypes.byref, sizes)) == \
        _native.APEX_ERR_INVALID_ARGUMENT


@pytest.mark.parametrize("kw,code", [(dict(head_dim=128), _native.APEX_ERR_UNSUPPORTED),
                                     (dict(q_heads=12, kv_heads=8), _native.APEX_ERR_INVALID_ARGUMENT),
                                     (dict(rope_pairs=200), _native.APEX_ERR_INVALID_ARGUMENT),
                                     (dict(head_dim=512, rope_pairs=300), _native.APEX_ERR_INVALID_ARGUMENT),
                                     (dict(head_dim=512, rope_pairs=64, qk_norm=0), _native.APEX_ERR_UNSUPPORTED)])
def test_prefill_rejects_bad_params_without_gpu(kw, code):
    lib = _native.load()
    p = _params(**kw)
    rc = lib.apex_attn_prefill_bf16(ctypes.byref(p), *([None] * 7), 16, 1, 16, 0, None, None, 0, None)
    assert rc == code
    assert lib.apex_cuda_last_error()


def test_prefill_rejects_null_and_misaligned_tensors():
    lib = _native.load()
    p = _params()
    assert lib.apex_attn_prefill_bf16(ctypes.byref(p), *([None] * 7), 16, 1, 16, 0, None, None, 0,
                                      None) == _native.APEX_ERR_INVALID_ARGUMENT
    fake = 0x1000
    args = [fake + 2] + [fake] * 6
    rc = lib.apex_attn_prefill_bf16(ctypes.byref(p), *args, 16, 1, 16, 0, fake, fake, 1 << 30, None)
    assert rc == _native.APEX_ERR_INVALID_ARGUMENT
    assert b"aligned" in lib.apex_cuda_last_error()


def test_prefill_rejects_capacity_and_workspace_errors():
    lib = _native.load()
    p = _params()
    f = 0x1000
    # pos0 + tokens > capacity
    assert lib.apex_attn_prefill_bf16(ctypes.byref(p), f, f, f, None, None, f, f, 16, 1, 8, 9, f, f, 1 << 30,
                                      None) == _native.APEX_ERR_INVALID_ARGUMENT
    # workspace too small
    assert lib.apex_attn_prefill_bf16(ctypes.byref(p), f, f, f, None, None, f, f, 64, 1, 8, 0, f, f, 16,
                                      None) == _native.APEX_ERR_WORKSPACE


def test_decode_rejects_bad_shapes_without_gpu():
    lib = _native.load()
    f = 0x1000
    for kw in (dict(q_heads=32, kv_heads=2), dict(head_dim=128)):   # group 16, head_dim 128: not built
        p = _params(**kw)
        assert lib.apex_attn_decode_bf16(ctypes.byref(p), f, f, f, None, None, f, f, 1024, f, 1, 1024, f, f,
                                         1 << 30, None) == _native.APEX_ERR_UNSUPPORTED
    # the wide-group / head_dim 512 form checks its arguments before touching a GPU
    p = _params(q_heads=16, kv_heads=2, head_dim=512, rope_pairs=64)
    assert lib.apex_attn_decode_bf16(ctypes.byref(p), f, f, f, None, None, f, f, 512, f, 1, 1024, f, f, 1 << 30,
                                     None) == _native.APEX_ERR_INVALID_ARGUMENT   # max_seq_len > capacity
    assert lib.apex_attn_decode_bf16(ctypes.byref(p), f, f, f, None, None, f, f, 1024, f, 1, 1024, f, f, 64,
                                     None) == _native.APEX_ERR_WORKSPACE
    p = _params()
    # max_seq_len beyond capacity
    assert lib.apex_attn_decode_bf16(ctypes.byref(p), f, f, f, None, None, f, f, 512, f, 1, 1024, f, f, 1 << 30,
                                     None) == _native.APEX_ERR_INVALID_ARGUMENT
    # workspace too small
    assert lib.apex_attn_decode_bf16(ctypes.byref(p), f, f, f, None, None, f, f, 1024, f, 1, 1024, f, f, 8,
                                     None) == _native.APEX_ERR_WORKSPACE


def test_f32_dropins_reject_bad_head_dim():
    lib = _native.load()
    f = 0x1000
    assert lib.apex_head_norm_rope_f32(f, f, f, 1, 1, 1024, 1, 0, 1e4, 0, 1024, 1024, 1e-6,
                                       None) == _native.APEX_ERR_INVALID_ARGUMENT
    assert lib.apex_attention_f32(f, f, f, f, 1, 16, 8, 1024, 4, 0, 0, None) == _native.APEX_ERR_INVALID_ARGUMENT
    assert lib.apex_attention_f32(f, f, f, f, 4, 16, 8, 64, 4, 1, 0, None) == _native.APEX_ERR_INVALID_ARGUMENT


def test_ring_rejections():
    lib = _native.load()
    f = 0x1000
    import dataclasses
    from apex_b200 import ops
    base = ops.AttentionShape(16, 8, 256, 128, 1e4, 0, 1 / 16, 1e-6, True, False, True)
    for window, code in ((0, _native.APEX_ERR_INVALID_ARGUMENT), (2048, _native.APEX_ERR_INVALID_ARGUMENT)):
        p = dataclasses.replace(base, window=window).c()
        import ctypes
        assert lib.apex_attn_decode_bf16(ctypes.byref(p), f, f, f, None, None, f, f, 1024, f, 1, 9000, f, f, 1 << 30,
                                         None) == code
    p = dataclasses.replace(base, window=1024).c()
    import ctypes
    assert lib.apex_attn_decode_partial_bf16(ctypes.byref(p), f, f, f, None, None, f, f, 1024, f, 1, 9000, 0, 4096, f,
                                             f, 1 << 30, None) == _native.APEX_ERR_UNSUPPORTED
    assert lib.apex_attn_prefill_bf16(ctypes.byref(p), f, f, f, None, None, f, f, 1024, 1, 16, 0, f, f, 1 << 30,
                                      None) == _native.APEX_ERR_UNSUPPORTED
