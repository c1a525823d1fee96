"""GPU test of apex_attn_decode_bf16_noalloc, the decode entry point for callers that cannot
allocate device memory (an engine that keeps all device memory under its own fixed budget, or
a decode loop that cannot take cudaMalloc's implicit synchronisation).  It must give the same
result as apex_attn_decode_bf16 with a caller-provided workspace, also on the second of two
calls in a row, since every call reuses the same static scratch array.

Named test_zz_* so pytest collects it last; it builds all of its own inputs, so it also passes
alone in a fresh process."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from apex_b200 import _native, ops

pytestmark = pytest.mark.gpu

TOL_MAX, TOL_MEAN = 2e-2, 2e-3   # the parity tolerance of the other tests


def _case(seed, lens, cap):
    g = torch.Generator(device="cuda").manual_seed(seed)
    B, Hq, Hkv, D = len(lens), 16, 8, 256

    def r(*s, scale=1.0, mean=0.0):
        return (torch.randn(*s, generator=g, device="cuda") * scale + mean).to(torch.bfloat16)

    return dict(q=r(B, Hq, D), k=r(B, Hkv, D), v=r(B, Hkv, D), qw=r(D, scale=0.1, mean=1.0),
                kw=r(D, scale=0.1, mean=1.0), kc=r(B, Hkv, cap, D), vc=r(B, Hkv, cap, D),
                lens=torch.tensor(lens, dtype=torch.int32, device="cuda"), cap=cap, max_len=max(lens))


def _with_workspace(shape, c):
    cache = ops.KvCache(c["kc"].clone(), c["vc"].clone())
    out = torch.empty_like(c["q"])
    ws = ops.DecodeWorkspace(shape, c["lens"].numel(), c["max_len"])
    ops.attention_decode(shape, c["q"], c["k"], c["v"], c["qw"], c["kw"], cache, c["lens"], c["max_len"], out, ws)
    return out


def _no_alloc(shape, c):
    lib = _native.load()
    cache_k, cache_v = c["kc"].clone(), c["vc"].clone()
    out = torch.empty_like(c["q"])
    p = shape.c()
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]      # cudaMemGetInfo around the call alone
    rc = lib.apex_attn_decode_bf16_noalloc(
        ctypes.byref(p), c["q"].data_ptr(), c["k"].data_ptr(), c["v"].data_ptr(), c["qw"].data_ptr(),
        c["kw"].data_ptr(), cache_k.data_ptr(), cache_v.data_ptr(), c["cap"], c["lens"].data_ptr(),
        c["lens"].numel(), c["max_len"], out.data_ptr(), torch.cuda.current_stream().cuda_stream)
    _native.check(rc)
    torch.cuda.synchronize()
    return out, cache_k, free_before - torch.cuda.mem_get_info()[0]


def _close(a, b):
    e = (a.float() - b.float()).abs()
    assert torch.isfinite(a.float()).all()
    assert e.max().item() <= TOL_MAX and e.mean().item() <= TOL_MEAN, (e.max().item(), e.mean().item())


def test_no_alloc_decode_matches_workspace_decode_on_two_calls_in_a_row():
    shape = ops.AttentionShape(16, 8, 256, 128, 1e6, 0, 1 / 16, 1e-6, True, False)
    first = _case(61, [5000, 513, 8192, 77, 3001], 8192)
    second = _case(62, [1024, 1], 1024)                 # different shape: stale scratch must not leak
    for i, c in enumerate((first, second)):
        want = _with_workspace(shape, c)
        got, cache_k, allocated = _no_alloc(shape, c)
        _close(got, want)
        if i == 1:
            # the first call may load the library's device code (and with it the static array);
            # the second must not change the device's free memory at all
            assert allocated == 0, f"device free memory changed by {allocated} bytes"
        # the new token's key was appended at position seq_lens[b]-1, as the workspace path does
        L = int(c["lens"][0].item())
        assert not torch.equal(cache_k[0, :, L - 1], c["kc"][0, :, L - 1])
    ops.device_status()


def test_no_alloc_decode_rejects_requests_beyond_its_scratch():
    shape = ops.AttentionShape(16, 8, 256, 128, 1e6, 0, 1 / 16, 1e-6, True, False)
    lib = _native.load()
    p = shape.c()
    fake = 0x1000
    # 1024 sequences of up to 131072 keys need far more than the static scratch holds
    rc = lib.apex_attn_decode_bf16_noalloc(ctypes.byref(p), fake, fake, fake, None, None, fake, fake, 131072,
                                           fake, 1024, 131072, fake, None)
    assert rc == _native.APEX_ERR_WORKSPACE
    assert b"static scratch" in lib.apex_cuda_last_error()


def test_no_alloc_decode_rejected_call_queues_nothing():
    """A call rejected for a bad argument (here a misaligned cache pointer) returns before it
    queues anything, so a stream capture around it records no node."""
    shape = ops.AttentionShape(16, 8, 256, 128, 1e6, 0, 1 / 16, 1e-6, True, False)
    c = _case(63, [100], 128)
    _no_alloc(shape, c)  # the first call on a device comes before any capture
    lib = _native.load()
    p = shape.c()
    out = torch.empty_like(c["q"])
    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        rc = lib.apex_attn_decode_bf16_noalloc(
            ctypes.byref(p), c["q"].data_ptr(), c["k"].data_ptr(), c["v"].data_ptr(), c["qw"].data_ptr(),
            c["kw"].data_ptr(), c["kc"].data_ptr() + 2, c["vc"].data_ptr(), c["cap"], c["lens"].data_ptr(), 1,
            c["max_len"], out.data_ptr(), stream.cuda_stream)
    assert rc == _native.APEX_ERR_INVALID_ARGUMENT
    assert b"aligned" in lib.apex_cuda_last_error()
    del g
