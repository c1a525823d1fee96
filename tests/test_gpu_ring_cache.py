"""Ring KV caches for sliding layers (the reference's planned 1024-entry ring, position p at slot
p % 1024, docs/B6_3_attention.md:99-102): a decode over a ring equals the decode over the linear
cache holding the same keys, across the wrap, for window == ring size and window < ring size, step
after step; the new token lands in its slot; the ring is built from a linear (prefill) cache by
apex_kv_ring_store."""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from apex_b200 import _native, ops
from apex_b200.configs import CONFIGS
from helpers import assert_close, bf16_dev_to_f32, oracle_decode_seq
from test_gpu_decode import build_decode

pytestmark = pytest.mark.gpu
R = 1024


def _ring_of(t, lens, ring=R):
    B, Hkv, _, D = t["cache"].k.shape
    rc = ops.KvCache(torch.zeros(B, Hkv, ring, D, dtype=torch.bfloat16, device="cuda"),
                     torch.zeros(B, Hkv, ring, D, dtype=torch.bfloat16, device="cuda"))
    for b, L in enumerate(lens):  # sequence b's positions [L-1-ring, L-1) -> slots
        lin = ops.KvCache(t["cache"].k[b:b + 1].contiguous(), t["cache"].v[b:b + 1].contiguous())
        one = ops.KvCache(rc.k[b:b + 1].contiguous(), rc.v[b:b + 1].contiguous())
        ops.kv_ring_store(lin, one, L - 1)
        rc.k[b:b + 1] = one.k
        rc.v[b:b + 1] = one.v
    return rc


def _decode(shape, t, cache, lens, max_len):
    B = len(lens)
    out = torch.empty(B, shape.q_heads, shape.head_dim, dtype=torch.bfloat16, device="cuda")
    ws = ops.DecodeWorkspace(shape, B, max_len)
    ops.attention_decode(shape, t["q_raw"], t["k_new"], t["v_new"], t["qw"], t["kw"], cache, t["lens"], max_len, out, ws)
    ops.device_status()
    return out


@pytest.mark.parametrize("window", [R, 512])
def test_ring_decode_equals_linear_decode(window):
    cfg = dataclasses.replace(CONFIGS["c1_decode"], window=window, seed=81, batch=5)
    lens = [100, 1024, 1025, 3000, 5001]   # below, at and past the first wrap; several wraps
    shape_lin, t = build_decode(cfg, list(range(5)), lens, cap=5001)
    ring = _ring_of(t, lens)
    lin = _decode(shape_lin, t, t["cache"], lens, 5001)
    shape_ring = dataclasses.replace(shape_lin, ring=True)
    got = _decode(shape_ring, t, ring, lens, 5001)
    assert_close(bf16_dev_to_f32(got), bf16_dev_to_f32(lin), "ring vs linear decode", max_abs=4e-3, mean_abs=2e-4)
    for b, L in enumerate(lens):
        ref, _, _ = oracle_decode_seq(cfg, b, L)
        assert_close(bf16_dev_to_f32(got[b]), ref, f"ring decode L={L} window={window}")
        # the new token's K/V went to slot (L-1) % R, the same bits as the linear cache's position L-1
        assert torch.equal(ring.k[b, :, (L - 1) % R], t["cache"].k[b, :, L - 1])
        assert torch.equal(ring.v[b, :, (L - 1) % R], t["cache"].v[b, :, L - 1])


def test_ring_decode_step_after_step():
    """Five decode steps in a row on one ring (each step's new token overwrites the oldest slot)."""
    cfg = dataclasses.replace(CONFIGS["c1_decode"], window=R, seed=82, batch=1)
    L0, steps = 2040, 5
    shape, t = build_decode(cfg, [0], [L0 + steps - 1], cap=L0 + steps)
    ring = _ring_of(t, [L0])
    shape_ring = dataclasses.replace(shape, ring=True)
    from oracle import inputs as I
    from helpers import to_dev_bf16
    for s in range(steps):
        L = L0 + s
        q = to_dev_bf16(I.q_rows(cfg, 0, L - 1, L)[0][None])
        k = to_dev_bf16(I.k_rows(cfg, 0, L - 1, L)[0][None])
        v = to_dev_bf16(I.v_rows(cfg, 0, L - 1, L)[0][None])
        tt = dict(t, q_raw=q, k_new=k, v_new=v, lens=torch.tensor([L], dtype=torch.int32, device="cuda"))
        got = _decode(shape_ring, tt, ring, [L], L)
        ref, _, _ = oracle_decode_seq(cfg, 0, L)
        assert_close(bf16_dev_to_f32(got[0]), ref, f"ring step {s} (L={L})")
