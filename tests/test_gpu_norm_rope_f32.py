"""GPU parity of the f32 drop-ins (head_norm_rope_f32, attention_f32) and the bf16 norm+rope,
against the goldens made by the reference's CPU code and the oracle.  The f32 kernels use the
reference's own gate, rel-L2 < 1e-5 (src/tests/test_norm.cpp:92)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from apex_b200 import ops
from helpers import bf16_dev_to_f32, golden, manifest, to_dev_bf16

pytestmark = pytest.mark.gpu
MAN = manifest()


def rel_l2(a, b):
    a = np.asarray(a, np.float64).ravel()
    b = np.asarray(b, np.float64).ravel()
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("name", ["hnr_q_sliding", "hnr_k_full_cache", "hnr_v_cache"])
def test_head_norm_rope_f32_vs_reference_golden(name):
    c = MAN[name]
    n = c["tokens"] * c["heads"] * c["head_dim"]
    x = oracle.bf16_to_f32(oracle.normal_bf16(n, c["seed"], 1))
    w = oracle.normal_bf16(c["head_dim"], c["seed"], 4, 0, 1.0, 0.1)
    out = torch.full((c["out_len"],), c["sentinel"], dtype=torch.float32, device="cuda")
    ops.head_norm_rope(torch.from_numpy(x).cuda(), to_dev_bf16(w), bool(c["has_weight"]), out,
                       c["tokens"], c["heads"], c["head_dim"], c["rope_pairs"], c["rope_base"],
                       c["abs_pos"], c["ots"], c["ohs"], c["eps"])
    got = out.cpu().numpy()
    g = golden(name)
    untouched = g == c["sentinel"]
    np.testing.assert_array_equal(got[untouched], g[untouched])   # strided writes only
    assert rel_l2(got, g) < 1e-5
    assert np.abs(got - g).max() < 1e-4


def test_head_norm_rope_f32_in_place():
    T, H, D = 9, 16, 256
    x = oracle.bf16_to_f32(oracle.normal_bf16(T * H * D, 5, 1))
    w = oracle.normal_bf16(D, 5, 4, 0, 1.0, 0.1)
    ref = np.zeros_like(x)
    oracle.head_norm_rope_f32(x, w, ref, T, H, D, 1, 128, 1e4, 100, H * D, D, 1e-6)
    buf = torch.from_numpy(x.copy()).cuda()
    ops.head_norm_rope(buf, to_dev_bf16(w), True, buf, T, H, D, 128, 1e4, 100, H * D, D, 1e-6)
    assert rel_l2(buf.cpu().numpy(), ref) < 1e-5


@pytest.mark.parametrize("T,H,D,pairs,pos", [(5, 8, 256, 128, 0), (3, 2, 512, 64, 131000), (4, 3, 96, 48, 7)])
def test_head_norm_rope_bf16_vs_oracle(T, H, D, pairs, pos):
    xu = oracle.normal_bf16(T * H * D, 6, 1)
    w = oracle.normal_bf16(D, 6, 4, 0, 1.0, 0.1)
    ref = np.zeros(T * H * D, np.float32)
    oracle.head_norm_rope_f32(oracle.bf16_to_f32(xu), w, ref, T, H, D, 1, pairs, 1e6, pos, H * D, D, 1e-6)
    out = torch.zeros(T * H * D, dtype=torch.bfloat16, device="cuda")
    ops.head_norm_rope(to_dev_bf16(xu), to_dev_bf16(w), True, out, T, H, D, pairs, 1e6, pos, H * D, D, 1e-6)
    got = bf16_dev_to_f32(out)
    # one bf16 rounding of |y| (<= ~4 sigma * 1.3 weight) plus angle error at large positions
    assert np.abs(got - ref).max() <= 3e-2
    assert np.abs(got - ref).mean() <= 2e-3


@pytest.mark.parametrize("name", ["attn_f32_window16", "attn_f32_global"])
def test_attention_f32_vs_reference_golden(name):
    c = MAN[name]
    T, Hq, Hkv, hd, cap = c["tokens"], c["q_heads"], c["kv_heads"], c["head_dim"], c["capacity"]
    q = oracle.bf16_to_f32(oracle.normal_bf16(T * Hq * hd, c["seed"], 1)) * c["q_mul"]
    K = oracle.bf16_to_f32(oracle.normal_bf16(Hkv * cap * hd, c["seed"], 2)) * c["k_mul"]
    V = oracle.bf16_to_f32(oracle.normal_bf16(Hkv * cap * hd, c["seed"], 3))
    out = torch.zeros(T * Hq * hd, dtype=torch.float32, device="cuda")
    shape = ops.AttentionShape(Hq, Hkv, hd, 0, 1e4, c["window"], c["scale"])
    cache = ops.KvCache(torch.from_numpy(K).cuda().view(Hkv, cap, hd), torch.from_numpy(V).cuda().view(Hkv, cap, hd))
    ops.attention(torch.from_numpy(q).cuda(), cache, out, shape, T, c["pos0"])
    got = out.cpu().numpy().reshape(T, Hq, hd)
    assert rel_l2(got, golden(name)) < 1e-5


@pytest.mark.parametrize("T,Hq,Hkv,hd,pos0,window", [(3, 16, 2, 512, 0, 0), (17, 8, 8, 100, 30, 7), (1, 4, 1, 32, 999, 0)])
def test_attention_f32_shapes_vs_oracle(T, Hq, Hkv, hd, pos0, window):
    cap = pos0 + T + 3
    rng = np.random.default_rng(T + hd)
    q = (rng.standard_normal(T * Hq * hd) * 0.3).astype(np.float32)
    K = (rng.standard_normal(Hkv * cap * hd) * 0.3).astype(np.float32)
    V = rng.standard_normal(Hkv * cap * hd).astype(np.float32)
    ref = oracle.attention_f32(q, K, V, T, Hq, Hkv, hd, cap, pos0, window, 1.0)
    out = torch.zeros(T * Hq * hd, dtype=torch.float32, device="cuda")
    shape = ops.AttentionShape(Hq, Hkv, hd, 0, 1e4, window, 1.0)
    cache = ops.KvCache(torch.from_numpy(K).cuda().view(Hkv, cap, hd), torch.from_numpy(V).cuda().view(Hkv, cap, hd))
    ops.attention(torch.from_numpy(q).cuda(), cache, out, shape, T, pos0)
    assert rel_l2(out.cpu().numpy(), ref) < 1e-5
