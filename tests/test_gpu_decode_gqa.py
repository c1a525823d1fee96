"""GPU parity of the decode form for wide GQA groups and head_dim 512 (decode_gqa.cu, reached
through apex_attn_decode_bf16): the reference model's global layers -- 16 q heads over 2 kv heads of
head_dim 512, RoPE on the first 64 of 256 pairs, theta 1e6, weightless RMSNorm of V
(docs/B6_3_attention.md:46-60) -- against the reference-code goldens and the fp32 oracle, plus
groups 4 and 8 at head_dim 256, windows, and V taken from the raw k projection."""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from oracle import inputs as I
from apex_b200 import ops
from apex_b200.configs import CONFIGS
from helpers import assert_close, bf16_dev_to_f32, golden, manifest, oracle_decode_seq, to_dev_bf16
from test_gpu_decode import build_decode, run_decode

pytestmark = pytest.mark.gpu
G = CONFIGS["global_decode"]


def test_global_layer_decode_vs_reference_golden():
    rows = manifest()["global_decode"]["rows"]
    g = golden("global_decode")
    for i, r in enumerate(rows):
        shape, t = build_decode(G, [r["seq"]], [r["context"]])
        got, _ = run_decode(shape, t)
        mx, mn = assert_close(got[0], g[i], f"global layer seq {r['seq']} L={r['context']} vs reference golden")
        print(f"global decode L={r['context']}: max {mx:.2e} mean {mn:.2e}")


@pytest.mark.parametrize("window", [0, 300])
def test_global_layer_decode_lengths_vs_oracle(window):
    """Every tile edge (16 keys), one and several splits, ragged batch, repeated calls."""
    cfg = dataclasses.replace(G, window=window, seed=71)
    lens = [1, 2, 15, 16, 17, 33, 100, 1000, 4097, 9000]
    shape, t = build_decode(cfg, list(range(len(lens))), lens, cap=9000)
    got, ws = run_decode(shape, t)
    again, _ = run_decode(shape, t, ws)
    np.testing.assert_array_equal(got, again)
    for i, L in enumerate(lens):
        ref, Kc, Vc = oracle_decode_seq(cfg, i, L)
        assert_close(got[i], ref, f"L={L} window={window}")
    # the new token's K (norm + partial RoPE) and V (weightless norm) were appended at L-1
    L = lens[-1]
    _, Kc, Vc = oracle_decode_seq(cfg, len(lens) - 1, L)
    assert_close(bf16_dev_to_f32(t["cache"].k[len(lens) - 1, :, L - 1]), Kc[:, L - 1], "appended K",
                 max_abs=3e-2, mean_abs=3e-3)
    assert_close(bf16_dev_to_f32(t["cache"].v[len(lens) - 1, :, L - 1]), Vc[:, L - 1], "appended V",
                 max_abs=3e-2, mean_abs=3e-3)


def test_global_layer_v_from_raw_k():
    """Full layers have no v_proj: V = weightless rmsnorm(k_raw) (docs/B6_3_attention.md:30-31), so the
    caller passes the raw k row as v_new; the cache then holds norm(k_raw) on the V side."""
    cfg = dataclasses.replace(G, seed=72)
    lens = [700, 2048]
    shape, t = build_decode(cfg, [0, 1], lens, cap=2048)
    t["v_new"] = t["k_new"]
    got, _ = run_decode(shape, t)
    for i, L in enumerate(lens):
        # the oracle's v stream replaced by k for the new token: rebuild the reference with v_new = k_new
        from oracle import inputs as OI
        import oracle
        qw, kw = OI.norm_weights(cfg)
        D, Hkv, Hq = cfg.head_dim, cfg.kv_heads, cfg.q_heads
        k = OI.f32(OI.k_rows(cfg, i, 0, L))
        v = OI.f32(OI.v_rows(cfg, i, 0, L))
        q = OI.f32(OI.q_rows(cfg, i, L - 1, L))
        Kc = np.zeros(Hkv * L * D, np.float32)
        Vc = np.zeros_like(Kc)
        oracle.kv_append(k[:L - 1], kw, 1, cfg.rope_pairs, cfg.rope_theta, cfg.eps, Kc, L, 0, L - 1, Hkv, D)
        oracle.kv_append(v[:L - 1], None, 1, 0, cfg.rope_theta, cfg.eps, Vc, L, 0, L - 1, Hkv, D)
        ref = oracle.decode(q, k[L - 1:], k[L - 1:], qw, kw, qk_norm=1, v_norm=1, rope_pairs=cfg.rope_pairs,
                            rope_base=cfg.rope_theta, eps=cfg.eps, scale=cfg.scale, window=0, Kc=Kc, Vc=Vc, cap=L,
                            lens=np.array([L], np.int32), B=1, Hq=Hq, Hkv=Hkv, D=D)
        assert_close(got[i], ref[0], f"V from raw k, L={L}")


@pytest.mark.parametrize("q_heads,kv_heads,head_dim", [(16, 4, 256), (16, 2, 256), (8, 8, 512), (24, 3, 512)])
def test_gqa_groups_vs_oracle(q_heads, kv_heads, head_dim):
    cfg = dataclasses.replace(CONFIGS["c1_decode"], q_heads=q_heads, kv_heads=kv_heads, head_dim=head_dim,
                              seed=73 + q_heads + head_dim, rope_theta=1e6)
    lens = [1, 257, 3000]
    shape, t = build_decode(cfg, [0, 1, 2], lens, cap=3000)
    got, _ = run_decode(shape, t)
    for i, L in enumerate(lens):
        ref, _, _ = oracle_decode_seq(cfg, i, L)
        assert_close(got[i], ref, f"Hq={q_heads} Hkv={kv_heads} hd={head_dim} L={L}")


@pytest.mark.parametrize("lens", [[20000], [5000, 7]])
def test_global_layer_decode_small_batch_many_splits(lens):
    """One or two sequences take up to ~300 splits per kv head; their last CTAs stream the partials
    through shared memory in pieces of 15 splits (several pieces per head, a short last piece)."""
    cfg = dataclasses.replace(G, seed=74 + len(lens))
    shape, t = build_decode(cfg, list(range(len(lens))), lens)
    got, ws = run_decode(shape, t)
    again, _ = run_decode(shape, t, ws)
    np.testing.assert_array_equal(got, again)
    for i, L in enumerate(lens):
        ref, _, _ = oracle_decode_seq(cfg, i, L)
        assert_close(got[i], ref, f"small batch L={L}")
