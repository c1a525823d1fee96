"""GPU parity of the head_dim-512 prefill (prefill_gqa.cu, reached through apex_attn_prefill_bf16):
the reference model's global layers -- 16 q heads over 2 kv heads of head_dim 512, RoPE on the first
64 of 256 pairs, theta 1e6, weightless RMSNorm of V (docs/B6_3_attention.md:46-60) -- against the
reference-code goldens of the global-layer decode (a decode of L keys is the prefill row at position
L - 1 of the same sequence: every input row is a function of its position only) and the fp32 oracle:
tile edges (16 queries, 32 keys), chunks starting off a tile edge, windows, odd groups, batches,
and the caches the preparation writes."""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest

import oracle
from oracle import inputs as I
from apex_b200.configs import CONFIGS
from helpers import assert_close, bf16_dev_to_f32, golden, manifest, oracle_prefill_rows
from test_gpu_prefill import edge_rows, run_prefill

pytestmark = pytest.mark.gpu
G = dataclasses.replace(CONFIGS["global_decode"], kind="prefill", batch=1)


def test_global_prefill_rows_vs_reference_golden():
    g = golden("global_decode")
    for i, r in enumerate(manifest()["global_decode"]["rows"]):
        L = r["context"]
        cfg = dataclasses.replace(G, seq_len=L, chunk=L)
        got, _ = run_prefill(cfg, [r["seq"]], L, L)
        mx, mn = assert_close(got[0, L - 1], g[i], f"global prefill seq {r['seq']} row {L - 1} vs reference golden")
        print(f"global prefill T={L} last row: max {mx:.2e} mean {mn:.2e}")


@pytest.mark.parametrize("T,window", [(1, 0), (17, 0), (300, 0), (1100, 0), (700, 100)])
def test_global_prefill_rows_vs_oracle(T, window):
    cfg = dataclasses.replace(G, seq_len=T, chunk=T, window=window, seed=81 + T)
    got, cache = run_prefill(cfg, [0], T, T)
    rng = np.random.default_rng(T)
    rows = sorted(set(edge_rows(T, window, extra=(15, 16, 31, 32, 33))) |
                  set(rng.choice(T, min(T, 40), replace=False).tolist()))
    ref = oracle_prefill_rows(cfg, 0, T, rows)
    mx, mn = assert_close(got[0, rows], ref, f"T={T} window={window}")
    print(f"global prefill T={T} window={window}: {len(rows)} rows, max {mx:.2e} mean {mn:.2e}")


def test_global_prefill_caches_vs_oracle():
    """K: norm + partial RoPE at each position; V: weightless norm of the raw rows."""
    T = 200
    cfg = dataclasses.replace(G, seq_len=T, chunk=T, seed=90)
    _, cache = run_prefill(cfg, [0], T, T)
    _, kw = I.norm_weights(cfg)
    k = I.f32(I.k_rows(cfg, 0, 0, T))
    v = I.f32(I.v_rows(cfg, 0, 0, T))
    D, Hkv = cfg.head_dim, cfg.kv_heads
    Kc = np.zeros(Hkv * T * D, np.float32)
    Vc = np.zeros_like(Kc)
    oracle.kv_append(k, kw, 1, cfg.rope_pairs, cfg.rope_theta, cfg.eps, Kc, T, 0, T, Hkv, D)
    oracle.kv_append(v, None, 1, 0, cfg.rope_theta, cfg.eps, Vc, T, 0, T, Hkv, D)
    assert_close(bf16_dev_to_f32(cache.k[0]), Kc.reshape(Hkv, T, D), "K cache", max_abs=3e-2, mean_abs=3e-3)
    assert_close(bf16_dev_to_f32(cache.v[0]), Vc.reshape(Hkv, T, D), "V cache", max_abs=3e-2, mean_abs=3e-3)


@pytest.mark.parametrize("window", [0, 50])
def test_global_prefill_chunks_match_one_shot(window):
    """Chunks of 150 tokens start off the query-tile and 32-key tile edges; chunked and one-call rows
    both match the oracle."""
    T = 600
    cfg = dataclasses.replace(G, seq_len=T, chunk=T, window=window, seed=91)
    one, _ = run_prefill(cfg, [0], T, T)
    chunked, _ = run_prefill(cfg, [0], T, 150)
    rows = edge_rows(T, window, extra=(149, 150, 151, 299, 300, 450))
    ref = oracle_prefill_rows(cfg, 0, T, rows)
    assert_close(chunked[0, rows], ref, f"chunked window={window}")
    assert_close(one[0, rows], ref, f"one call window={window}")


@pytest.mark.parametrize("q_heads,kv_heads", [(6, 2), (10, 2), (16, 1), (8, 8), (4, 1), (8, 4)])
def test_prefill_512_group_sizes(q_heads, kv_heads):
    """Groups of 1, 2, 4 and 8 take the tensor-core pair kernel (128 / group queries per item); groups
    of 3, 5 and 16 the mma.sync form (groups of 3 and 5 leave one head slot of a CTA idle)."""
    T = 130
    cfg = dataclasses.replace(G, q_heads=q_heads, kv_heads=kv_heads, seq_len=T, chunk=T, seed=95 + q_heads)
    got, _ = run_prefill(cfg, [0], T, T)
    rows = edge_rows(T, 0)
    ref = oracle_prefill_rows(cfg, 0, T, rows)
    assert_close(got[0, rows], ref, f"Hq={q_heads} Hkv={kv_heads}")


def test_global_prefill_batch_equals_per_sequence():
    T = 260
    cfg = dataclasses.replace(G, batch=3, seq_len=T, chunk=T, seed=97)
    got, _ = run_prefill(cfg, [0, 1, 2], T, 130)
    for b in (0, 2):
        one, _ = run_prefill(cfg, [b], T, 130)
        np.testing.assert_array_equal(got[b], one[0])
