"""GPU parity of the fused tcgen05 prefill (apex_attn_prefill_bf16) against the fp32 oracle and
the reference-code goldens: full C2, full-size C4 rows, odd and chunked shapes, cache contents."""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

import oracle
from oracle import inputs as I
from apex_b200 import ops
from apex_b200.configs import CONFIGS
from helpers import (assert_close, bf16_dev_to_f32, golden, manifest, oracle_prefill_rows, to_dev_bf16)

pytestmark = pytest.mark.gpu
MAN = manifest()


def run_prefill(cfg, seqs, T_total, chunk, cap=None, device_out=False):
    """Prefill config sequences `seqs` over positions 0..T_total-1 in chunks; returns
    (out f32 numpy [B, T_total, Hq, D] -- or the bf16 device tensor with device_out -- , cache)."""
    B = len(seqs)
    Hq, Hkv, D = cfg.q_heads, cfg.kv_heads, cfg.head_dim
    cap = cap or T_total
    shape = ops.AttentionShape.from_config(cfg)
    qw, kw = I.norm_weights(cfg)
    q = to_dev_bf16(np.stack([I.q_rows(cfg, b, 0, T_total) for b in seqs]))
    k = to_dev_bf16(np.stack([I.k_rows(cfg, b, 0, T_total) for b in seqs]))
    v = to_dev_bf16(np.stack([I.v_rows(cfg, b, 0, T_total) for b in seqs]))
    cache = ops.KvCache(torch.zeros(B, Hkv, cap, D, dtype=torch.bfloat16, device="cuda"),
                        torch.zeros(B, Hkv, cap, D, dtype=torch.bfloat16, device="cuda"))
    out = torch.empty(B, T_total, Hq, D, dtype=torch.bfloat16, device="cuda")
    ws = ops.PrefillWorkspace(shape, B, chunk)
    for c0 in range(0, T_total, chunk):
        T = min(chunk, T_total - c0)
        o = torch.empty(B, T, Hq, D, dtype=torch.bfloat16, device="cuda")
        ops.attention_prefill(shape, q[:, c0:c0 + T].contiguous(), k[:, c0:c0 + T].contiguous(),
                              v[:, c0:c0 + T].contiguous(), to_dev_bf16(qw), to_dev_bf16(kw), cache, c0, o, ws)
        out[:, c0:c0 + T] = o
    ops.device_status()
    return (out if device_out else bf16_dev_to_f32(out)), cache


def edge_rows(T, window, extra=()):
    rows = {0, 1, 2, 63, 64, 127, 128, 129, T - 1, T - 2, T // 2}
    if window:
        rows |= {window - 2, window - 1, window, window + 1, window + 127, window + 128}
    rows |= set(extra)
    return sorted(r for r in rows if 0 <= r < T)


def test_c2_prefill_window_vs_golden_and_oracle():
    cfg = CONFIGS["c2_prefill_window"]
    T = cfg.seq_len
    got, cache = run_prefill(cfg, [0], T, T)
    rows_g = MAN["c2_prefill_window"]["positions"]
    mx, mn = assert_close(got[0, rows_g], golden("c2_prefill_window"), "c2 vs reference golden")
    rng = np.random.default_rng(0)
    rows = sorted(set(edge_rows(T, cfg.window)) | set(rng.choice(T, 200, replace=False).tolist()))
    ref = oracle_prefill_rows(cfg, 0, T, rows)
    assert_close(got[0, rows], ref, "c2 vs oracle (sampled rows)")
    # K/V appended to the cache: K = rope(rmsnorm(k)) rounded once, V = v
    qw, kw = I.norm_weights(cfg)
    k = I.f32(I.k_rows(cfg, 0, 0, T))
    Kc = np.zeros(cfg.kv_heads * T * cfg.head_dim, np.float32)
    oracle.kv_append(k, kw, 1, cfg.rope_pairs, cfg.rope_theta, cfg.eps, Kc, T, 0, T, cfg.kv_heads, cfg.head_dim)
    kd = bf16_dev_to_f32(cache.k[0])
    assert_close(kd, Kc.reshape(cfg.kv_heads, T, cfg.head_dim), "K cache", max_abs=3e-2, mean_abs=2e-3)
    np.testing.assert_array_equal(bf16_dev_to_f32(cache.v[0]),
                                  I.f32(I.v_rows(cfg, 0, 0, T)).transpose(1, 0, 2))
    print(f"c2 prefill vs golden: max {mx:.2e} mean {mn:.2e}")


@pytest.mark.parametrize("T,window", [(1, 0), (7, 0), (129, 0), (300, 5), (300, 200), (1000, 128), (513, 512)])
def test_prefill_odd_shapes_all_rows(T, window):
    cfg = dataclasses.replace(CONFIGS["c2_prefill_window"], seq_len=T, chunk=T, window=window, seed=31 + T)
    got, _ = run_prefill(cfg, [0], T, T)
    ref = oracle_prefill_rows(cfg, 0, T, list(range(T)))
    assert_close(got[0], ref, f"T={T} window={window}")


@pytest.mark.parametrize("window", [0, 700])
def test_chunked_prefill_matches_one_shot_rows(window):
    cfg = dataclasses.replace(CONFIGS["c4_chunked_prefill"], batch=2, seq_len=3000, chunk=1000,
                              window=window, seed=41)
    got, _ = run_prefill(cfg, [0, 1], 3000, 1000, cap=3100)
    rows = edge_rows(3000, window, extra=(999, 1000, 1001, 1999, 2000, 2001, 2999))
    for b in (0, 1):
        ref = oracle_prefill_rows(cfg, b, 3000, rows)
        assert_close(got[b, rows], ref, f"chunked seq {b} window {window}")


def test_c4_chunked_prefill_rows_vs_reference_golden():
    cfg = CONFIGS["c4_chunked_prefill"]
    m = MAN["c4_chunked_prefill"]["rows"]
    seqs = [r["seq"] for r in m]
    got, _ = run_prefill(cfg, seqs, cfg.seq_len, cfg.chunk)
    g = golden("c4_chunked_prefill")
    i = 0
    worst = (0.0, 0.0)
    for bi, r in enumerate(m):
        n = len(r["positions"])
        mx, mn = assert_close(got[bi, r["positions"]], g[i:i + n], f"c4 seq {r['seq']} vs reference golden")
        worst = (max(worst[0], mx), max(worst[1], mn))
        i += n
    print(f"c4 rows vs golden: max {worst[0]:.2e} mean {worst[1]:.2e}")


def test_c4_chunked_prefill_256_rows_all_sequences():
    """The whole C4 configuration (4 x 32768 tokens in 8 chunks of 4096, appended to the cache in
    order) with 64 sampled rows of every sequence: the first rows, every chunk edge (p0 - 1, p0,
    p0 + 1), the last row and random rows, against the fp32 restatement (which equals the
    reference's own CPU code bit for bit, tests/test_oracle.py)."""
    cfg = CONFIGS["c4_chunked_prefill"]
    S, C = cfg.seq_len, cfg.chunk
    got, _ = run_prefill(cfg, list(range(cfg.batch)), S, C, device_out=True)
    edges = {0, 1, 2, S - 1}
    for p0 in range(C, S, C):
        edges |= {p0 - 1, p0, p0 + 1}
    rng = np.random.default_rng(4)
    worst, n_rows = (0.0, 0.0), 0
    for b in range(cfg.batch):
        rest = [int(r) for r in rng.choice(S, 64 - len(edges), replace=False) if int(r) not in edges]
        rows = sorted(edges | set(rest))
        ref = oracle_prefill_rows(cfg, b, max(rows) + 1, rows)
        mx, mn = assert_close(bf16_dev_to_f32(got[b, rows]), ref, f"c4 seq {b} ({len(rows)} rows)")
        worst = (max(worst[0], mx), max(worst[1], mn))
        n_rows += len(rows)
    assert n_rows >= 250
    print(f"c4 {n_rows} rows over {cfg.batch} sequences: max {worst[0]:.2e} mean {worst[1]:.2e}")


def test_batched_prefill_equals_per_sequence():
    cfg = dataclasses.replace(CONFIGS["c4_chunked_prefill"], batch=3, seq_len=1536, chunk=768, seed=51)
    got, _ = run_prefill(cfg, [0, 1, 2], 1536, 768)
    for b in (0, 2):
        one, _ = run_prefill(cfg, [b], 1536, 768)
        np.testing.assert_array_equal(got[b], one[0])


@pytest.mark.parametrize("q_heads,kv_heads,T,window", [(8, 8, 700, 0), (16, 4, 515, 300), (6, 2, 300, 0),
                                                        (16, 8, 1, 0), (8, 8, 129, 64)])
def test_prefill_gqa_group_sizes(q_heads, kv_heads, T, window):
    """Even groups pair the two heads of a group in one CTA pair; odd groups (incl. MHA) pair
    256 consecutive queries of one head."""
    cfg = dataclasses.replace(CONFIGS["c2_prefill_window"], q_heads=q_heads, kv_heads=kv_heads, seq_len=T,
                              chunk=T, window=window, seed=61 + q_heads + T)
    got, _ = run_prefill(cfg, [0], T, T)
    rng = np.random.default_rng(T)
    rows = sorted(set(edge_rows(T, window, extra=(255, 256, 257, 383, 384))) |
                  set(rng.choice(T, min(T, 64), replace=False).tolist()))
    ref = oracle_prefill_rows(cfg, 0, T, rows)
    assert_close(got[0, rows], ref, f"Hq={q_heads} Hkv={kv_heads} T={T} window={window}")
