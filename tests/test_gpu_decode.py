"""GPU parity of the fused split-KV decode (apex_attn_decode_bf16 / _partial_bf16 / merge)
against the fp32 oracle and the reference-code goldens, at the configurations' full sizes."""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

import oracle
from oracle import inputs as I
from apex_b200 import ops
from apex_b200.configs import CONFIGS
from helpers import (assert_close, bf16_dev_to_f32, fill_k_cache, fill_v_cache, golden, manifest,
                     oracle_decode_seq, to_dev_bf16)

pytestmark = pytest.mark.gpu
MAN = manifest()


def build_decode(cfg, seqs, lens, cap=None):
    """Device inputs for config sequences `seqs` with key counts `lens` (history in the cache,
    new token at L-1).  Returns (shape, tensors dict)."""
    B = len(seqs)
    Hq, Hkv, D = cfg.q_heads, cfg.kv_heads, cfg.head_dim
    cap = cap or int(max(lens))
    qw, kw = I.norm_weights(cfg)
    kc = torch.zeros(B, Hkv, cap, D, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    q_raw = np.stack([I.q_rows(cfg, b, L - 1, L)[0] for b, L in zip(seqs, lens)])
    k_new = np.stack([I.k_rows(cfg, b, L - 1, L)[0] for b, L in zip(seqs, lens)])
    v_new = np.stack([I.v_rows(cfg, b, L - 1, L)[0] for b, L in zip(seqs, lens)])
    for i, (b, L) in enumerate(zip(seqs, lens)):
        fill_k_cache(kc[i], I.k_rows(cfg, b, 0, L - 1), kw, cfg)
        fill_v_cache(vc[i], I.v_rows(cfg, b, 0, L - 1), cfg=cfg)
    t = dict(q_raw=to_dev_bf16(q_raw), k_new=to_dev_bf16(k_new), v_new=to_dev_bf16(v_new),
             qw=to_dev_bf16(qw), kw=to_dev_bf16(kw), cache=ops.KvCache(kc, vc),
             lens=torch.tensor(np.asarray(lens, np.int32), device="cuda"), max_len=int(max(lens)))
    return ops.AttentionShape.from_config(cfg), t


def run_decode(shape, t, ws=None):
    B = t["lens"].numel()
    ws = ws or ops.DecodeWorkspace(shape, B, t["max_len"])
    out = torch.empty(B, shape.q_heads, shape.head_dim, dtype=torch.bfloat16, device="cuda")
    ops.attention_decode(shape, t["q_raw"], t["k_new"], t["v_new"], t["qw"], t["kw"], t["cache"], t["lens"],
                         t["max_len"], out, ws)
    ops.device_status()
    return bf16_dev_to_f32(out), ws


def test_c1_decode_vs_golden_and_oracle():
    cfg = CONFIGS["c1_decode"]
    shape, t = build_decode(cfg, [0], [cfg.context])
    got, _ = run_decode(shape, t)
    ref, Kc, Vc = oracle_decode_seq(cfg, 0, cfg.context)
    mx, mn = assert_close(got[0], golden("c1_decode")[0], "c1 vs reference golden")
    assert_close(got[0], ref, "c1 vs oracle")
    # the new token's K/V were appended to the cache at position L-1
    L = cfg.context
    k_dev = bf16_dev_to_f32(t["cache"].k[0, :, L - 1, :])
    np.testing.assert_allclose(k_dev, Kc[:, L - 1, :], rtol=1e-2, atol=2e-2)
    np.testing.assert_array_equal(bf16_dev_to_f32(t["cache"].v[0, :, L - 1, :]),
                                  oracle.round_bf16(Vc[:, L - 1, :]))
    print(f"c1 decode vs golden: max {mx:.2e} mean {mn:.2e}")


def test_c3_ragged_decode_all_sequences_vs_oracle():
    cfg = CONFIGS["c3_ragged_decode"]
    lens = [int(x) for x in I.decode_lens(cfg)]
    shape, t = build_decode(cfg, list(range(cfg.batch)), lens, cap=cfg.lens_range[1])
    got, _ = run_decode(shape, t)
    worst = (0.0, 0.0)
    for b in range(cfg.batch):
        ref, _, _ = oracle_decode_seq(cfg, b, lens[b])
        mx, mn = assert_close(got[b], ref, f"c3 seq {b} (L={lens[b]})")
        worst = (max(worst[0], mx), max(worst[1], mn))
    m = MAN["c3_ragged_decode"]
    g = golden("c3_ragged_decode")
    for i, b in enumerate(m["seqs"]):
        assert_close(got[b], g[i], f"c3 seq {b} vs reference golden")
    print(f"c3 decode worst: max {worst[0]:.2e} mean {worst[1]:.2e}")


@pytest.mark.parametrize("window", [0, 64])
def test_decode_edge_lengths(window):
    cfg = dataclasses.replace(CONFIGS["c1_decode"], window=window, seed=21)
    lens = [1, 2, 31, 32, 33, 63, 64, 65, 100, 257, 1000, 4103]
    shape, t = build_decode(cfg, list(range(len(lens))), lens, cap=4200)
    got, _ = run_decode(shape, t)
    for i, L in enumerate(lens):
        ref, _, _ = oracle_decode_seq(cfg, i, L)
        assert_close(got[i], ref, f"L={L} window={window}")


@pytest.mark.parametrize("window", [0, 64])
def test_short_context_cluster_form(window):
    """Small batches at contexts up to 4096 take the cluster form (one thread-block cluster per
    (sequence, kv head), partials merged in the leader CTA's shared memory): one split up to 16,
    splits of several stages, and a ragged batch whose short sequences leave splits idle."""
    cfg = dataclasses.replace(CONFIGS["c1_decode"], window=window, seed=31)
    for lens in ([1], [2], [63], [64], [65], [130], [500], [1000], [1024], [1025], [2047], [4096], [100, 1024, 7]):
        shape, t = build_decode(cfg, list(range(len(lens))), lens, cap=max(lens))
        got, ws = run_decode(shape, t)
        again, _ = run_decode(shape, t, ws)
        np.testing.assert_array_equal(got, again)
        for i, L in enumerate(lens):
            ref, _, _ = oracle_decode_seq(cfg, i, L)
            assert_close(got[i], ref, f"L={L} window={window}")


def test_decode_repeated_calls_are_identical():
    cfg = dataclasses.replace(CONFIGS["c3_ragged_decode"], batch=6, seed=22)
    lens = [5000, 700, 8192, 513, 3000, 6001]
    shape, t = build_decode(cfg, list(range(6)), lens, cap=8192)
    a, ws = run_decode(shape, t)
    b, _ = run_decode(shape, t, ws)   # counters must be back to zero; the append is idempotent
    c, _ = run_decode(shape, t, ws)
    np.testing.assert_array_equal(a, b)
    np.testing.assert_array_equal(a, c)


def test_decode_kv_split_partials_merge_to_full():
    cfg = dataclasses.replace(CONFIGS["c1_decode"], batch=2, seed=23, rope_theta=1e6)
    lens = [9000, 6000]
    shape, t = build_decode(cfg, [0, 1], lens, cap=9000)
    full, _ = run_decode(shape, t)
    bounds = [0, 2500, 6000, 9000]          # three "ranks"; rank 2 holds no keys of sequence 1
    parts = []
    for r in range(3):
        lo, hi = bounds[r], bounds[r + 1]
        local = ops.KvCache(t["cache"].k[:, :, lo:hi, :].contiguous(), t["cache"].v[:, :, lo:hi, :].contiguous())
        ws = ops.DecodeWorkspace(shape, 2, 9000)
        part = torch.empty(2, shape.q_heads, shape.head_dim + 2, dtype=torch.float32, device="cuda")
        ops.attention_decode_partial(shape, t["q_raw"], t["k_new"], t["v_new"], t["qw"], t["kw"], local, t["lens"],
                                     9000, lo, hi, part, ws)
        parts.append(part)
    ops.device_status()
    out = torch.empty(2 * shape.q_heads, shape.head_dim, dtype=torch.bfloat16, device="cuda")
    ops.merge_partials(torch.stack(parts).view(3, 2 * shape.q_heads, shape.head_dim + 2), out)
    merged = bf16_dev_to_f32(out).reshape(2, shape.q_heads, shape.head_dim)
    assert_close(merged, full, "merged vs single-call", max_abs=4e-3, mean_abs=2e-4)
    for i, L in enumerate(lens):
        ref, _, _ = oracle_decode_seq(cfg, i, L)
        assert_close(merged[i], ref, f"merged seq {i} vs oracle")


@pytest.mark.parametrize("name,cfg_name,seq", [("c5_long_decode_b1", "c5_long_decode_b1", 0),
                                               ("c5_long_decode_b8_seq7", "c5_long_decode_b8", 7)])
def test_c5_long_decode_vs_reference_golden(name, cfg_name, seq):
    cfg = CONFIGS[cfg_name]
    shape, t = build_decode(cfg, [seq], [cfg.context])
    got, _ = run_decode(shape, t)
    mx, mn = assert_close(got[0], golden(name)[0], f"{name} vs reference golden")
    print(f"{name}: max {mx:.2e} mean {mn:.2e}")


def test_c5_batch8_equals_single_sequence_runs():
    """Full-size B=8 x 131072 keys: the batched call equals eight B=1 calls (property check;
    inputs drawn on the device)."""
    cfg = CONFIGS["c5_long_decode_b8"]
    shape = ops.AttentionShape.from_config(cfg)
    B, L, Hq, Hkv, D = cfg.batch, cfg.context, cfg.q_heads, cfg.kv_heads, cfg.head_dim
    g = torch.Generator(device="cuda").manual_seed(cfg.seed)
    kc = torch.randn(B, Hkv, L, D, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(B, Hkv, L, D, generator=g, device="cuda").to(torch.bfloat16)
    q = (torch.randn(B, Hq, D, generator=g, device="cuda") * 0.0625).to(torch.bfloat16)
    kn = torch.randn(B, Hkv, D, generator=g, device="cuda").to(torch.bfloat16)
    vn = torch.randn(B, Hkv, D, generator=g, device="cuda").to(torch.bfloat16)
    lens = torch.full((B,), L, dtype=torch.int32, device="cuda")
    out = torch.empty(B, Hq, D, dtype=torch.bfloat16, device="cuda")
    ws = ops.DecodeWorkspace(shape, B, L)
    ops.attention_decode(shape, q, kn, vn, None, None, ops.KvCache(kc, vc), lens, L, out, ws)
    ws1 = ops.DecodeWorkspace(shape, 1, L)
    for b in (0, 3, 7):
        o1 = torch.empty(1, Hq, D, dtype=torch.bfloat16, device="cuda")
        ops.attention_decode(shape, q[b:b + 1].contiguous(), kn[b:b + 1].contiguous(), vn[b:b + 1].contiguous(), None,
                             None, ops.KvCache(kc[b:b + 1].contiguous(), vc[b:b + 1].contiguous()), lens[b:b + 1], L,
                             o1, ws1)
        diff = (o1[0].float() - out[b].float()).abs().max().item()
        assert diff <= 4e-3, (b, diff)
    ops.device_status()
    assert torch.isfinite(out.float()).all()
