"""Shared helpers of the parity tests: seeded host inputs, device upload, oracle runs and the
tolerance check (fp32 accumulation, bf16 output: max |err| <= 2e-2, mean |err| <= 2e-3
against the fp32 oracle)."""
from __future__ import annotations

import json
import pathlib

import numpy as np

import oracle
from oracle import inputs as I

TOL_MAX = 2e-2
TOL_MEAN = 2e-3
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"


def golden(name):
    return np.load(GOLDEN / f"{name}.npy")


def manifest():
    return json.loads((GOLDEN / "manifest.json").read_text())["cases"]


def err_stats(got, ref):
    g = np.asarray(got, np.float64)
    r = np.asarray(ref, np.float64)
    if not (np.isfinite(g).all() and np.isfinite(r).all()):
        return float("inf"), float("inf")
    e = np.abs(g - r)
    return float(e.max(initial=0.0)), float(e.mean()) if e.size else 0.0


def assert_close(got, ref, what="", max_abs=TOL_MAX, mean_abs=TOL_MEAN):
    mx, mn = err_stats(got, ref)
    assert mx <= max_abs and mn <= mean_abs, f"{what}: max |err| {mx:.3e} (<= {max_abs}), mean {mn:.3e} (<= {mean_abs})"
    return mx, mn


# ---------------------------------------------------------------------------- torch glue

def to_dev_bf16(u16: np.ndarray):
    import torch
    return torch.from_numpy(np.ascontiguousarray(u16).view(np.int16)).to("cuda").view(torch.bfloat16)


def bf16_dev_to_f32(t) -> np.ndarray:
    import torch
    return oracle.bf16_to_f32(t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16))


def fill_k_cache(cache_k_b, k_rows_u16, w_u16, cfg, pos0=0):
    """K rows [n, Hkv, D] -> cache_k_b [Hkv, cap, D] at pos0.. through the product's bf16
    head_norm_rope (the reference's K-into-cache call, docs/B6_3_attention.md:449-450)."""
    from apex_b200 import ops
    n = k_rows_u16.shape[0]
    if n == 0:
        return
    cap, D = cache_k_b.shape[-2], cfg.head_dim
    src = to_dev_bf16(k_rows_u16)
    w = to_dev_bf16(w_u16) if w_u16 is not None else None
    ops.head_norm_rope(src, w, w is not None, cache_k_b[:, pos0:, :], n, cfg.kv_heads, D,
                       cfg.rope_pairs, cfg.rope_theta, pos0, D, cap * D, cfg.eps)


def fill_v_cache(cache_v_b, v_rows_u16, pos0=0, cfg=None):
    """V rows [n, Hkv, D] -> cache_v_b [Hkv, cap, D] at pos0..: as they are (the benchmark
    configurations), or through the product's weightless RMSNorm when cfg.v_norm (the reference
    model's layers, docs/B6_3_attention.md:25)."""
    from apex_b200 import ops
    n = v_rows_u16.shape[0]
    if n == 0:
        return
    if cfg is not None and cfg.v_norm:
        cap, D = cache_v_b.shape[-2], cfg.head_dim
        ops.head_norm_rope(to_dev_bf16(v_rows_u16), None, False, cache_v_b[:, pos0:, :], n, cfg.kv_heads, D, 0,
                           cfg.rope_theta, pos0, D, cap * D, cfg.eps)
        return
    cache_v_b[:, pos0:pos0 + n, :] = to_dev_bf16(v_rows_u16).permute(1, 0, 2)


# ---------------------------------------------------------------------------- oracle runs

def oracle_decode_seq(cfg, b, L, round_bf16=0, window=None):
    """Oracle output [Hq, D] for sequence b with L keys (new token at L-1)."""
    qw, kw = I.norm_weights(cfg)
    D, Hkv, Hq = cfg.head_dim, cfg.kv_heads, cfg.q_heads
    win = cfg.window if window is None else window
    k = I.f32(I.k_rows(cfg, b, 0, L))
    v = I.f32(I.v_rows(cfg, b, 0, L))
    q = I.f32(I.q_rows(cfg, b, L - 1, L))
    Kc = np.zeros(Hkv * L * D, np.float32)
    Vc = np.zeros_like(Kc)
    oracle.kv_append(k[:L - 1], kw, cfg.qk_norm, cfg.rope_pairs, cfg.rope_theta, cfg.eps, Kc, L, 0,
                     L - 1, Hkv, D, round_bf16)
    oracle.kv_append(v[:L - 1], None, cfg.v_norm, 0, cfg.rope_theta, cfg.eps, Vc, L, 0, L - 1, Hkv, D,
                     round_bf16)
    out = oracle.decode(q, k[L - 1:], v[L - 1:], qw, kw, qk_norm=cfg.qk_norm, v_norm=cfg.v_norm,
                        rope_pairs=cfg.rope_pairs, rope_base=cfg.rope_theta, eps=cfg.eps,
                        scale=cfg.scale, window=win, Kc=Kc, Vc=Vc, cap=L,
                        lens=np.array([L], np.int32), B=1, Hq=Hq, Hkv=Hkv, D=D,
                        round_bf16=round_bf16)
    return out[0], Kc.reshape(Hkv, L, D), Vc.reshape(Hkv, L, D)


def oracle_prefill_rows(cfg, b, seq_tokens, rows, round_bf16=0, window=None):
    """Oracle outputs [len(rows), Hq, D] for absolute query positions `rows` of sequence b
    after prefilling positions 0..seq_tokens-1 (chunking does not change the result)."""
    qw, kw = I.norm_weights(cfg)
    D, Hkv, Hq = cfg.head_dim, cfg.kv_heads, cfg.q_heads
    win = cfg.window if window is None else window
    T = seq_tokens
    q = I.f32(I.q_rows(cfg, b, 0, T))
    k = I.f32(I.k_rows(cfg, b, 0, T))
    v = I.f32(I.v_rows(cfg, b, 0, T))
    Kc = np.zeros(Hkv * T * D, np.float32)
    Vc = np.zeros_like(Kc)
    return oracle.prefill(q, k, v, qw, kw, qk_norm=cfg.qk_norm, v_norm=cfg.v_norm,
                          rope_pairs=cfg.rope_pairs, rope_base=cfg.rope_theta, eps=cfg.eps,
                          scale=cfg.scale, window=win, Kc=Kc, Vc=Vc, cap=T, pos0=0, T=T, Hq=Hq,
                          Hkv=Hkv, D=D, rows=np.asarray(rows, np.int32), round_bf16=round_bf16)
