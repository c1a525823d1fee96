"""CPU tests of the oracle: pinned to the golden fixtures made by the reference's own CPU code,
cross-checked against that code live (when oracle/_ref is built), and against closed forms
(the unit cases of the reference's failure table, docs/B6_3_attention.md:700-711)."""
from __future__ import annotations

import hashlib
import pathlib

import numpy as np
import pytest

import oracle
from oracle import inputs as I
from apex_b200.configs import CONFIGS
from helpers import golden, manifest, oracle_decode_seq, oracle_prefill_rows

MAN = manifest()


def _sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


# ------------------------------------------------------------------ goldens (reference code)

@pytest.mark.parametrize("name", ["hnr_q_sliding", "hnr_k_full_cache", "hnr_v_cache"])
def test_head_norm_rope_matches_reference_golden(name):
    c = MAN[name]
    n = c["tokens"] * c["heads"] * c["head_dim"]
    x = oracle.bf16_to_f32(oracle.normal_bf16(n, c["seed"], 1))
    w = oracle.normal_bf16(c["head_dim"], c["seed"], 4, 0, 1.0, 0.1)
    assert _sha(x, w) == c["input_sha"], "synthetic-input generator drifted"
    out = np.full(c["out_len"], c["sentinel"], np.float32)
    oracle.head_norm_rope_f32(x, w, out, c["tokens"], c["heads"], c["head_dim"], c["has_weight"],
                              c["rope_pairs"], c["rope_base"], c["abs_pos"], c["ots"], c["ohs"], c["eps"])
    np.testing.assert_array_equal(out, golden(name))


@pytest.mark.parametrize("name", ["attn_f32_window16", "attn_f32_global"])
def test_attention_f32_matches_reference_golden(name):
    c = MAN[name]
    T, Hq, Hkv, hd, cap = c["tokens"], c["q_heads"], c["kv_heads"], c["head_dim"], c["capacity"]
    q = oracle.bf16_to_f32(oracle.normal_bf16(T * Hq * hd, c["seed"], 1)) * c["q_mul"]
    K = oracle.bf16_to_f32(oracle.normal_bf16(Hkv * cap * hd, c["seed"], 2)) * c["k_mul"]
    V = oracle.bf16_to_f32(oracle.normal_bf16(Hkv * cap * hd, c["seed"], 3))
    assert _sha(q, K, V) == c["input_sha"]
    out = oracle.attention_f32(q, K, V, T, Hq, Hkv, hd, cap, c["pos0"], c["window"], c["scale"])
    np.testing.assert_allclose(out.reshape(T, Hq, hd), golden(name), rtol=0, atol=1e-7)


def test_c1_decode_matches_reference_golden():
    cfg = CONFIGS["c1_decode"]
    out, _, _ = oracle_decode_seq(cfg, 0, cfg.context)
    np.testing.assert_allclose(out, golden("c1_decode")[0], rtol=0, atol=1e-7)


def test_c2_prefill_rows_match_reference_golden():
    cfg = CONFIGS["c2_prefill_window"]
    rows = MAN["c2_prefill_window"]["positions"]
    out = oracle_prefill_rows(cfg, 0, cfg.seq_len, rows)
    np.testing.assert_allclose(out, golden("c2_prefill_window"), rtol=0, atol=1e-7)


def test_c3_ragged_lengths_and_rows_match_reference_golden():
    cfg = CONFIGS["c3_ragged_decode"]
    lens = I.decode_lens(cfg)
    m = MAN["c3_ragged_decode"]
    assert _sha(lens) == m["lens_sha"]
    g = golden("c3_ragged_decode")
    for i, b in enumerate(m["seqs"][:3]):       # the three first sampled sequences (seconds)
        assert int(lens[b]) == m["lens"][i]
        out, _, _ = oracle_decode_seq(cfg, b, int(lens[b]))
        np.testing.assert_allclose(out, g[i], rtol=0, atol=1e-7)


# ------------------------------------------------------------------ live reference cross-check

ref_only = pytest.mark.skipif(oracle.ref_lib() is None, reason="reference tree not available to build oracle/_ref")


@ref_only
@pytest.mark.parametrize("head_dim,pairs,base,has_w,abs_pos", [
    (256, 128, 1e4, 1, 0), (512, 64, 1e6, 1, 131071), (128, 64, 1e4, 0, 5), (64, 0, 1e4, 1, 9), (96, 48, 1e6, 1, 3000)])
def test_head_norm_rope_equals_reference_code(head_dim, pairs, base, has_w, abs_pos):
    tokens, heads = 3, 5
    x = oracle.bf16_to_f32(oracle.normal_bf16(tokens * heads * head_dim, 7, head_dim))
    w = oracle.normal_bf16(head_dim, 7, 99, 0, 1.0, 0.1)
    a = np.zeros(tokens * heads * head_dim, np.float32)
    b = np.zeros_like(a)
    args = (tokens, heads, head_dim, has_w, pairs, base, abs_pos, heads * head_dim, head_dim, 1e-6)
    oracle.head_norm_rope_f32(x, w, a, *args)
    oracle.head_norm_rope_f32(x, w, b, *args, ref=True)
    np.testing.assert_array_equal(a, b)


@ref_only
@pytest.mark.parametrize("T,Hq,Hkv,hd,pos0,window", [(7, 16, 2, 512, 0, 0), (33, 4, 4, 64, 10, 5), (20, 8, 1, 32, 1000, 1)])
def test_attention_equals_reference_code(T, Hq, Hkv, hd, pos0, window):
    cap = pos0 + T
    q = oracle.bf16_to_f32(oracle.normal_bf16(T * Hq * hd, 11, 1)) * 0.2
    K = oracle.bf16_to_f32(oracle.normal_bf16(Hkv * cap * hd, 11, 2)) * 0.2
    V = oracle.bf16_to_f32(oracle.normal_bf16(Hkv * cap * hd, 11, 3))
    a = oracle.attention_f32(q, K, V, T, Hq, Hkv, hd, cap, pos0, window, 1.0)
    b = oracle.attention_f32(q, K, V, T, Hq, Hkv, hd, cap, pos0, window, 1.0, ref=True)
    np.testing.assert_allclose(a, b, rtol=0, atol=1e-7)


# ------------------------------------------------------------------ closed forms

def test_rope_at_position_zero_is_identity():
    x = np.random.default_rng(0).standard_normal(256).astype(np.float32)
    y = x.copy()
    oracle.lib().orc_rope(y, 256, 128, 1e4, 0)
    np.testing.assert_array_equal(x, y)


def test_rope_pairs_i_with_i_plus_half():
    x = np.zeros(8, np.float32)
    x[1] = 1.0                          # pair (1, 5) rotates; (0, 4) untouched by pairs=2 too
    oracle.lib().orc_rope(x, 8, 2, 1e4, 3)
    ang = 3 * 1e4 ** (-2 * 1 / 8)
    np.testing.assert_allclose([x[1], x[5]], [np.cos(ang), np.sin(ang)], rtol=1e-6)
    assert x[2] == 0 and x[3] == 0 and x[6] == 0


def test_rmsnorm_of_constant_vector():
    x = np.full(256, 3.0, np.float32)
    y = np.zeros_like(x)
    oracle.lib().orc_rms_norm(x, None, y, 256, 0.0)
    np.testing.assert_allclose(y, 1.0, rtol=1e-6)


def test_one_visible_key_returns_its_value():
    hd = 64
    q = np.random.default_rng(1).standard_normal(hd).astype(np.float32)
    K = np.random.default_rng(2).standard_normal(4 * hd).astype(np.float32)
    V = np.random.default_rng(3).standard_normal(4 * hd).astype(np.float32)
    out = np.zeros(hd, np.float32)
    oracle.lib().orc_attention_row(q, K, V, out, hd, 2, 2, 1.0)
    np.testing.assert_allclose(out, V[2 * hd:3 * hd], rtol=1e-6)


def test_gqa_head_map_and_window_edges():
    # q heads 2g and 2g+1 read kv head g; window W: the query at t sees t-W+1..t.
    T, Hq, Hkv, hd, W = 12, 4, 2, 16, 4
    rng = np.random.default_rng(4)
    q = rng.standard_normal(T * Hq * hd).astype(np.float32)
    K = rng.standard_normal(Hkv * T * hd).astype(np.float32)
    V = rng.standard_normal(Hkv * T * hd).astype(np.float32)
    out = oracle.attention_f32(q, K, V, T, Hq, Hkv, hd, T, 0, W, 0.7).reshape(T, Hq, hd)
    for t in (W - 1, W, W + 1, T - 1):
        for h in range(Hq):
            kvh = h // (Hq // Hkv)
            first = t + 1 - W if t + 1 > W else 0
            row = np.zeros(hd, np.float32)
            oracle.lib().orc_attention_row(np.ascontiguousarray(q.reshape(T, Hq, hd)[t, h]),
                                           np.ascontiguousarray(K.reshape(Hkv, T, hd)[kvh]).ravel(),
                                           np.ascontiguousarray(V.reshape(Hkv, T, hd)[kvh]).ravel(),
                                           row, hd, first, t, 0.7)
            np.testing.assert_allclose(out[t, h], row, rtol=1e-6, atol=1e-7)


def test_split_partials_merge_to_full_attention():
    hd, n = 32, 100
    rng = np.random.default_rng(5)
    q = rng.standard_normal(hd).astype(np.float32)
    K = rng.standard_normal(n * hd).astype(np.float32)
    V = rng.standard_normal(n * hd).astype(np.float32)
    full = np.zeros(hd, np.float32)
    oracle.lib().orc_attention_row(q, K, V, full, hd, 0, n - 1, 0.3)
    parts = np.stack([oracle.partial_row(q, K, V, hd, lo, hi, 0.3) for lo, hi in ((0, 17), (17, 64), (64, 100))])
    empty = np.zeros(hd + 2, np.float32)          # l = 0: a rank that holds no keys
    merged = oracle.merge_partials(np.concatenate([parts, empty[None]]), hd)
    np.testing.assert_allclose(merged, full, rtol=1e-5, atol=1e-6)


def test_generator_is_sliceable_and_standard_normal():
    a = oracle.normal_bf16(4096, 3, 2, offset=1000)
    b = oracle.normal_bf16(5096, 3, 2)[1000:]
    np.testing.assert_array_equal(a, b)
    x = oracle.bf16_to_f32(oracle.normal_bf16(1 << 20, 9, 1))
    assert abs(float(x.mean())) < 5e-3 and abs(float(x.std()) - 1.0) < 5e-3


def test_nvfp4_and_rms_norm_restatement_equals_reference_goldens():
    """The C restatement of matvecNvfp4Cpu / rmsNormCpu reproduces the goldens made by the
    reference's own code bit for bit, on the recorded inputs."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_goldens", pathlib.Path(__file__).parent / "golden" / "make_goldens.py")
    mg = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mg)
    man = manifest()
    for name, c in mg.PROJ_CASES.items():
        if name == "rms_norm_rows":
            x, w = mg.proj_inputs(name)
            assert mg.sha(x, w) == man[name]["input_sha"]
            got = oracle.rms_norm_rows(x, w, c["rows"], c["n"], 1e-6)
        else:
            codes, scales, x, w = mg.proj_inputs(name)
            assert mg.sha(codes, scales, x, w) == man[name]["input_sha"]
            got = oracle.matvec_nvfp4(codes, scales, x, c["tokens"], c["rows"], c["n"])
            if name == "oproj_post_norm":
                got = oracle.rms_norm_rows(got, w, c["tokens"], c["rows"], 1e-6)
        np.testing.assert_array_equal(got, golden(name))


def test_e2m1_e4m3_tables():
    L = oracle.lib()
    assert [L.orc_e2m1(c) for c in range(8)] == [0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0]
    assert [L.orc_e2m1(c | 8) for c in range(1, 8)] == [-0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0]
    assert L.orc_e4m3(0x38) == 1.0 and L.orc_e4m3(0x01) == 2.0 ** -9 and L.orc_e4m3(0x7E) == 448.0
    assert L.orc_e4m3(0xB8) == -1.0


def test_global_layer_restatement_vs_reference_golden():
    """Head_dim 512, partial RoPE, V norm: the restatement's decode composition against the goldens
    the reference's own CPU code made (the reference gate, rel-L2 < 1e-5)."""
    cfg = CONFIGS["global_decode"]
    g = golden("global_decode")
    for i, r in enumerate(manifest()["global_decode"]["rows"]):
        ref, _, _ = oracle_decode_seq(cfg, r["seq"], r["context"])
        _, rel = oracle.diff(ref, g[i])
        assert rel < 1e-5, rel
