"""Generate the golden fixtures in tests/golden/ from the reference's OWN CPU code.

The outputs come from oracle/_ref/libapexref.so: the reference's ``rmsNormCpu``
(src/tests/cpu_ref.h:14-25) and the ``ropeCpu`` / ``attentionRowCpu`` of
docs/B6_3_attention.md section 5, composed as the doc's ``attentionCpu`` does
(docs/B6_3_attention.md:643-670).  Inputs come from the seeded generator in
oracle/apex_oracle.c (index scheme in apex_b200/configs.py), so only outputs, arguments and
input checksums are stored.  Everything is f32 (the fp32 reference the tolerance is stated
against); files are ``<f4`` .npy, the format src/npy.h reads.

The NVFP4 projection and RMSNorm cases come from the reference's matvecNvfp4Cpu
(src/tests/cpu_ref.h:48-63, with src/nvfp4.h) and rmsNormCpu on seeded synthetic matrices.

Usage (needs the reference tree to build oracle/_ref):
    python tests/golden/make_goldens.py            # every case
    python tests/golden/make_goldens.py --only nvfp4_matvec,rms_norm_rows,oproj_post_norm
"""
from __future__ import annotations

import hashlib
import json
import pathlib
import sys

import numpy as np

ROOT = pathlib.Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

import oracle  # noqa: E402
from oracle import inputs as I  # noqa: E402
from apex_b200.configs import CONFIGS  # noqa: E402

OUT = pathlib.Path(__file__).resolve().parent


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()[:16]


def ref_cache(cfg, b, L, kw):
    """K cache [Hkv][L][D] = rope(rmsnorm(k, k_w)) and V cache = v (no norm), positions 0..L-1,
    through the reference's CPU ops; built in position blocks to bound memory."""
    R = oracle.ref_lib()
    Hkv, D = cfg.kv_heads, cfg.head_dim
    Kc = np.zeros(Hkv * L * D, np.float32)
    Vc = np.zeros((Hkv, L, D), np.float32)
    digest = hashlib.sha256()
    step = 8192
    for p0 in range(0, L, step):
        p1 = min(L, p0 + step)
        k = I.k_rows(cfg, b, p0, p1)
        v = I.v_rows(cfg, b, p0, p1)
        digest.update(k.tobytes())
        digest.update(v.tobytes())
        kf = oracle.bf16_to_f32(k).ravel()
        R.ref_head_norm_rope_f32(kf, kw, Kc[p0 * D:], p1 - p0, Hkv, D, 1, cfg.rope_pairs,
                                 cfg.rope_theta, p0, D, L * D, cfg.eps)
        Vc[:, p0:p1, :] = oracle.bf16_to_f32(v).transpose(1, 0, 2)
    return Kc, Vc.ravel(), digest.hexdigest()[:16]


def ref_query(cfg, b, pos, qw):
    """Normalised + roped q [Hq][D] at position pos of sequence b (reference CPU ops)."""
    R = oracle.ref_lib()
    q = oracle.bf16_to_f32(I.q_rows(cfg, b, pos, pos + 1)).ravel()
    qn = np.zeros_like(q)
    R.ref_head_norm_rope_f32(q, qw, qn, 1, cfg.q_heads, cfg.head_dim, 1, cfg.rope_pairs,
                             cfg.rope_theta, pos, cfg.q_heads * cfg.head_dim, cfg.head_dim, cfg.eps)
    return qn


def ref_rows(cfg, b, positions, L):
    """Outputs [len(positions)][Hq][D] for queries of sequence b at the given positions,
    attending the cache of length L (positions < L)."""
    qw, kw = I.norm_weights(cfg)
    Kc, Vc, kv_digest = ref_cache(cfg, b, L, kw)
    out = []
    for pos in positions:
        qn = ref_query(cfg, b, pos, qw)
        out.append(oracle.attention_f32(qn, Kc, Vc, 1, cfg.q_heads, cfg.kv_heads, cfg.head_dim,
                                        L, pos, cfg.window, cfg.scale, ref=True))
    return np.stack(out).reshape(len(positions), cfg.q_heads, cfg.head_dim), kv_digest


PROJ_CASES = {
    # (w_rows, hidden_dim, tokens, seed): a small matrix, and o_proj of a sliding layer (2816 x 4096)
    "nvfp4_matvec": dict(rows=48, n=256, tokens=3, seed=300),
    "rms_norm_rows": dict(rows=3, n=2816, seed=301),
    "oproj_post_norm": dict(rows=2816, n=4096, tokens=2, seed=302),
}


def proj_inputs(name):
    """Seeded inputs of a projection / norm case (also used by the tests)."""
    c = PROJ_CASES[name]
    if name == "rms_norm_rows":
        x = oracle.bf16_to_f32(oracle.normal_bf16(c["rows"] * c["n"], c["seed"], 1)).reshape(c["rows"], c["n"]) * 3.0
        w = oracle.normal_bf16(c["n"], c["seed"], 4, 0, 1.0, 0.1)
        return x, w
    codes, scales = oracle.nvfp4_matrix(c["rows"], c["n"], c["seed"])
    x = oracle.bf16_to_f32(oracle.normal_bf16(c["tokens"] * c["n"], c["seed"], 1)).reshape(c["tokens"], c["n"])
    w = oracle.normal_bf16(c["rows"], c["seed"], 4, 0, 1.0, 0.1)
    return codes, scales, x, w


def global_goldens(save):
    """Global-layer decode (head_dim 512, 2 kv heads, RoPE on 64 pairs, V normalised): the cache of
    sequence b built by the reference's head_norm_rope (K: weight + partial RoPE; V: weightless norm)
    and its attention row at the last position."""
    cfg = CONFIGS["global_decode"]
    R = oracle.ref_lib()
    Hq, Hkv, D = cfg.q_heads, cfg.kv_heads, cfg.head_dim
    qw, kw = I.norm_weights(cfg)
    outs, meta = [], []
    for b, L in ((0, 3000), (5, 17)):
        k = oracle.bf16_to_f32(I.k_rows(cfg, b, 0, L)).ravel()
        v = oracle.bf16_to_f32(I.v_rows(cfg, b, 0, L)).ravel()
        Kc = np.zeros(Hkv * L * D, np.float32)
        Vc = np.zeros(Hkv * L * D, np.float32)
        R.ref_head_norm_rope_f32(k, kw, Kc, L, Hkv, D, 1, cfg.rope_pairs, cfg.rope_theta, 0, D, L * D, cfg.eps)
        R.ref_head_norm_rope_f32(v, None, Vc, L, Hkv, D, 0, 0, cfg.rope_theta, 0, D, L * D, cfg.eps)
        qn = ref_query(cfg, b, L - 1, qw)
        out = oracle.attention_f32(qn, Kc, Vc, 1, Hq, Hkv, D, L, L - 1, cfg.window, cfg.scale, ref=True)
        outs.append(out.reshape(Hq, D))
        meta.append(dict(seq=b, context=L, kv_sha=sha(k, v)))
    save("global_decode", np.stack(outs), dict(config=cfg.name, rows=meta))


def proj_goldens(save):
    for name, c in PROJ_CASES.items():
        if name == "rms_norm_rows":
            x, w = proj_inputs(name)
            out = oracle.rms_norm_rows(x, w, c["rows"], c["n"], 1e-6, ref=True)
            save(name, out, dict(c, eps=1e-6, input_sha=sha(x, w)))
            continue
        codes, scales, x, w = proj_inputs(name)
        out = oracle.matvec_nvfp4(codes, scales, x, c["tokens"], c["rows"], c["n"], ref=True)
        if name == "oproj_post_norm":
            out = oracle.rms_norm_rows(out, w, c["tokens"], c["rows"], 1e-6, ref=True)
        save(name, out, dict(c, eps=1e-6, input_sha=sha(codes, scales, x, w)))


def main() -> int:
    if oracle.ref_lib() is None:
        print("reference tree not available: cannot build oracle/_ref", file=sys.stderr)
        return 1
    only = None
    if len(sys.argv) > 2 and sys.argv[1] == "--only":
        only = set(sys.argv[2].split(","))
    manifest = {"generator": "oracle/apex_oracle.c orc_fill_normal_bf16 (splitmix64 + Box-Muller)",
                "source": "oracle/_ref (reference cpu_ref.h + docs/B6_3_attention.md section 5)",
                "cases": {}}
    if only is not None:
        manifest = json.loads((OUT / "manifest.json").read_text())
    R = oracle.ref_lib()

    def save(name, arr, meta):
        np.save(OUT / f"{name}.npy", np.ascontiguousarray(arr, dtype="<f4"))
        manifest["cases"][name] = meta
        print(name, arr.shape)

    if only is not None:
        proj_goldens(lambda name, arr, meta: save(name, arr, meta) if name in only else None)
        global_goldens(lambda name, arr, meta: save(name, arr, meta) if name in only else None)
        (OUT / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
        return 0

    # 1. head_norm_rope_f32 -- the shipped kernel's semantics (shaders/head_norm_rope.metal).
    hnr = [
        # q in place layout: token stride heads*hd, head stride hd; full rope (sliding layer)
        dict(name="hnr_q_sliding", tokens=5, heads=16, head_dim=256, has_weight=1, rope_pairs=128,
             rope_base=1e4, abs_pos=37, ots=16 * 256, ohs=256, out_len=5 * 16 * 256, seed=100),
        # K into a cache [heads][cap=8][512] at pos0=1500; partial rope 64 pairs (full layer)
        dict(name="hnr_k_full_cache", tokens=3, heads=2, head_dim=512, has_weight=1, rope_pairs=64,
             rope_base=1e6, abs_pos=1500, ots=512, ohs=8 * 512, out_len=2 * 8 * 512, seed=101),
        # V: weightless norm, no rope, into a cache [8][cap=6][256]
        dict(name="hnr_v_cache", tokens=4, heads=8, head_dim=256, has_weight=0, rope_pairs=0,
             rope_base=1e4, abs_pos=0, ots=256, ohs=6 * 256, out_len=8 * 6 * 256, seed=102),
    ]
    for c in hnr:
        n = c["tokens"] * c["heads"] * c["head_dim"]
        x = oracle.bf16_to_f32(oracle.normal_bf16(n, c["seed"], 1))
        w = oracle.normal_bf16(c["head_dim"], c["seed"], 4, 0, 1.0, 0.1)
        out = np.full(c["out_len"], 7.0, np.float32)   # sentinel: untouched slots stay 7.0
        R.ref_head_norm_rope_f32(x, w, out, c["tokens"], c["heads"], c["head_dim"], c["has_weight"],
                                 c["rope_pairs"], c["rope_base"], c["abs_pos"], c["ots"], c["ohs"],
                                 1e-6)
        meta = {k: v for k, v in c.items() if k != "name"}
        meta.update(eps=1e-6, input_sha=sha(x, w), sentinel=7.0)
        save(c["name"], out, meta)

    # 2. attention_f32 -- the designed kernel (scale 1.0, f32 cache [Hkv][cap][hd]).
    for name, window in (("attn_f32_window16", 16), ("attn_f32_global", 0)):
        T, Hq, Hkv, hd, cap, pos0 = 40, 4, 2, 64, 48, 5
        q = oracle.bf16_to_f32(oracle.normal_bf16(T * Hq * hd, 200, 1)) * 0.25
        K = oracle.bf16_to_f32(oracle.normal_bf16(Hkv * cap * hd, 200, 2)) * 0.25
        V = oracle.bf16_to_f32(oracle.normal_bf16(Hkv * cap * hd, 200, 3))
        out = oracle.attention_f32(q, K, V, T, Hq, Hkv, hd, cap, pos0, window, 1.0, ref=True)
        save(name, out.reshape(T, Hq, hd),
             dict(tokens=T, q_heads=Hq, kv_heads=Hkv, head_dim=hd, capacity=cap, pos0=pos0,
                  window=window, scale=1.0, seed=200, q_mul=0.25, k_mul=0.25,
                  input_sha=sha(q, K, V)))

    # 3. The five benchmark configurations (bf16 inputs, f32 reference arithmetic).
    c1 = CONFIGS["c1_decode"]
    L = c1.context
    out, d = ref_rows(c1, 0, [L - 1], L)
    save("c1_decode", out, dict(config=c1.name, seq=0, positions=[L - 1], context=L, kv_sha=d))

    c2 = CONFIGS["c2_prefill_window"]
    rows = [0, 1, 2, 127, 128, 511, 1022, 1023, 1024, 1025, 1500, 2046, 2047, 777, 1337, 1999]
    out, d = ref_rows(c2, 0, rows, c2.seq_len)
    save("c2_prefill_window", out, dict(config=c2.name, seq=0, positions=rows, kv_sha=d))

    c3 = CONFIGS["c3_ragged_decode"]
    lens = I.decode_lens(c3)
    seqs = sorted({0, 1, 7, 21, int(np.argmin(lens)), int(np.argmax(lens)), 42, 63})
    outs, digests = [], []
    for b in seqs:
        o, d = ref_rows(c3, b, [int(lens[b]) - 1], int(lens[b]))
        outs.append(o[0])
        digests.append(d)
    save("c3_ragged_decode", np.stack(outs),
         dict(config=c3.name, seqs=seqs, lens=[int(lens[b]) for b in seqs], lens_sha=sha(lens),
              kv_sha=digests))

    c4 = CONFIGS["c4_chunked_prefill"]
    picks = {0: [0, 4095, 4096, 12287, 32767], 3: [8191, 20000, 28672]}
    outs, meta_rows = [], []
    for b, positions in picks.items():
        o, d = ref_rows(c4, b, positions, max(positions) + 1)
        outs.append(o)
        meta_rows.append(dict(seq=b, positions=positions, kv_sha=d))
    save("c4_chunked_prefill", np.concatenate(outs), dict(config=c4.name, rows=meta_rows))

    c5 = CONFIGS["c5_long_decode_b1"]
    L = c5.context
    out, d = ref_rows(c5, 0, [L - 1], L)
    save("c5_long_decode_b1", out, dict(config=c5.name, seq=0, positions=[L - 1], context=L, kv_sha=d))
    c5b = CONFIGS["c5_long_decode_b8"]
    out, d = ref_rows(c5b, 7, [L - 1], L)
    save("c5_long_decode_b8_seq7", out,
         dict(config=c5b.name, seq=7, positions=[L - 1], context=L, kv_sha=d))

    proj_goldens(save)
    global_goldens(save)
    (OUT / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
