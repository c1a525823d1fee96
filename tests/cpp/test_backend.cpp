// test_backend.cpp -- C++ parity harness over the drop-in boundary: CudaBackend + ops.h
// driven the way the reference's tests drive MetalBackend + its ops (src/tests/test_norm.cpp:
// 17-112, the designed run_test_attn of docs/B6_3_attention.md:527-599): allocate buffers,
// memcpy inputs into contents(), queue ops, sync(), compare with the CPU oracle.
// TEST INFRASTRUCTURE: links the oracle (oracle/apex_oracle.c) as the checker.
//
// Prints one line per case and returns the number of failures (the reference's convention).
#include <cmath>
#include <cstdio>
#include <cstring>
#include <random>
#include <string>
#include <vector>

#include "backend/cuda/cuda_backend.h"
#include "ops.h"

extern "C" {
uint16_t orc_f32_to_bf16(float f);
float orc_bf16_to_f32(uint16_t h);
void orc_head_norm_rope_f32(const float *, const uint16_t *, float *, uint32_t, uint32_t, uint32_t, uint32_t,
                            uint32_t, float, uint32_t, uint32_t, uint32_t, float);
void orc_attention_f32(const float *, const float *, const float *, float *, uint32_t, uint32_t, uint32_t,
                       uint32_t, uint32_t, uint32_t, uint32_t, float);
void orc_kv_append(const float *, const uint16_t *, int, uint32_t, float, float, float *, uint32_t, uint32_t,
                   uint32_t, uint32_t, uint32_t, int);
void orc_prefill(const float *, const float *, const float *, const uint16_t *, const uint16_t *, int, int,
                 uint32_t, float, float, float, uint32_t, float *, float *, uint32_t, uint32_t, uint32_t, uint32_t,
                 uint32_t, uint32_t, const int32_t *, uint32_t, float *, int);
void orc_matvec_nvfp4(const uint32_t *, const uint8_t *, const float *, float *, size_t, size_t, size_t);
void orc_rms_norm_rows(const float *, const uint16_t *, float *, size_t, size_t, float);
}

namespace {

struct Diff {
    double max_abs = 0, rel_l2 = 0, mean_abs = 0;
};

Diff diff(const float *a, const float *b, size_t n) {
    double num = 0, den = 0, sum = 0;
    Diff d;
    for (size_t i = 0; i < n; ++i) {
        if (!std::isfinite(a[i]) || !std::isfinite(b[i])) return {INFINITY, INFINITY, INFINITY};
        const double e = double(a[i]) - b[i];
        num += e * e;
        den += double(b[i]) * b[i];
        sum += std::fabs(e);
        d.max_abs = std::max(d.max_abs, std::fabs(e));
    }
    d.rel_l2 = den > 0 ? std::sqrt(num / den) : std::sqrt(num);
    d.mean_abs = n ? sum / n : 0;
    return d;
}

std::vector<float> normal(size_t n, uint32_t seed, float scale = 1.f) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> nd(0.f, 1.f);
    std::vector<float> v(n);
    for (auto &x : v) x = orc_bf16_to_f32(orc_f32_to_bf16(nd(rng) * scale));  // bf16-exact values
    return v;
}

std::vector<uint16_t> weights(size_t n, uint32_t seed) {
    std::mt19937 rng(seed);
    std::normal_distribution<float> nd(1.f, 0.1f);
    std::vector<uint16_t> w(n);
    for (auto &x : w) x = orc_f32_to_bf16(nd(rng));
    return w;
}

apex::Buffer *upload(apex::Backend &be, const void *src, size_t bytes, const char *cat) {
    apex::Buffer *b = be.allocate(bytes, cat);
    std::memcpy(be.contents(b), src, bytes);
    return b;
}

int failures = 0;

void report(const char *name, const Diff &d, bool ok) {
    failures += !ok;
    std::printf("%-44s rel %.2e max %.2e mean %.2e  %s\n", name, d.rel_l2, d.max_abs, d.mean_abs, ok ? "ok" : "FAIL");
}

// headNormRope on q in place and K/V into a cache layout, f32 (the reference kernel's uses).
void test_head_norm_rope(apex::CudaBackend &be) {
    const uint32_t T = 7, H = 16, hd = 256, cap = 12, pos0 = 3;
    auto x = normal(size_t(T) * H * hd, 1);
    auto w = weights(hd, 2);
    apex::Buffer *in = upload(be, x.data(), x.size() * 4, "activations");
    apex::Buffer *wb = upload(be, w.data(), w.size() * 2, "weights");
    // q in place
    apex::headNormRope(be, in, wb, 0, true, in, 0, T, H, hd, 128, 1e4f, pos0, H * hd, hd, 1e-6f);
    // K into a [H][cap][hd] cache at pos0 (byte offset), partial RoPE, hd 256
    auto k = normal(size_t(T) * H * hd, 3);
    apex::Buffer *kb = upload(be, k.data(), k.size() * 4, "activations");
    apex::Buffer *cache = be.allocate(size_t(H) * cap * hd * 4, "kv_cache");
    std::memset(be.contents(cache), 0, size_t(H) * cap * hd * 4);
    apex::headNormRope(be, kb, wb, 0, true, cache, size_t(pos0) * hd * 4, T, H, hd, 64, 1e6f, pos0, hd, cap * hd,
                       1e-6f);
    be.sync();
    std::vector<float> ref(x.size()), cref(size_t(H) * cap * hd, 0.f);
    orc_head_norm_rope_f32(x.data(), w.data(), ref.data(), T, H, hd, 1, 128, 1e4f, pos0, H * hd, hd, 1e-6f);
    orc_head_norm_rope_f32(k.data(), w.data(), cref.data() + size_t(pos0) * hd, T, H, hd, 1, 64, 1e6f, pos0, hd,
                           cap * hd, 1e-6f);
    Diff d = diff(static_cast<float *>(be.contents(in)), ref.data(), ref.size());
    report("headNormRope q in place (f32)", d, d.rel_l2 < 1e-5);
    d = diff(static_cast<float *>(be.contents(cache)), cref.data(), cref.size());
    report("headNormRope K -> cache at pos0 (f32)", d, d.rel_l2 < 1e-5);
    for (auto *b : {in, wb, kb, cache}) be.release(b);
}

// attentionAfterProjections: the doc's attentionBlock body on f32, both Gemma layer kinds.
void test_attention_block(apex::CudaBackend &be, bool full) {
    const uint32_t T = 200;
    const apex::AttentionShape s = full ? apex::AttentionShape{16, 2, 512, 64, 1e6f, 0}
                                        : apex::AttentionShape{16, 8, 256, 128, 1e4f, 64};
    const uint32_t hd = s.head_dim, nq = s.q_heads, nkv = s.kv_heads, cap = T;
    auto q = normal(size_t(T) * nq * hd, 11);
    auto k = normal(size_t(T) * nkv * hd, 12);
    auto v = normal(size_t(T) * nkv * hd, 13);
    auto qw = weights(hd, 14), kw = weights(hd, 15);
    std::vector<uint16_t> norms(qw);
    norms.insert(norms.end(), kw.begin(), kw.end());
    apex::Buffer *qb = upload(be, q.data(), q.size() * 4, "activations");
    apex::Buffer *kb = upload(be, k.data(), k.size() * 4, "activations");
    apex::Buffer *vb = upload(be, v.data(), v.size() * 4, "activations");
    apex::Buffer *nb = upload(be, norms.data(), norms.size() * 2, "weights");
    apex::KvCache cache{be.allocate(size_t(nkv) * cap * hd * 4, "kv_cache"), be.allocate(size_t(nkv) * cap * hd * 4, "kv_cache"), cap};
    apex::Buffer *o = be.allocate(size_t(T) * nq * hd * 4, "activations");
    apex::attentionAfterProjections(be, qb, kb, vb, nb, 0, hd * 2, s, cache, o, T, 0, 1e-6f);
    be.sync();
    // CPU: the doc's attentionCpu steps (docs/B6_3_attention.md:643-670), scale 1.0
    std::vector<float> qn(q.size()), K(size_t(nkv) * cap * hd), V(K.size()), out(q.size());
    orc_head_norm_rope_f32(q.data(), qw.data(), qn.data(), T, nq, hd, 1, s.rope_pairs, s.rope_base, 0, nq * hd, hd, 1e-6f);
    orc_kv_append(k.data(), kw.data(), 1, s.rope_pairs, s.rope_base, 1e-6f, K.data(), cap, 0, T, nkv, hd, 0);
    orc_kv_append(v.data(), nullptr, 1, 0, s.rope_base, 1e-6f, V.data(), cap, 0, T, nkv, hd, 0);
    orc_attention_f32(qn.data(), K.data(), V.data(), out.data(), T, nq, nkv, hd, cap, 0, s.window, 1.0f);
    const Diff d = diff(static_cast<float *>(be.contents(o)), out.data(), out.size());
    report(full ? "attention block, full layer (f32, hd 512)" : "attention block, sliding layer (f32)", d,
           d.rel_l2 < 1e-5);
    for (auto *b : {qb, kb, vb, nb, cache.k, cache.v, o}) be.release(b);
}

// bf16 fused prefill then one decode step through ops.h, vs the fp32 oracle.
void test_bf16_prefill_decode(apex::CudaBackend &be) {
    const uint32_t T = 333, Hq = 16, Hkv = 8, D = 256, cap = T + 1;
    const apex::AttentionShape s{Hq, Hkv, D, D / 2, 1e4f, 100};
    const apex_attn_params p = apex::attnParams(s, 1.0f / 16, 1e-6f, true, false);
    auto q = normal(size_t(cap) * Hq * D, 21), k = normal(size_t(cap) * Hkv * D, 22), v = normal(size_t(cap) * Hkv * D, 23);
    auto qw = weights(D, 24), kw = weights(D, 25);
    auto bf = [](const std::vector<float> &f, size_t off, size_t n) {
        std::vector<uint16_t> r(n);
        for (size_t i = 0; i < n; ++i) r[i] = orc_f32_to_bf16(f[off + i]);
        return r;
    };
    auto qh = bf(q, 0, size_t(T) * Hq * D), kh = bf(k, 0, size_t(T) * Hkv * D), vh = bf(v, 0, size_t(T) * Hkv * D);
    apex::Buffer *qb = upload(be, qh.data(), qh.size() * 2, "activations");
    apex::Buffer *kb = upload(be, kh.data(), kh.size() * 2, "activations");
    apex::Buffer *vb = upload(be, vh.data(), vh.size() * 2, "activations");
    apex::Buffer *qwb = upload(be, qw.data(), D * 2, "weights");
    apex::Buffer *kwb = upload(be, kw.data(), D * 2, "weights");
    apex::KvCacheBf16 cache{be.allocate(size_t(Hkv) * cap * D * 2, "kv_cache"), be.allocate(size_t(Hkv) * cap * D * 2, "kv_cache"), cap};
    apex::Buffer *o = be.allocate(size_t(T) * Hq * D * 2, "activations");
    apex::Buffer *ws = be.allocate(apex::prefillWorkspaceBytes(p, 1, T), "scratch");
    apex::attentionPrefillBf16(be, p, qb, kb, vb, qwb, kwb, cache, 1, T, 0, o, ws);
    // decode the token at position T on top of the prefilled cache
    auto qd = bf(q, size_t(T) * Hq * D, size_t(Hq) * D), kd = bf(k, size_t(T) * Hkv * D, size_t(Hkv) * D),
         vd = bf(v, size_t(T) * Hkv * D, size_t(Hkv) * D);
    apex::Buffer *qdb = upload(be, qd.data(), qd.size() * 2, "activations");
    apex::Buffer *kdb = upload(be, kd.data(), kd.size() * 2, "activations");
    apex::Buffer *vdb = upload(be, vd.data(), vd.size() * 2, "activations");
    const int32_t L = int32_t(cap);
    apex::Buffer *lens = upload(be, &L, 4, "activations");
    apex::Buffer *od = be.allocate(size_t(Hq) * D * 2, "activations");
    const size_t wsb = apex::decodeWorkspaceBytes(p, 1, cap);
    apex::Buffer *wsd = be.allocate(wsb, "scratch");
    std::memset(be.contents(wsd), 0, wsb);
    apex::attentionDecodeBf16(be, p, qdb, kdb, vdb, qwb, kwb, cache, lens, 1, cap, od, wsd);
    be.sync();
    std::vector<float> Kc(size_t(Hkv) * cap * D), Vc(Kc.size()), ref(size_t(cap) * Hq * D);
    orc_prefill(q.data(), k.data(), v.data(), qw.data(), kw.data(), 1, 0, D / 2, 1e4f, 1e-6f, 1.0f / 16, 100,
                Kc.data(), Vc.data(), cap, 0, cap, Hq, Hkv, D, nullptr, 0, ref.data(), 0);
    auto to_f32 = [&](apex::Buffer *b, size_t n) {
        std::vector<float> r(n);
        const auto *h = static_cast<const uint16_t *>(be.contents(b));
        for (size_t i = 0; i < n; ++i) r[i] = orc_bf16_to_f32(h[i]);
        return r;
    };
    auto gp = to_f32(o, size_t(T) * Hq * D);
    Diff d = diff(gp.data(), ref.data(), gp.size());
    report("bf16 fused prefill (tcgen05) vs fp32 oracle", d, d.max_abs <= 2e-2 && d.mean_abs <= 2e-3);
    auto gd = to_f32(od, size_t(Hq) * D);
    d = diff(gd.data(), ref.data() + size_t(T) * Hq * D, gd.size());
    report("bf16 fused decode (split-KV) vs fp32 oracle", d, d.max_abs <= 2e-2 && d.mean_abs <= 2e-3);
    for (auto *b : {qb, kb, vb, qwb, kwb, cache.k, cache.v, o, ws, qdb, kdb, vdb, lens, od, wsd}) be.release(b);
}

// The reference's test-norm / test-mlp call pattern (src/tests/test_norm.cpp:67-71,
// src/tests/dense_mlp.cpp:92-96): rmsNorm, then matmulNvfp4 with codes and scales at offsets in one
// weight buffer, queued through the Backend and compared after sync() with the reference gate.
void test_norm_and_nvfp4(apex::CudaBackend &be) {
    const uint32_t T = 3, H = 2816, R = 200;
    auto x = normal(size_t(T) * H, 31, 2.f);
    auto nw = weights(H, 32);
    std::mt19937 rng(33);
    std::vector<uint32_t> codes(size_t(R) * H / 8);
    for (auto &c : codes) c = rng();
    std::vector<uint8_t> scales(size_t(R) * H / 16);
    for (auto &sc : scales) sc = uint8_t(0x20 + rng() % 0x20);
    // one weight buffer: norm weight, then codes, then scales (offsets as core.bin would give them)
    const size_t off_codes = 16384, off_scales = off_codes + codes.size() * 4;
    std::vector<uint8_t> blob(off_scales + scales.size(), 0);
    std::memcpy(blob.data(), nw.data(), nw.size() * 2);
    std::memcpy(blob.data() + off_codes, codes.data(), codes.size() * 4);
    std::memcpy(blob.data() + off_scales, scales.data(), scales.size());
    apex::Buffer *wb = upload(be, blob.data(), blob.size(), "weights");
    apex::Buffer *in = upload(be, x.data(), x.size() * 4, "activations");
    apex::Buffer *normed = be.allocate(x.size() * 4, "activations");
    apex::Buffer *out = be.allocate(size_t(T) * R * 4, "activations");
    apex::rmsNorm(be, in, wb, 0, normed, T, H, 1e-6f);
    const apex::Nvfp4Matrix W{wb, off_codes, wb, off_scales, R, H};
    apex::matmulNvfp4(be, normed, W, out, T);
    be.sync();
    std::vector<float> nref(x.size()), oref(size_t(T) * R);
    orc_rms_norm_rows(x.data(), nw.data(), nref.data(), T, H, 1e-6f);
    orc_matvec_nvfp4(codes.data(), scales.data(), nref.data(), oref.data(), T, R, H);
    Diff d = diff(static_cast<float *>(be.contents(normed)), nref.data(), nref.size());
    report("rmsNorm (f32, hidden 2816)", d, d.rel_l2 < 1e-5);
    d = diff(static_cast<float *>(be.contents(out)), oref.data(), oref.size());
    report("matmulNvfp4 (f32 in/out, offsets in one buffer)", d, d.rel_l2 < 1e-5);
    for (auto *b : {wb, in, normed, out}) be.release(b);
}

}  // namespace

int main() {
    try {
        apex::CudaBackend backend;
        std::printf("device: %s\n", backend.deviceName());
        test_head_norm_rope(backend);
        test_attention_block(backend, false);
        test_attention_block(backend, true);
        test_bf16_prefill_decode(backend);
        test_norm_and_nvfp4(backend);
        apex::PhaseTable::get().print(stdout);
        apex::MemoryLedger::get().print(stdout);
    } catch (const std::exception &e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 100;
    }
    std::printf("%d failures\n", failures);
    return failures;
}
