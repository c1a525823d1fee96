// sha256.h -- SHA-256 (FIPS 180-4) for checking packed weights against the manifest's digests.
// The round constants and the initial state are the first 32 fractional bits of the cube roots
// of the first 64 primes and of the square roots of the first 8 primes (FIPS 180-4 4.2.2 and
// 5.3.3); they are computed once here from that definition.  Streaming: update() any number of
// times, then hex().
#pragma once

#include <cmath>
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <string>

namespace apex {

class Sha256 {
  public:
    Sha256() { reset(); }

    void reset() {
        const Tables &t = tables();
        std::memcpy(h_, t.h0, sizeof(h_));
        len_ = 0;
        fill_ = 0;
    }

    void update(const void *data, size_t n) {
        const uint8_t *p = static_cast<const uint8_t *>(data);
        len_ += n;
        if (fill_) {
            const size_t take = n < 64 - fill_ ? n : 64 - fill_;
            std::memcpy(buf_ + fill_, p, take);
            fill_ += take;
            p += take;
            n -= take;
            if (fill_ < 64) return;
            block(buf_);
            fill_ = 0;
        }
        for (; n >= 64; n -= 64, p += 64) block(p);
        std::memcpy(buf_, p, n);
        fill_ = n;
    }

    // Finishes the message and returns the digest as 64 lowercase hex characters.
    std::string hex() {
        const uint64_t bits = len_ * 8;
        const uint8_t one = 0x80, zero = 0;
        update(&one, 1);
        while (fill_ != 56) update(&zero, 1);
        uint8_t be[8];
        for (int i = 0; i < 8; ++i) be[i] = static_cast<uint8_t>(bits >> (56 - 8 * i));
        update(be, 8);
        static const char *digits = "0123456789abcdef";
        std::string out(64, '0');
        for (int i = 0; i < 8; ++i)
            for (int j = 0; j < 8; ++j) out[8 * i + j] = digits[(h_[i] >> (28 - 4 * j)) & 0xF];
        return out;
    }

  private:
    struct Tables {
        uint32_t k[64];
        uint32_t h0[8];
        Tables() {
            int primes[64], n = 0;
            for (int c = 2; n < 64; ++c) {
                bool prime = true;
                for (int d = 2; d * d <= c; ++d)
                    if (c % d == 0) {
                        prime = false;
                        break;
                    }
                if (prime) primes[n++] = c;
            }
            for (int i = 0; i < 64; ++i) k[i] = frac32(std::cbrt(static_cast<long double>(primes[i])));
            for (int i = 0; i < 8; ++i) h0[i] = frac32(std::sqrt(static_cast<long double>(primes[i])));
        }
        static uint32_t frac32(long double x) {
            const long double f = x - std::floor(x);
            return static_cast<uint32_t>(std::floor(f * 4294967296.0L));
        }
    };
    static const Tables &tables() {
        static const Tables t;
        return t;
    }
    static uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

    void block(const uint8_t *p) {
        const Tables &t = tables();
        uint32_t w[64];
        for (int i = 0; i < 16; ++i)
            w[i] = (uint32_t(p[4 * i]) << 24) | (uint32_t(p[4 * i + 1]) << 16) | (uint32_t(p[4 * i + 2]) << 8) |
                   uint32_t(p[4 * i + 3]);
        for (int i = 16; i < 64; ++i) {
            const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
            const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
            w[i] = w[i - 16] + s0 + w[i - 7] + s1;
        }
        uint32_t a = h_[0], b = h_[1], c = h_[2], d = h_[3], e = h_[4], f = h_[5], g = h_[6], h = h_[7];
        for (int i = 0; i < 64; ++i) {
            const uint32_t S1 = rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25);
            const uint32_t ch = (e & f) ^ (~e & g);
            const uint32_t t1 = h + S1 + ch + t.k[i] + w[i];
            const uint32_t S0 = rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22);
            const uint32_t maj = (a & b) ^ (a & c) ^ (b & c);
            const uint32_t t2 = S0 + maj;
            h = g;
            g = f;
            f = e;
            e = d + t1;
            d = c;
            c = b;
            b = a;
            a = t1 + t2;
        }
        h_[0] += a; h_[1] += b; h_[2] += c; h_[3] += d;
        h_[4] += e; h_[5] += f; h_[6] += g; h_[7] += h;
    }

    uint32_t h_[8];
    uint64_t len_ = 0;
    uint8_t buf_[64];
    size_t fill_ = 0;
};

}  // namespace apex
