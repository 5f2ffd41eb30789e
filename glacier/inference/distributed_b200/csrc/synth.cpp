// synth.cpp -- seeded synthetic weights and activations (see synth.h for the
// generator definition).  Built with -ffp-contract=off; every value depends
// only on (seed, tag, index), never on the thread count.
#include "synth.h"

#include <cmath>
#include <cstring>
#include <thread>
#include <vector>

namespace glc {

static constexpr uint64_t kGamma = 0x9E3779B97F4A7C15ull;

uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
uint64_t stream_seed(uint64_t seed, uint64_t tag) { return mix64(seed + kGamma * (tag + 1)); }
static inline uint64_t draw(uint64_t s, uint64_t i) { return mix64(s + kGamma * (i + 1)); }
static inline float uniform_at(uint64_t s, uint64_t i) {
    return ((float)(draw(s, i) >> 40) + 0.5f) * 5.9604644775390625e-8f;
}
float normal_at(uint64_t s, uint64_t i) {
    const float u1 = uniform_at(s, 2 * i);
    const float u2 = uniform_at(s, 2 * i + 1);
    const double r = std::sqrt(-2.0 * std::log((double)u1));
    const double th = 6.283185307179586 * (double)u2;
    return (float)(r * std::cos(th));
}
uint64_t expert_tag(int expert, int matrix) { return 1000ull + 4ull * (uint64_t)expert + (uint64_t)matrix; }

// binary16 round-to-nearest-even of a finite or non-finite float.
uint16_t f32_to_f16_host(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFFu) return (uint16_t)(man ? (sign | 0x7E00u | (man >> 13)) : (sign | 0x7C00u));
    const int e = (int)exp - 112;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        const int shift = 14 - e;
        uint32_t hm = man >> shift;
        const uint32_t rem = man & ((1u << shift) - 1u);
        const uint32_t half = 1u << (shift - 1);
        if (rem > half || (rem == half && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rem = man & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)h;
}

template <class F>
static void parallel_for(size_t n, int nthreads, F&& f) {
    if (nthreads <= 1 || n < 4096) {
        f(0, n);
        return;
    }
    std::vector<std::thread> th;
    for (int t = 0; t < nthreads; ++t) {
        const size_t a = n * t / nthreads, b = n * (t + 1) / nthreads;
        th.emplace_back([&f, a, b] { f(a, b); });
    }
    for (auto& x : th) x.join();
}

void synth_normal(uint64_t seed, uint64_t tag, float sigma, float* out, size_t n, int nthreads) {
    const uint64_t s = stream_seed(seed, tag);
    parallel_for(n, nthreads, [&](size_t a, size_t b) {
        for (size_t i = a; i < b; ++i) out[i] = sigma * normal_at(s, i);
    });
}

void synth_q4k(uint64_t seed, uint64_t tag, float sigma_d, uint8_t* out, size_t n_blocks, int nthreads) {
    const uint64_t s = stream_seed(seed, tag);
    const uint64_t sb = mix64(s ^ 0xD1B54A32D192ED03ull);
    parallel_for(n_blocks, nthreads, [&](size_t a, size_t b) {
        uint8_t tmp[144];
        for (size_t blk = a; blk < b; ++blk) {
            uint8_t* o = out + blk * 144;
            const uint16_t d = f32_to_f16_host(std::fabs(sigma_d * normal_at(s, 2 * blk)));
            const uint16_t dm = f32_to_f16_host(std::fabs(sigma_d * normal_at(s, 2 * blk + 1)));
            o[0] = (uint8_t)d; o[1] = (uint8_t)(d >> 8);
            o[2] = (uint8_t)dm; o[3] = (uint8_t)(dm >> 8);
            for (int j = 0; j < 18; ++j) {
                const uint64_t v = draw(sb, 18 * blk + j);
                for (int t = 0; t < 8; ++t) tmp[8 * j + t] = (uint8_t)(v >> (8 * t));
            }
            std::memcpy(o + 4, tmp, 140);
        }
    });
}

}  // namespace glc
