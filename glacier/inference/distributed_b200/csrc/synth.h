// synth.h -- documented seeded synthetic inputs (host side).
//
// Streams: SplitMix64 output function applied at index i of a stream,
//   mix64(z)           = SplitMix64 finaliser
//   stream(seed, tag)  = mix64(seed + G*(tag+1)),  G = 0x9E3779B97F4A7C15
//   draw(s, i)         = mix64(s + G*(i+1))
//   uniform(s, i)      = ((draw >> 40) + 0.5) * 2^-24            in (0,1)
//   normal(s, i)       = sqrt(-2 ln u1) cos(2 pi u2), u1 = uniform(s,2i),
//                        u2 = uniform(s,2i+1), evaluated in double, rounded to f32
// Tensor tags: 1 = input activations, 2 = router, 3 = shared-expert gate,
// 1000 + 4e + m = expert e matrix m (0 gate/W1, 1 up/W3, 2 down/W2); the shared
// expert uses e = 65535.
// Q4_K super-block b of a matrix stream s: d = fp16(|sigma_d * normal(s,2b)|),
// dmin = fp16(|sigma_d * normal(s,2b+1)|), and bytes 4..143 (scales + quants)
// are bytes 0..139 of draws 18b..18b+17 of stream mix64(s ^ 0xD1B54A32D192ED03),
// little-endian.
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace glc {

uint64_t mix64(uint64_t z);
uint64_t stream_seed(uint64_t seed, uint64_t tag);
float normal_at(uint64_t stream, uint64_t i);
uint16_t f32_to_f16_host(float f);
uint64_t expert_tag(int expert, int matrix);
constexpr uint64_t kTagInput = 1, kTagRouter = 2, kTagSharedGate = 3;
constexpr int kSharedExpertIndex = 65535;

void synth_normal(uint64_t seed, uint64_t tag, float sigma, float* out, size_t n, int nthreads);
void synth_q4k(uint64_t seed, uint64_t tag, float sigma_d, uint8_t* out, size_t n_blocks,
               int nthreads);

}  // namespace glc
