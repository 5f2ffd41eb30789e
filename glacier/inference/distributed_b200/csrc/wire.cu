// wire.cu -- stage-boundary activation codec on sm_100a, bit-exact with
// QuantizationKernels (Protocol/QuantizationKernels.cs):
//   INT8_Symmetric  [f32 scale LE][D x int8]  (:222-474, dequant :479-586)
//   FP8_E4M3        [f32 scale LE][D x e4m3]  (:593-736)
//   FP16            [D x binary16]            (:184-201)
//   FP32            [D x f32]                 (:169-178)
// One CTA per token; tokens are contiguous at GetPackedTokenBytes(mode, D)
// (:57-67).  Divisions, products and rounding use the IEEE round-to-nearest
// intrinsics so the bytes match the reference's scalar and SIMD paths.
#include "common.cuh"
#include "kernels.h"

namespace glc {

constexpr int kWireThreads = 256;

__host__ __device__ inline int wire_token_bytes(int mode, int dim) {
    switch (mode) {
        case 0: return dim * 4;
        case 1: return dim * 2;
        case 2: return dim + 4;
        case 3: return dim + 4;
        default: return dim * 2;
    }
}

// binary16 round-to-nearest-even; NaN keeps the top payload bits, quiet bit set.
__device__ __forceinline__ uint16_t f32_to_f16_bits(float f) {
    const uint32_t x = __float_as_uint(f);
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

__device__ __forceinline__ uint8_t f32_to_e4m3(float val) {
    const uint32_t bits = __float_as_uint(val);
    const uint8_t sign = (uint8_t)((bits >> 24) & 0x80u);
    const uint32_t ab = bits & 0x7FFFFFFFu;
    if (ab == 0 || ab > 0x7F800000u) return 0;
    if (ab >= 0x43E00000u) return (uint8_t)(sign | 0x7E);
    if (ab < 0x3C800000u) {
        const int sub = __float2int_rn(__fmul_rn(__uint_as_float(ab), 512.0f));
        if (sub <= 0) return sign;
        if (sub >= 8) return (uint8_t)(sign | 0x08);
        return (uint8_t)(sign | sub);
    }
    int e4 = (int)(ab >> 23) - 120;
    const uint32_t m23 = ab & 0x7FFFFFu;
    uint32_t m3 = m23 >> 20;
    const uint32_t rem = m23 & 0xFFFFFu;
    if (rem > 0x80000u || (rem == 0x80000u && (m3 & 1u))) {
        m3++;
        if (m3 >= 8u) { m3 = 0; e4++; }
    }
    if (e4 >= 15 && m3 >= 7u) { e4 = 15; m3 = 6u; }
    return (uint8_t)(sign | (e4 << 3) | (int)m3);
}

// E4M3FN decode (table of QuantizationKernels.cs:23-51; NaN -> 0).  Every
// entry is an exact power of two times an exact fraction.
__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
    const float sign = (b & 0x80) ? -1.0f : 1.0f;
    const int exp = (b >> 3) & 0x0F, mant = b & 0x07;
    if (exp == 15 && mant == 7) return 0.0f;
    if (exp == 0) return sign * ((float)mant * (1.0f / 512.0f));
    return sign * (ldexpf(1.0f, exp - 7) * (1.0f + (float)mant * 0.125f));
}

__device__ __forceinline__ void put_f32_le(uint8_t* p, float f) {
    const uint32_t u = __float_as_uint(f);
    p[0] = (uint8_t)u; p[1] = (uint8_t)(u >> 8); p[2] = (uint8_t)(u >> 16); p[3] = (uint8_t)(u >> 24);
}
__device__ __forceinline__ float get_f32_le(const uint8_t* p) {
    return __uint_as_float((uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) |
                           ((uint32_t)p[3] << 24));
}

__global__ void __launch_bounds__(kWireThreads) wire_quantize_kernel(int mode, const float* __restrict__ x,
                                                                    int D, uint8_t* __restrict__ out) {
    __shared__ float smax[kWireThreads / 32];
    __shared__ int snan[kWireThreads / 32];
    __shared__ float s_inv, s_scale;
    __shared__ int s_zero;
    const int t = blockIdx.x, tid = threadIdx.x;
    const float* xt = x + (size_t)t * D;
    uint8_t* o = out + (size_t)t * wire_token_bytes(mode, D);
    if (mode == 0) {
        for (int i = tid; i < D; i += kWireThreads) put_f32_le(o + 4 * i, xt[i]);
        return;
    }
    if (mode != 2 && mode != 3) {
        for (int i = tid; i < D; i += kWireThreads) {
            const uint16_t h = f32_to_f16_bits(xt[i]);
            o[2 * i] = (uint8_t)h;
            o[2 * i + 1] = (uint8_t)(h >> 8);
        }
        return;
    }
    // FindMaxAbsolute: |MaxMagnitude(x)|, NaN propagates (QuantizationKernels.cs:212-216).
    float m = 0.f;
    int nan = 0;
    for (int i = tid; i < D; i += kWireThreads) {
        const float a = fabsf(xt[i]);
        if (isnan(a)) nan = 1;
        else m = fmaxf(m, a);
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) {
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
        nan |= __shfl_xor_sync(0xffffffffu, nan, off);
    }
    if ((tid & 31) == 0) { smax[tid >> 5] = m; snan[tid >> 5] = nan; }
    __syncthreads();
    if (tid == 0) {
        float mx = 0.f;
        int any_nan = 0;
        for (int w = 0; w < kWireThreads / 32; ++w) { mx = fmaxf(mx, smax[w]); any_nan |= snan[w]; }
        const float qmax = (mode == 2) ? 127.0f : 448.0f;
        int zero = any_nan || !isfinite(mx) || mx < 1e-10f;
        float scale = 1.0f, inv = 0.f;
        if (!zero) {
            scale = __fdiv_rn(mx, qmax);
            inv = __fdiv_rn(qmax, mx);
            if (!isfinite(scale) || !isfinite(inv) || scale <= 0.0f) { zero = 1; scale = 1.0f; }
        }
        s_zero = zero;
        s_scale = zero ? 1.0f : scale;
        s_inv = inv;
        put_f32_le(o, s_scale);
    }
    __syncthreads();
    const int zero = s_zero;
    const float inv = s_inv;
    uint8_t* q = o + 4;
    for (int i = tid; i < D; i += kWireThreads) {
        uint8_t b = 0;
        if (!zero) {
            const float v = __fmul_rn(xt[i], inv);
            if (mode == 2) {
                // clamp(round-half-even(v), -127, 127)
                const float c = fminf(fmaxf(v, -127.0f), 127.0f);
                b = (uint8_t)(int8_t)__float2int_rn(c);
            } else {
                b = f32_to_e4m3(v);
            }
        }
        q[i] = b;
    }
}

__global__ void __launch_bounds__(kWireThreads) wire_dequantize_kernel(int mode, const uint8_t* __restrict__ in,
                                                                      int D, float* __restrict__ out) {
    const int t = blockIdx.x, tid = threadIdx.x;
    const uint8_t* s = in + (size_t)t * wire_token_bytes(mode, D);
    float* o = out + (size_t)t * D;
    if (mode == 0) {
        for (int i = tid; i < D; i += kWireThreads) o[i] = get_f32_le(s + 4 * i);
        return;
    }
    if (mode != 2 && mode != 3) {
        for (int i = tid; i < D; i += kWireThreads)
            o[i] = __half2float(__ushort_as_half((unsigned short)(s[2 * i] | (s[2 * i + 1] << 8))));
        return;
    }
    const float scale = get_f32_le(s);
    const bool fin = isfinite(scale);
    for (int i = tid; i < D; i += kWireThreads) {
        float v = 0.f;
        if (fin) {
            v = (mode == 2) ? __fmul_rn((float)(int8_t)s[4 + i], scale)
                            : __fmul_rn(e4m3_to_f32(s[4 + i]), scale);
        }
        o[i] = v;
    }
}

cudaError_t wire_quantize_launch(int mode, const float* x, int T, int D, uint8_t* out, cudaStream_t stream) {
    if (T <= 0) return cudaSuccess;
    wire_quantize_kernel<<<T, kWireThreads, 0, stream>>>(mode, x, D, out);
    return cudaGetLastError();
}

cudaError_t wire_dequantize_launch(int mode, const uint8_t* in, int T, int D, float* out, cudaStream_t stream) {
    if (T <= 0) return cudaSuccess;
    wire_dequantize_kernel<<<T, kWireThreads, 0, stream>>>(mode, in, D, out);
    return cudaGetLastError();
}

}  // namespace glc
