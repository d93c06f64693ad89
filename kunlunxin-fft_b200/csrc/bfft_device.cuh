// bfft_device.cuh -- device-side building blocks of the B200 FFT library.
//
// Complex data is interleaved complex64 (float2), batch-major (B, N), the
// public torch layout.  All transforms are forward DFTs
//     X[k] = sum_n x[n] exp(-2 pi i n k / N)
// in the core; the inverse is the conjugate trick (conjugate on load,
// conjugate + scale on store), as in the reference entry layer
// (src/xpu/entry.py:619-628).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace bfft {

// ---------------------------------------------------------------- complex ops
__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 cconj(float2 a) { return make_float2(a.x, -a.y); }

// Packed FP32x2 forms of cadd / csub (sm_100 `add.rn.f32x2` / `sub.rn.f32x2`):
// one instruction per complex add, each lane rounded exactly like the scalar
// add.  Chosen per kernel (the PK parameter of Dft / stockham_passes) by
// measurement: they pay where the butterflies dominate the instruction count.
__device__ __forceinline__ unsigned long long pack2(float2 a) {
    unsigned long long r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
    return r;
}
__device__ __forceinline__ float2 unpack2(unsigned long long r) {
    float2 d;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d.x), "=f"(d.y) : "l"(r));
    return d;
}
template <bool PK>
__device__ __forceinline__ float2 cadd_p(float2 a, float2 b) {
    if constexpr (PK) {
        unsigned long long d;
        asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack2(a)), "l"(pack2(b)));
        return unpack2(d);
    } else {
        return cadd(a, b);
    }
}
template <bool PK>
__device__ __forceinline__ float2 csub_p(float2 a, float2 b) {
    if constexpr (PK) {
        unsigned long long d;
        asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(pack2(a)), "l"(pack2(b)));
        return unpack2(d);
    } else {
        return csub(a, b);
    }
}
__device__ __forceinline__ float2 cscale(float2 a, float s) { return make_float2(a.x * s, a.y * s); }

// Bit reversal of the low `bits` bits (bits in [0, 32]).  Reference index map:
// include/butterfly/bit_reverse.hpp:15-22, src/xpu/kernels.py:27-38.
__device__ __forceinline__ uint32_t brev_bits(uint32_t x, int bits) {
    return bits == 0 ? 0u : (__brev(x) >> (32 - bits));
}

// Radix-4 digit reversal folded into the first DIT stage of the radix-4
// cascade (src/xpu/kernels.py:41-57): 2-bit digits from the low end land
// reversed; an odd top bit moves to bit 0.
__device__ __forceinline__ uint32_t dit_digit_reverse(uint32_t x, int bits) {
    uint32_t r = 0;
    for (int q = 0; q < bits / 2; ++q) r |= ((x >> (2 * q)) & 3u) << (bits - 2 * q - 2);
    if (bits & 1) r |= (x >> (bits - 1)) & 1u;
    return r;
}

// Output permutation of the radix-4 DIF cascade (src/xpu/kernels.py:60-78):
// for odd `bits` the bottom bit takes the top output weight.
__device__ __forceinline__ uint32_t dif_digit_reverse(uint32_t x, int bits) {
    if (!(bits & 1)) return dit_digit_reverse(x, bits);
    uint32_t r = (x & 1u) << (bits - 1);
    for (int q = 1; q <= bits / 2; ++q) r |= ((x >> (2 * q - 1)) & 3u) << (bits - 1 - 2 * q);
    return r;
}

// ---------------------------------------------------------------- twiddles
// exp(-2 pi i k / 16) for k in [0, 16): the constants of the in-register
// radix-2/4/8/16 DFTs.  cos/sin of multiples of pi/8, rounded to float.
struct W16 {
    static constexpr float C1 = 0.92387953251128675613f;  // cos(pi/8)
    static constexpr float S1 = 0.38268343236508977173f;  // sin(pi/8)
    static constexpr float R2 = 0.70710678118654752440f;  // cos(pi/4)
};

// v * exp(-2 pi i k / R) for a compile-time (k, R), R | 16.  Multiplications
// by 1, -i, (1-i)/sqrt2 and (-1-i)/sqrt2 are spelled out so that they cost
// adds only.
template <int K, int R>
__device__ __forceinline__ float2 mul_wconst(float2 v) {
    constexpr int k16 = (K * 16 / R) & 15;
    if constexpr (k16 == 0) {
        return v;
    } else if constexpr (k16 == 4) {  // -i
        return make_float2(v.y, -v.x);
    } else if constexpr (k16 == 8) {  // -1
        return make_float2(-v.x, -v.y);
    } else if constexpr (k16 == 12) {  // +i
        return make_float2(-v.y, v.x);
    } else if constexpr (k16 == 2) {  // (1 - i)/sqrt2
        return make_float2((v.x + v.y) * W16::R2, (v.y - v.x) * W16::R2);
    } else if constexpr (k16 == 6) {  // (-1 - i)/sqrt2
        return make_float2((v.y - v.x) * W16::R2, -(v.x + v.y) * W16::R2);
    } else if constexpr (k16 == 10) {  // (-1 + i)/sqrt2
        return make_float2(-(v.x + v.y) * W16::R2, (v.x - v.y) * W16::R2);
    } else if constexpr (k16 == 14) {  // (1 + i)/sqrt2
        return make_float2((v.x - v.y) * W16::R2, (v.x + v.y) * W16::R2);
    } else {
        // odd multiples of pi/8: cos/sin are +-C1 or +-S1
        constexpr float c = (k16 == 1 || k16 == 15) ? W16::C1
                          : (k16 == 3 || k16 == 13) ? W16::S1
                          : (k16 == 5 || k16 == 11) ? -W16::S1 : -W16::C1;
        constexpr float s = (k16 == 1 || k16 == 7) ? -W16::S1
                          : (k16 == 3 || k16 == 5) ? -W16::C1
                          : (k16 == 9 || k16 == 15) ? W16::S1 : W16::C1;
        return make_float2(v.x * c - v.y * s, v.x * s + v.y * c);
    }
}

// ---------------------------------------------------------------- in-register DFT
// Natural-order forward DFT of R values held in registers (R | 16), by
// radix-2 decimation in time; fully unrolled, all indices compile-time.
// PK: complex adds as packed FP32x2 instructions (same results).
template <int R, bool PK = false>
struct Dft {
    static __device__ __forceinline__ void run(float2 (&v)[R]) {
        float2 e[R / 2], o[R / 2];
#pragma unroll
        for (int i = 0; i < R / 2; ++i) {
            e[i] = v[2 * i];
            o[i] = v[2 * i + 1];
        }
        Dft<R / 2, PK>::run(e);
        Dft<R / 2, PK>::run(o);
        combine<0>(v, e, o);
    }
    template <int K>
    static __device__ __forceinline__ void combine(float2 (&v)[R], const float2 (&e)[R / 2],
                                                   const float2 (&o)[R / 2]) {
        if constexpr (K < R / 2) {
            float2 t = mul_wconst<K, R>(o[K]);
            v[K] = cadd_p<PK>(e[K], t);
            v[K + R / 2] = csub_p<PK>(e[K], t);
            combine<K + 1>(v, e, o);
        }
    }
};
template <bool PK>
struct Dft<1, PK> {
    static __device__ __forceinline__ void run(float2 (&)[1]) {}
};
template <bool PK>
struct Dft<2, PK> {
    static __device__ __forceinline__ void run(float2 (&v)[2]) {
        float2 a = v[0], b = v[1];
        v[0] = cadd_p<PK>(a, b);
        v[1] = csub_p<PK>(a, b);
    }
};
template <bool PK>
struct Dft<4, PK> {
    static __device__ __forceinline__ void run(float2 (&v)[4]) {
        float2 s02 = cadd_p<PK>(v[0], v[2]), d02 = csub_p<PK>(v[0], v[2]);
        float2 s13 = cadd_p<PK>(v[1], v[3]), d13 = csub_p<PK>(v[1], v[3]);
        float2 d13m = make_float2(d13.y, -d13.x);  // -i * d13
        v[0] = cadd_p<PK>(s02, s13);
        v[2] = csub_p<PK>(s02, s13);
        v[1] = cadd_p<PK>(d02, d13m);
        v[3] = csub_p<PK>(d02, d13m);
    }
};

// ---------------------------------------------------------------- twiddle tables
// Twiddles come from tables computed in float64 and rounded once to float
// (twiddle_init_* in bfft_kernels.cu):
//   * g_tw_unit: exp(-2 pi i e / kTwUnit), e < kTwUnit -- any W_L^e with
//     L | kTwUnit is g_tw_unit[e * kTwUnit / L];
//   * per-plan two-level tables for W_N^e, e < N:
//     W_N^e = hi[e >> lo_bits] * lo[e & (2^lo_bits - 1)].
constexpr int kTwUnitBits = 14;
constexpr int kTwUnit = 1 << kTwUnitBits;

struct TwoLevel {
    const float2* lo;
    const float2* hi;
    int lo_bits;
    int log2n;
    // Optional three-level form of the same W_N (N > 2^22): level j = 0, 1, 2
    // holds 2^l3_bits entries at l3 + j * 2^l3_bits, entry k of level j being
    // W_N^{k 2^(j l3_bits)} -- small enough to stage in shared memory.
    const float2* l3 = nullptr;
    int l3_bits = 0;
};

// Exponents are taken mod N (N | 2^32), so 32-bit wrap-around arithmetic on
// the caller's side is exact.
__device__ __forceinline__ float2 tw_two_level(const TwoLevel& t, uint32_t e) {
    e &= (t.log2n >= 32) ? 0xffffffffu : ((1u << t.log2n) - 1u);
    float2 a = __ldg(t.lo + (e & ((1u << t.lo_bits) - 1u)));
    if (t.log2n <= t.lo_bits) return a;
    float2 b = __ldg(t.hi + (e >> t.lo_bits));
    return cmul(a, b);
}

}  // namespace bfft
