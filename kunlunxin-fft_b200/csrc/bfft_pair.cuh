// bfft_pair.cuh -- paired complex arithmetic for the consumers of the fused
// and row-pair kernels.
//
// A thread carries the same element of two columns (two independent
// sub-FFTs) as one "pair": re = (a.re, b.re) and im = (a.im, b.im), each a
// 64-bit register pair operated on by sm_100's packed FP32x2 instructions
// (add/sub/mul/fma.rn.f32x2).  Every butterfly add, constant-twiddle
// multiply and table-twiddle multiply then serves two transforms with one
// instruction per component, and the Stockham exchange moves a pair with one
// 16-byte shared-memory access.  Each lane rounds exactly like the scalar
// FP32 instruction, so a pair computes bit for bit what two scalar threads
// running the same operation sequence would.
//
// Included by bfft_kernels.cu (uses the unit twiddle levels and the Stockham
// pass shapes: radix_log2, tw_split, tw_offset, tw_total).
#pragma once

namespace bfft {

using u64 = unsigned long long;

struct CPair {
    u64 re, im;
};

__device__ __forceinline__ u64 f2add(u64 a, u64 b) {
    u64 d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ u64 f2sub(u64 a, u64 b) {
    u64 d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ u64 f2mul(u64 a, u64 b) {
    u64 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ u64 f2fma(u64 a, u64 b, u64 c) {  // a * b + c
    u64 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ u64 f2pack(float lo, float hi) {
    u64 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ u64 f2splat(float c) { return f2pack(c, c); }

// IEEE-754 bits of a normal float (or zero), at compile time, so constant
// pairs are plain 64-bit literals the compiler can keep and share.
__host__ __device__ constexpr uint32_t fbits(float f) {
    if (f == 0.0f) return 0u;
    const uint32_t sign = f < 0.0f ? 0x80000000u : 0u;
    double a = f < 0.0f ? -(double)f : (double)f;
    int e = 0;
    while (a >= 2.0) { a *= 0.5; ++e; }
    while (a < 1.0) { a *= 2.0; --e; }
    const uint32_t mant = static_cast<uint32_t>((a - 1.0) * 8388608.0);  // exact: f has 24 significant bits
    return sign | (static_cast<uint32_t>(e + 127) << 23) | mant;
}
__host__ __device__ constexpr u64 splat_bits(float f) {
    return (static_cast<u64>(fbits(f)) << 32) | fbits(f);
}
static_assert(fbits(1.0f) == 0x3f800000u && fbits(-0.5f) == 0xbf000000u, "fbits");
static_assert(fbits(W16::R2) == 0x3f3504f3u && fbits(W16::C1) == 0x3f6c835eu && fbits(W16::S1) == 0x3ec3ef15u,
              "fbits of the DFT16 constants");
__device__ __forceinline__ float f2lo(u64 r) { return __uint_as_float(static_cast<unsigned>(r)); }
__device__ __forceinline__ float f2hi(u64 r) { return __uint_as_float(static_cast<unsigned>(r >> 32)); }

__device__ __forceinline__ CPair cp_add(CPair a, CPair b) { return CPair{f2add(a.re, b.re), f2add(a.im, b.im)}; }
__device__ __forceinline__ CPair cp_sub(CPair a, CPair b) { return CPair{f2sub(a.re, b.re), f2sub(a.im, b.im)}; }
// a * w for a pair of twiddles w = (wr, wi) pairs: re = ar wr - ai wi, im = ar wi + ai wr
__device__ __forceinline__ CPair cp_mul(CPair a, CPair w) {
    return CPair{f2sub(f2mul(a.re, w.re), f2mul(a.im, w.im)), f2fma(a.re, w.im, f2mul(a.im, w.re))};
}
// pair of two scalar complex values (a of the first column, b of the second)
__device__ __forceinline__ CPair cp_make(float2 a, float2 b) { return CPair{f2pack(a.x, b.x), f2pack(a.y, b.y)}; }
__device__ __forceinline__ float2 cp_first(CPair p) { return make_float2(f2lo(p.re), f2lo(p.im)); }
__device__ __forceinline__ float2 cp_second(CPair p) { return make_float2(f2hi(p.re), f2hi(p.im)); }

// v * exp(-2 pi i k / R) for a compile-time (k, R), R | 16, k16 = k 16 / R.
template <int K, int R>
__device__ __forceinline__ CPair cp_mul_wconst(CPair v) {
    constexpr int k16 = (K * 16 / R) & 15;
    if constexpr (k16 == 0) {
        return v;
    } else if constexpr (k16 == 8) {  // -1
        const u64 z = 0;
        return CPair{f2sub(z, v.re), f2sub(z, v.im)};
    } else if constexpr (k16 == 2) {  // (1 - i)/sqrt2: ((x + y) r, (y - x) r)
        constexpr u64 r = splat_bits(W16::R2);
        return CPair{f2mul(f2add(v.re, v.im), r), f2mul(f2sub(v.im, v.re), r)};
    } else if constexpr (k16 == 6) {  // (-1 - i)/sqrt2: ((y - x) r, (x + y) (-r))
        constexpr u64 r = splat_bits(W16::R2), nr = splat_bits(-W16::R2);
        return CPair{f2mul(f2sub(v.im, v.re), r), f2mul(f2add(v.re, v.im), nr)};
    } else {
        // c = cos, s = sin of -2 pi k16 / 16: re = x c - y s, im = x s + y c
        constexpr float c = (k16 == 1 || k16 == 15) ? W16::C1
                          : (k16 == 3 || k16 == 13) ? W16::S1
                          : (k16 == 5 || k16 == 11) ? -W16::S1 : -W16::C1;
        constexpr float s = (k16 == 1 || k16 == 7) ? -W16::S1
                          : (k16 == 3 || k16 == 5) ? -W16::C1
                          : (k16 == 9 || k16 == 15) ? W16::S1 : W16::C1;
        static_assert(k16 != 4 && k16 != 12, "multiples of -i are folded by the callers");
        constexpr u64 kc = splat_bits(c), ks = splat_bits(s), kns = splat_bits(-s);
        return CPair{f2fma(v.im, kns, f2mul(v.re, kc)), f2fma(v.im, kc, f2mul(v.re, ks))};
    }
}

// Natural-order forward DFT of R pairs in registers (R | 16): radix-2
// decimation in time, the multiply by -i of each level folded into its
// butterfly (no negation).
template <int R>
struct PairDft {
    static __device__ __forceinline__ void run(CPair (&v)[R]) {
        CPair e[R / 2], o[R / 2];
#pragma unroll
        for (int i = 0; i < R / 2; ++i) {
            e[i] = v[2 * i];
            o[i] = v[2 * i + 1];
        }
        PairDft<R / 2>::run(e);
        PairDft<R / 2>::run(o);
        combine<0>(v, e, o);
    }
    template <int K>
    static __device__ __forceinline__ void combine(CPair (&v)[R], const CPair (&e)[R / 2], const CPair (&o)[R / 2]) {
        if constexpr (K < R / 2) {
            if constexpr (K * 4 == R) {  // twiddle -i: e -+ i o
                v[K] = CPair{f2add(e[K].re, o[K].im), f2sub(e[K].im, o[K].re)};
                v[K + R / 2] = CPair{f2sub(e[K].re, o[K].im), f2add(e[K].im, o[K].re)};
            } else {
                const CPair t = cp_mul_wconst<K, R>(o[K]);
                v[K] = cp_add(e[K], t);
                v[K + R / 2] = cp_sub(e[K], t);
            }
            combine<K + 1>(v, e, o);
        }
    }
};
template <>
struct PairDft<1> {
    static __device__ __forceinline__ void run(CPair (&)[1]) {}
};
template <>
struct PairDft<2> {
    static __device__ __forceinline__ void run(CPair (&v)[2]) {
        const CPair a = v[0], b = v[1];
        v[0] = cp_add(a, b);
        v[1] = cp_sub(a, b);
    }
};

// Pair twiddle tables of the Stockham passes: the entries of tw_offset /
// tw_total (row k of pass p holds W_{Rp}^{j k}, j = 1..R-1; pass 2 of radix
// R >= 4 the split rows kl then kh, W_{256 R}^{j kl} and W_{16 R}^{j kh}),
// each stored as (wr, wr, wi, wi) so one 16-byte load gives the pair operand.
// Sub-FFTs of up to 1024 points (three passes).
template <int LOG2L>
__device__ __forceinline__ void fill_pair_twiddles(CPair* tw) {
    constexpr int NP = LOG2L <= 4 ? 1 : (LOG2L + 3) / 4;
    static_assert(NP <= 3, "pair passes: sub-FFTs of at most 4096 points");
    for (int pass = 1; pass < NP; ++pass) {
        const int r = 1 << radix_log2(LOG2L, pass), p = 1 << (4 * pass);
        CPair* dst = tw + tw_offset(LOG2L, pass);
        if (tw_split(LOG2L, pass)) {
            const int cnt = 2 * 16 * (r - 1);
            for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
                const int row = i / (r - 1), j = i - row * (r - 1) + 1;
                const float2 w = row < 16 ? g_tw_levels[r * p + j * row] : g_tw_levels[r * 16 + j * (row - 16)];
                dst[i] = CPair{f2splat(w.x), f2splat(w.y)};
            }
            continue;
        }
        const float2* lvl = g_tw_levels + r * p;
        const int cnt = p * (r - 1);
        for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
            const int k = i / (r - 1), j = i - k * (r - 1) + 1;
            const float2 w = lvl[j * k];
            dst[i] = CPair{f2splat(w.x), f2splat(w.y)};
        }
    }
}

// Exchange slot of pair index i: the low three bits XORed with bits 4..6, a
// permutation within aligned groups of 8 slots (128 bytes: one row of the 32
// banks for 16-byte pairs).  A pass-0 store sends lane b's output j to slot
// 16 b + j, 256 bytes apart for consecutive b, so without it the lanes of a
// warp meet on the same four banks (32-way conflicts with one pair per
// index); with it, 8 consecutive b fill a whole bank row.  The later passes'
// stores and every read (consecutive indices) stay conflict-free.  With 8 or
// more pairs per index an index is a whole bank row already: no swizzle (its
// index arithmetic would only cost instructions).
template <int NPAIR>
__device__ __forceinline__ int pair_swizzle(int i) {
    if constexpr (NPAIR >= 8) return i;
    else return i ^ ((i >> 4) & 7);
}

// Stockham passes on pairs: the structure of stockham_passes (butterfly b
// of the thread takes slots q + j NB, output j goes to (b/p) p R + (b mod p)
// + j p), the exchange area holding pair i of the thread's column pair at
// region[pair_swizzle<NPAIR>(i) * NPAIR] (16 bytes each).  NBAR threads meet at named barrier 1.
template <int LOG2L, int PASS, int TF, int NPAIR, int NBAR>
__device__ __forceinline__ void pair_passes(CPair (&v)[16], int t, ulonglong2* region, const CPair* tw) {
    constexpr int E = 16;
    constexpr int NP = LOG2L <= 4 ? 1 : (LOG2L + 3) / 4;
    if constexpr (PASS < NP) {
        constexpr int LR = radix_log2(LOG2L, PASS);
        constexpr int R = 1 << LR;
        constexpr int LP = 4 * PASS;
        constexpr int NB = E / R;
#pragma unroll
        for (int q = 0; q < NB; ++q) {
            const int b = t + q * TF;
            const int k = b & ((1 << LP) - 1);
            CPair u[R];
#pragma unroll
            for (int j = 0; j < R; ++j) u[j] = v[q + j * NB];
            if constexpr (tw_split(LOG2L, PASS)) {  // W_{256 R}^{j k} = W_{256 R}^{j kl} W_{16 R}^{j kh}
                const CPair* tl = tw + tw_offset(LOG2L, PASS) + (k & 15) * (R - 1) - 1;
                const CPair* th = tw + tw_offset(LOG2L, PASS) + (16 + (k >> 4)) * (R - 1) - 1;
#pragma unroll
                for (int j = 1; j < R; ++j) u[j] = cp_mul(u[j], cp_mul(tl[j], th[j]));
            } else if constexpr (PASS > 0) {
                const CPair* w = tw + tw_offset(LOG2L, PASS) + k * (R - 1) - 1;
#pragma unroll
                for (int j = 1; j < R; ++j) u[j] = cp_mul(u[j], w[j]);
            }
            PairDft<R>::run(u);
#pragma unroll
            for (int j = 0; j < R; ++j) v[q + j * NB] = u[j];
        }
        if constexpr (PASS + 1 < NP) {
#pragma unroll
            for (int q = 0; q < NB; ++q) {
                const int b = t + q * TF;
                const int k = b & ((1 << LP) - 1);
                const int base = ((b >> LP) << (LP + LR)) + k;
#pragma unroll
                for (int j = 0; j < R; ++j) {
                    const CPair x = v[q + j * NB];
                    region[pair_swizzle<NPAIR>(base + (j << LP)) * NPAIR] = make_ulonglong2(x.re, x.im);
                }
            }
            group_sync<NBAR>();
#pragma unroll
            for (int m = 0; m < E; ++m) {
                const ulonglong2 x = region[pair_swizzle<NPAIR>(t + m * TF) * NPAIR];
                v[m] = CPair{x.x, x.y};
            }
            group_sync<NBAR>();
            pair_passes<LOG2L, PASS + 1, TF, NPAIR, NBAR>(v, t, region, tw);
        }
    }
}

}  // namespace bfft
