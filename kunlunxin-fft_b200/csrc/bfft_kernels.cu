// bfft_kernels.cu -- sm_100a kernels of the B200 FFT library.
//
// Two kernel families:
//   * global-stage kernels: one radix-2 or radix-4 stage per launch over the
//     whole (B, N) array -- the B200 realisation of the reference's M0/M4/M5
//     flows, with the same index maps, twiddle exponents and folded
//     permutations (src/xpu/kernels.py:100-423, :633-1124);
//   * the CTA-resident Stockham pass: a whole sub-FFT of up to 4096 points is
//     loaded once from HBM into registers, transformed with radix-16 register
//     butterflies whose stages exchange through padded shared memory, and
//     stored once.  One pass is a complete FFT for N <= 4096; larger N and the
//     reference's local-group / grouped-tail / 4-step flows are sequences of
//     such passes with fused twiddles.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <atomic>
#include <mutex>

#include "bfft_kernels.cuh"

namespace bfft {

// ============================================================== twiddle tables

__device__ float2 g_tw_levels[2 * kTwUnit];

__global__ void k_twiddle_levels() {
    int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx < 1 || idx >= 2 * kTwUnit) return;
    int lp = 1 << (31 - __clz(idx));  // level: idx in [lp, 2 lp)
    int e = idx - lp;
    double s, c;
    sincospi(2.0 * (double)e / (double)lp, &s, &c);
    g_tw_levels[idx] = make_float2((float)c, (float)(-s));
}

__global__ void k_twiddle_two_level(float2* lo, float2* hi, int lo_bits, int log2n) {
    int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    int64_t nlo = (int64_t)1 << (lo_bits < log2n ? lo_bits : log2n);
    int64_t nhi = log2n > lo_bits ? ((int64_t)1 << (log2n - lo_bits)) : 0;
    double inv_n = 1.0 / (double)((int64_t)1 << log2n);  // exact: power of two
    double s, c;
    if (idx < nlo) {
        sincospi(2.0 * (double)idx * inv_n, &s, &c);
        lo[idx] = make_float2((float)c, (float)(-s));
    } else if (idx < nlo + nhi) {
        int64_t h = idx - nlo;
        sincospi(2.0 * (double)(h << lo_bits) * inv_n, &s, &c);
        hi[h] = make_float2((float)c, (float)(-s));
    }
}

__global__ void k_twiddle_three_level(float2* t, int bits, int log2n) {
    const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= ((int64_t)3 << bits)) return;
    const int j = (int)(idx >> bits);
    const int64_t k = idx & (((int64_t)1 << bits) - 1);
    const int64_t e = (k << (bits * j)) & ((((int64_t)1) << log2n) - 1);
    double s, c;
    sincospi(2.0 * (double)e / (double)((int64_t)1 << log2n), &s, &c);
    t[idx] = make_float2((float)c, (float)(-s));
}

cudaError_t fill_three_level(float2* t, int bits, int log2n, cudaStream_t s) {
    const int64_t tot = (int64_t)3 << bits;
    k_twiddle_three_level<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(t, bits, log2n);
    return cudaGetLastError();
}

static std::mutex g_tw_mu;
static bool g_tw_ready[64];

cudaError_t ensure_unit_twiddles(int device, cudaStream_t stream) {
    if (device < 0 || device >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_tw_mu);
    if (g_tw_ready[device]) return cudaSuccess;
    k_twiddle_levels<<<(2 * kTwUnit + 255) / 256, 256, 0, stream>>>();
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess) g_tw_ready[device] = true;
    return e;
}

cudaError_t fill_two_level(float2* lo, float2* hi, int lo_bits, int log2n, cudaStream_t s) {
    int64_t nlo = (int64_t)1 << (lo_bits < log2n ? lo_bits : log2n);
    int64_t nhi = log2n > lo_bits ? ((int64_t)1 << (log2n - lo_bits)) : 0;
    int64_t tot = nlo + nhi;
    k_twiddle_two_level<<<(unsigned)((tot + 255) / 256), 256, 0, s>>>(lo, hi, lo_bits, log2n);
    return cudaGetLastError();
}

// ============================================================== global stages

__device__ __forceinline__ float2 ld_c(const float2* p, int conj) {
    float2 v = __ldg(p);
    return conj ? cconj(v) : v;
}
__device__ __forceinline__ float2 out_c(float2 v, int conj, float scale) {
    if (conj) v = cconj(v);
    return scale != 1.0f ? cscale(v, scale) : v;
}
__device__ __forceinline__ int64_t perm_out(int64_t i, int mode, int bits) {
    return mode == 1 ? (int64_t)brev_bits((uint32_t)i, bits)
         : mode == 2 ? (int64_t)dif_digit_reverse((uint32_t)i, bits) : i;
}

// One radix-2 stage (src/xpu/kernels.py:100-236, :993-1124):
//   off in [0, N/2): j = off % n, i = (off / n) * 2n + j, w = W_N^{j*M}
//   DIT: y[i] = a + b w, y[i+n] = a - b w   (a, b optionally bit-reversed reads)
//   DIF: y[P(i)] = a + b, y[P(i+n)] = (a - b) w
template <bool DIF>
__device__ __forceinline__ void radix2_body(const float2* __restrict__ x, float2* __restrict__ y,
                                            const StageArgs& a, int64_t row, int64_t off,
                                            int log2half) {
    const float2* xr = x + row * a.n;
    float2* yr = y + row * a.n;
    const int64_t n = a.half;
    const int64_t j = off & (n - 1);
    const int64_t i = ((off >> log2half) << (log2half + 1)) + j;
    const float2 w = tw_two_level(a.tw, (uint32_t)j * (uint32_t)a.M);
    int64_t s0 = i, s1 = i + n;
    if (!DIF && a.in_perm == 1) {
        s0 = brev_bits((uint32_t)s0, a.log2n);
        s1 = brev_bits((uint32_t)s1, a.log2n);
    }
    float2 va = ld_c(xr + s0, a.conj_in), vb = ld_c(xr + s1, a.conj_in);
    if (!DIF) {
        float2 bw = cmul(vb, w);
        yr[i] = out_c(cadd(va, bw), a.conj_out, a.scale);
        yr[i + n] = out_c(csub(va, bw), a.conj_out, a.scale);
    } else {
        float2 sm = cadd(va, vb);
        float2 df = cmul(csub(va, vb), w);
        yr[perm_out(i, a.out_perm, a.log2n)] = out_c(sm, a.conj_out, a.scale);
        yr[perm_out(i + n, a.out_perm, a.log2n)] = out_c(df, a.conj_out, a.scale);
    }
}

template <bool DIF>
__global__ void k_radix2_stage(const float2* __restrict__ x, float2* __restrict__ y, StageArgs a) {
    const int64_t half_n = a.n >> 1;
    const int log2half = 63 - __clzll(a.half);
    if (a.folded) {
        const int64_t total = a.batch * half_n;
        for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
             g += (int64_t)gridDim.x * blockDim.x)
            radix2_body<DIF>(x, y, a, g >> (a.log2n - 1), g & (half_n - 1), log2half);
    } else {
        const int64_t off = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
        if (off >= half_n) return;
        for (int64_t row = blockIdx.y; row < a.batch; row += gridDim.y)
            radix2_body<DIF>(x, y, a, row, off, log2half);
    }
}

// One radix-4 stage of span 4n (src/xpu/kernels.py:239-423, :633-809):
//   off in [0, N/4): j = off % n, i = (off / n) * 4n + j, exponents d*j*M.
//   DIT: twiddle inputs then 4-point DFT (optional digit-reversed reads).
//   DIF: 4-point DFT then twiddle outputs (optional digit-reversed stores).
template <bool DIF>
__device__ __forceinline__ void radix4_body(const float2* __restrict__ x, float2* __restrict__ y,
                                            const StageArgs& a, int64_t row, int64_t off,
                                            int log2q) {
    const float2* xr = x + row * a.n;
    float2* yr = y + row * a.n;
    const int64_t n = a.half;
    const int64_t j = off & (n - 1);
    const int64_t i = ((off >> log2q) << (log2q + 2)) + j;
    const uint32_t jm = (uint32_t)j * (uint32_t)a.M;
    float2 v[4];
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        int64_t s = i + d * n;
        if (!DIF && a.in_perm == 2) s = dit_digit_reverse((uint32_t)s, a.log2n);
        v[d] = ld_c(xr + s, a.conj_in);
    }
    if (!DIF) {
#pragma unroll
        for (int d = 1; d < 4; ++d) v[d] = cmul(v[d], tw_two_level(a.tw, jm * (uint32_t)d));
    }
    // 4-point DFT in the reference's column order (y0..y3)
    float2 y0 = cadd(cadd(v[0], v[1]), cadd(v[2], v[3]));
    float2 y1 = make_float2(v[0].x + v[1].y - v[2].x - v[3].y, v[0].y - v[1].x - v[2].y + v[3].x);
    float2 y2 = make_float2(v[0].x - v[1].x + v[2].x - v[3].x, v[0].y - v[1].y + v[2].y - v[3].y);
    float2 y3 = make_float2(v[0].x - v[1].y - v[2].x + v[3].y, v[0].y + v[1].x - v[2].y - v[3].x);
    float2 o[4] = {y0, y1, y2, y3};
    if (DIF) {
#pragma unroll
        for (int d = 1; d < 4; ++d) o[d] = cmul(o[d], tw_two_level(a.tw, jm * (uint32_t)d));
    }
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        int64_t dst = i + d * n;
        if (DIF && a.out_perm == 2) dst = dif_digit_reverse((uint32_t)dst, a.log2n);
        yr[dst] = out_c(o[d], a.conj_out, a.scale);
    }
}

template <bool DIF>
__global__ void k_radix4_stage(const float2* __restrict__ x, float2* __restrict__ y, StageArgs a) {
    const int64_t quarter = a.n >> 2;
    const int log2q = 63 - __clzll(a.half);
    if (a.folded) {
        const int64_t total = a.batch * quarter;
        for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
             g += (int64_t)gridDim.x * blockDim.x)
            radix4_body<DIF>(x, y, a, g >> (a.log2n - 2), g & (quarter - 1), log2q);
    } else {
        const int64_t off = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
        if (off >= quarter) return;
        for (int64_t row = blockIdx.y; row < a.batch; row += gridDim.y)
            radix4_body<DIF>(x, y, a, row, off, log2q);
    }
}

static int clamp_block(int block) {
    if (block < 32) return 32;
    if (block > 1024) return 1024;
    return block;
}

static dim3 stage_grid(int64_t per_row, int64_t batch, int block, bool folded) {
    if (folded) {
        int64_t blocks = (per_row * batch + block - 1) / block;
        if (blocks > 148 * 64) blocks = 148 * 64;
        return dim3((unsigned)(blocks < 1 ? 1 : blocks));
    }
    int64_t bx = (per_row + block - 1) / block;
    int64_t by = batch < 65535 ? batch : 65535;
    return dim3((unsigned)bx, (unsigned)by);
}

cudaError_t launch_radix2_stage(bool dif, const float2* x, float2* y, const StageArgs& a,
                                int block, cudaStream_t s) {
    block = clamp_block(block);
    dim3 g = stage_grid(a.n >> 1, a.batch, block, a.folded != 0);
    if (dif)
        k_radix2_stage<true><<<g, block, 0, s>>>(x, y, a);
    else
        k_radix2_stage<false><<<g, block, 0, s>>>(x, y, a);
    return cudaGetLastError();
}

cudaError_t launch_radix4_stage(bool dif, const float2* x, float2* y, const StageArgs& a,
                                int block, cudaStream_t s) {
    block = clamp_block(block);
    dim3 g = stage_grid(a.n >> 2, a.batch, block, a.folded != 0);
    if (dif)
        k_radix4_stage<true><<<g, block, 0, s>>>(x, y, a);
    else
        k_radix4_stage<false><<<g, block, 0, s>>>(x, y, a);
    return cudaGetLastError();
}

// ============================================================== permutation / epilogues

// Y[r, i] = X[r, bitrev(i)]  (src/xpu/kernels.py:81-97, :536-561), with an
// optional conjugate and scale folded into the store.
__global__ void k_bitrev(const float2* __restrict__ x, float2* __restrict__ y, int64_t n,
                         int64_t total, int log2n, int conj, float scale) {
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
         g += (int64_t)gridDim.x * blockDim.x) {
        int64_t row = g >> log2n, i = g & (n - 1);
        y[g] = out_c(__ldg(x + row * n + brev_bits((uint32_t)i, log2n)), conj, scale);
    }
}

static unsigned flat_grid(int64_t total, int block) {
    int64_t b = (total + block - 1) / block;
    if (b > 148 * 32) b = 148 * 32;
    return (unsigned)(b < 1 ? 1 : b);
}

cudaError_t launch_bitrev(const float2* x, float2* y, int64_t n, int64_t batch, int block,
                          cudaStream_t s, int conj, float scale) {
    block = clamp_block(block);
    int log2n = 63 - __builtin_clzll((unsigned long long)n);
    k_bitrev<<<flat_grid(n * batch, block), block, 0, s>>>(x, y, n, n * batch, log2n, conj, scale);
    return cudaGetLastError();
}

// Packed-compat helpers of the real transforms (src/xpu/entry.py:588-616):
// real -> complex with zero imaginary part, half-spectrum crop with scale,
// Hermitian rebuild (entry.py:671-696) with the inverse conjugation folded
// in, and the real-part extraction of the conjugated, scaled result.
__global__ void k_real_to_complex(const float* __restrict__ x, float2* __restrict__ y, int64_t total) {
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
         g += (int64_t)gridDim.x * blockDim.x)
        y[g] = make_float2(__ldg(x + g), 0.0f);
}

__global__ void k_crop(const float2* __restrict__ y, float2* __restrict__ out, int64_t n,
                       int64_t cols, int64_t total, float scale) {
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
         g += (int64_t)gridDim.x * blockDim.x) {
        int64_t b = g / cols, k = g - b * cols;
        out[g] = cscale(__ldg(y + b * n + k), scale);
    }
}

__global__ void k_hermitian_conj(const float2* __restrict__ xh, float2* __restrict__ full,
                                 int64_t n, int64_t total) {
    const int64_t m = n / 2 + 1;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
         g += (int64_t)gridDim.x * blockDim.x) {
        int64_t b = g / n, k = g - b * n;
        float2 v;
        if (k < m) {
            v = __ldg(xh + b * m + k);
            if (k == 0 || k == m - 1) v.y = 0.0f;
        } else {
            v = cconj(__ldg(xh + b * m + (n - k)));
        }
        full[g] = cconj(v);  // inverse via the conjugate trick
    }
}

__global__ void k_real_part(const float2* __restrict__ y, float* __restrict__ out, int64_t total,
                            float scale) {
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
         g += (int64_t)gridDim.x * blockDim.x)
        out[g] = __ldg(y + g).x * scale;
}

cudaError_t launch_real_to_complex(const float* x, float2* y, int64_t total, cudaStream_t s) {
    k_real_to_complex<<<flat_grid(total, 256), 256, 0, s>>>(x, y, total);
    return cudaGetLastError();
}
cudaError_t launch_crop(const float2* y, float2* out, int64_t n, int64_t batch, float scale,
                        cudaStream_t s) {
    int64_t cols = n / 2 + 1;
    k_crop<<<flat_grid(batch * cols, 256), 256, 0, s>>>(y, out, n, cols, batch * cols, scale);
    return cudaGetLastError();
}
cudaError_t launch_hermitian_conj(const float2* xh, float2* full, int64_t n, int64_t batch,
                                  cudaStream_t s) {
    k_hermitian_conj<<<flat_grid(batch * n, 256), 256, 0, s>>>(xh, full, n, batch * n);
    return cudaGetLastError();
}
cudaError_t launch_real_part(const float2* y, float* out, int64_t total, float scale,
                             cudaStream_t s) {
    k_real_part<<<flat_grid(total, 256), 256, 0, s>>>(y, out, total, scale);
    return cudaGetLastError();
}

// The kernels' index maps, materialised for bit-exact checks.
__global__ void k_index_map(int kind, int bits, uint32_t* out) {
    const uint32_t n = 1u << bits;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        out[i] = kind == 0 ? brev_bits(i, bits) : kind == 1 ? dit_digit_reverse(i, bits)
                                                            : dif_digit_reverse(i, bits);
}
cudaError_t launch_index_map(int kind, int bits, uint32_t* out, cudaStream_t s) {
    k_index_map<<<flat_grid((int64_t)1 << bits, 256), 256, 0, s>>>(kind, bits, out);
    return cudaGetLastError();
}

// Reference twiddle table as complex64: w[idx] = W_n^idx, idx < count
// (src/xpu/runner.py:93-97), float64 angles rounded once.
__global__ void k_twiddle_table(float2* w, int64_t n, int64_t count) {
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < count;
         g += (int64_t)gridDim.x * blockDim.x) {
        double s, c;
        sincospi(2.0 * (double)g / (double)n, &s, &c);
        w[g] = make_float2((float)c, (float)(-s));
    }
}
cudaError_t launch_twiddle_table(float2* w, int64_t n, int64_t count, cudaStream_t s) {
    k_twiddle_table<<<flat_grid(count, 256), 256, 0, s>>>(w, n, count);
    return cudaGetLastError();
}

// R2C stitch (src/xpu/kernels.py:1127-1177): from the N/2-point FFT Z of the
// packed pairs, X[k] = a - i w c, a = (Z[k] + conj Z[j]) / 2,
// c = (Z[k] - conj Z[j]) / 2, j = (N/2 - k) % (N/2), w = W_N^k; DC and
// Nyquist imaginary parts are exactly 0; scale fused into the store.
__device__ __forceinline__ float2 r2c_point(const float2* zb, int64_t np, int64_t k, float2 w,
                                            float scale) {
    const int64_t jc = (np - k) & (np - 1), zk = k & (np - 1);
    const float2 zkv = zb[zk], zjv = zb[jc];
    const float ar = 0.5f * (zkv.x + zjv.x), ai = 0.5f * (zkv.y - zjv.y);
    const float cr = 0.5f * (zkv.x - zjv.x), ci = 0.5f * (zkv.y + zjv.y);
    float xr = ar + w.x * ci + w.y * cr;
    float xi = ai - w.x * cr + w.y * ci;
    if (k == 0 || k == np) xi = 0.0f;
    return make_float2(xr * scale, xi * scale);
}

__global__ void k_r2c_stitch(const float2* __restrict__ z, float2* __restrict__ x, int64_t n,
                             int64_t batch, float scale, TwoLevel twn) {
    const int64_t np = n >> 1, cols = np + 1, total = batch * cols;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
         g += (int64_t)gridDim.x * blockDim.x) {
        int64_t b = g / cols, k = g - b * cols;
        x[g] = r2c_point(z + b * np, np, k, tw_two_level(twn, (uint32_t)k), scale);
    }
}

// C2R pre-twiddle (src/xpu/kernels.py:1180-1229): Z[k] = a + i w c with
// w = conj(W_N^k), DC / Nyquist imaginary parts ignored.
__device__ __forceinline__ float2 c2r_pre_point(const float2* xb, int64_t np, int64_t k, float2 w) {
    const int64_t j = np - k;
    float2 xk = xb[k], xj = xb[j];
    if (k == 0) xk.y = 0.0f;
    if (j == np) xj.y = 0.0f;
    const float ar = 0.5f * (xk.x + xj.x), ai = 0.5f * (xk.y - xj.y);
    const float cr = 0.5f * (xk.x - xj.x), ci = 0.5f * (xk.y + xj.y);
    const float wr = w.x, wi = -w.y;
    return make_float2(ar - (wr * ci + wi * cr), ai + (wr * cr - wi * ci));
}

__global__ void k_c2r_pre(const float2* __restrict__ xh, float2* __restrict__ z, int64_t n,
                          int64_t batch, TwoLevel twn) {
    const int64_t np = n >> 1, cols = np + 1, total = batch * np;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
         g += (int64_t)gridDim.x * blockDim.x) {
        int64_t b = g / np, k = g - b * np;
        z[g] = c2r_pre_point(xh + b * cols, np, k, tw_two_level(twn, (uint32_t)k));
    }
}

// C2R unpack (src/xpu/kernels.py:1232-1258): out[2k], out[2k+1] =
// scale * (Re, Im) u[(N/2 - k) % (N/2)].
__global__ void k_c2r_unpack(const float2* __restrict__ u, float2* __restrict__ out, int64_t n,
                             int64_t batch, float scale) {
    const int64_t np = n >> 1, total = batch * np;
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
         g += (int64_t)gridDim.x * blockDim.x) {
        int64_t b = g / np, k = g - b * np;
        float2 v = u[b * np + ((np - k) & (np - 1))];
        out[g] = make_float2(v.x * scale, v.y * scale);
    }
}

// Elementwise conj / scale; x == y (in place) is allowed.
__global__ void k_scale(const float2* x, float2* y, int64_t count, float scale, int conj) {
    for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < count;
         g += (int64_t)gridDim.x * blockDim.x)
        y[g] = out_c(x[g], conj, scale);
}

cudaError_t launch_r2c_stitch(const float2* z, float2* x, int64_t n, int64_t batch, float scale,
                              TwoLevel twn, cudaStream_t s) {
    k_r2c_stitch<<<flat_grid(batch * (n / 2 + 1), 256), 256, 0, s>>>(z, x, n, batch, scale, twn);
    return cudaGetLastError();
}
cudaError_t launch_c2r_pre(const float2* xh, float2* z, int64_t n, int64_t batch, TwoLevel twn,
                           cudaStream_t s) {
    k_c2r_pre<<<flat_grid(batch * (n / 2), 256), 256, 0, s>>>(xh, z, n, batch, twn);
    return cudaGetLastError();
}
cudaError_t launch_c2r_unpack(const float2* u, float* out, int64_t n, int64_t batch, float scale,
                              cudaStream_t s) {
    k_c2r_unpack<<<flat_grid(batch * (n / 2), 256), 256, 0, s>>>(u, reinterpret_cast<float2*>(out),
                                                                   n, batch, scale);
    return cudaGetLastError();
}
cudaError_t launch_scale(const float2* x, float2* y, int64_t count, float scale, int conj,
                         cudaStream_t s) {
    k_scale<<<flat_grid(count, 256), 256, 0, s>>>(x, y, count, scale, conj);
    return cudaGetLastError();
}

// ============================================================== Stockham pass

__device__ __forceinline__ int pad16(int a) { return a + (a >> 4); }

__host__ __device__ constexpr int radix_log2(int log2l, int pass) { return pass < log2l / 4 ? 4 : log2l % 4; }

// Radix-R Stockham pass with p = 16^PASS (all earlier radices are 16):
// butterfly b takes elements b + j L/R, twiddles them by W_{Rp}^{j (b mod p)},
// runs an R-point DFT and sends output j to (b/p) p R + (b mod p) + j p.
// Thread t owns elements t + m' TF (m' < E), so butterfly q of the thread
// reads and writes slots q + j (E/R).
// Shared-memory twiddle tables of one sub-FFT length: for every pass with
// p > 1, rows k < p of R-1 entries W_{Rp}^{j k} (j = 1..R-1).  The odd row
// stride R-1 keeps consecutive k on distinct banks; a thread's row depends
// only on its index, so a persistent CTA fills the tables once.
// Pass 2 (p = 256) of radix R >= 4 keeps two 16-row tables instead of one
// 256-row table: with k = 16 kh + kl, W_{256 R}^{j k} = W_{256 R}^{j kl}
// W_{16 R}^{j kh} (one more complex multiply, 8-16x less shared memory --
// what lets three CTAs of the 1024..4096-point passes share an SM).
__host__ __device__ constexpr bool tw_split(int log2l, int pass) {
    return pass == 2 && radix_log2(log2l, pass) >= 2;
}
__host__ __device__ constexpr int tw_pass_entries(int log2l, int pass) {
    return pass == 0 ? 0
         : tw_split(log2l, pass) ? 2 * 16 * ((1 << radix_log2(log2l, pass)) - 1)
                                 : (1 << (4 * pass)) * ((1 << radix_log2(log2l, pass)) - 1);
}
__host__ __device__ constexpr int tw_offset(int log2l, int pass) {
    int off = 0;
    for (int p = 1; p < pass; ++p) off += tw_pass_entries(log2l, p);
    return off;
}
__host__ __device__ constexpr int tw_total(int log2l) {
    return log2l <= 4 ? 0 : tw_offset(log2l, (log2l + 3) / 4);
}

template <int LOG2L>
__device__ __forceinline__ void fill_stockham_twiddles(float2* tw_smem) {
    constexpr int NP = LOG2L <= 4 ? 1 : (LOG2L + 3) / 4;
    for (int pass = 1; pass < NP; ++pass) {
        const int r = 1 << radix_log2(LOG2L, pass), p = 1 << (4 * pass);
        float2* dst = tw_smem + tw_offset(LOG2L, pass);
        if (tw_split(LOG2L, pass)) {  // rows kl (W_{256 r}^{j kl}) then rows kh (W_{16 r}^{j kh})
            const int cnt = 2 * 16 * (r - 1);
            for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
                const int row = i / (r - 1), j = i - row * (r - 1) + 1;
                dst[i] = row < 16 ? g_tw_levels[r * p + j * row] : g_tw_levels[r * 16 + j * (row - 16)];
            }
            continue;
        }
        const float2* lvl = g_tw_levels + r * p;
        const int cnt = p * (r - 1);
        for (int i = threadIdx.x; i < cnt; i += blockDim.x) {
            const int k = i / (r - 1), j = i - k * (r - 1) + 1;
            dst[i] = lvl[j * k];
        }
    }
}

// Exchange addressing: XS = 0 is a padded per-sub-FFT region (element i at
// pad16(i)); XS > 0 is a dense tile with the sub-FFT index fastest (element i
// of this sub-FFT at i * XS), conflict-free when 16 or more sub-FFTs share a
// warp's half.
template <int XS>
__device__ __forceinline__ int xaddr(int i) {
    if constexpr (XS == 0) return pad16(i);
    else return i * XS;
}

// Barrier of the threads that share the exchange area: the whole CTA
// (NBAR = 0), or the NBAR threads of named barrier 1 (warp-specialised
// kernels whose other warps do not take part).
template <int NBAR>
__device__ __forceinline__ void group_sync() {
    if constexpr (NBAR == 0) __syncthreads();
    else asm volatile("bar.sync 1, %0;" ::"n"(NBAR) : "memory");
}
// The same barrier, returning the OR of `pred` over its threads: one decision
// that every participant sees alike.
template <int NBAR>
__device__ __forceinline__ bool group_sync_or(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n"
        " .reg .pred p, q;\n"
        " setp.ne.u32 p, %1, 0;\n"
        " bar.red.or.pred q, 1, %2, p;\n"
        " selp.u32 %0, 1, 0, q;\n"
        "}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "n"(NBAR)
        : "memory");
    return r != 0;
}

template <int LOG2L, int PASS, int E, int TF, int XS = 0, bool PK = false, int NBAR = 0>
__device__ __forceinline__ void stockham_passes(float2 (&v)[E], int t, float2* region, const float2* tw_smem) {
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
            float2 u[R];
#pragma unroll
            for (int j = 0; j < R; ++j) u[j] = v[q + j * NB];
            if constexpr (tw_split(LOG2L, PASS)) {
                const float2* tl = tw_smem + tw_offset(LOG2L, PASS) + (k & 15) * (R - 1) - 1;
                const float2* th = tw_smem + tw_offset(LOG2L, PASS) + (16 + (k >> 4)) * (R - 1) - 1;
#pragma unroll
                for (int j = 1; j < R; ++j) u[j] = cmul(u[j], cmul(tl[j], th[j]));
            } else if constexpr (PASS > 0) {
                const float2* tw = tw_smem + tw_offset(LOG2L, PASS) + k * (R - 1) - 1;
#pragma unroll
                for (int j = 1; j < R; ++j) u[j] = cmul(u[j], tw[j]);
            }
            Dft<R, PK>::run(u);
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
                for (int j = 0; j < R; ++j) region[xaddr<XS>(base + (j << LP))] = v[q + j * NB];
            }
            group_sync<NBAR>();
#pragma unroll
            for (int m = 0; m < E; ++m) v[m] = region[xaddr<XS>(t + m * TF)];
            group_sync<NBAR>();
            stockham_passes<LOG2L, PASS + 1, E, TF, XS, PK, NBAR>(v, t, region, tw_smem);
        }
    }
}

__host__ __device__ constexpr int floor_pow2(int v) {
    int p = 1;
    while (p * 2 <= v) p *= 2;
    return p;
}

// ---- asynchronous global -> shared copies (cp.async, 8 bytes) ----
__device__ __forceinline__ void cp_async8(float2* sdst, const float2* gsrc) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(sdst);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }

// Persistent, software-pipelined pass.  Each CTA walks tiles of K sub-FFTs
// (tile, tile + gridDim.x, ...).  Shared memory holds two padded tile
// buffers: while tile i is transformed in buffer i&1 (its load stage, then its
// exchange area, then its store stage), the copies of tile i+1 are already in
// flight into the other buffer, so HBM reads overlap the arithmetic.
//
// LMAP 0: every thread copies exactly the elements it later owns (pattern
//         t + m TF), so it only waits for its own copies;
// LMAP 1: the tile is K*L contiguous elements and is copied cooperatively,
//         element index fastest across the CTA (coalesced for tiny L).
// SMAP 0: stores straight from registers;
// SMAP 1: stores staged through shared memory, element index fastest;
// SMAP 2: staged, sub-FFT index fastest (coalesced strided columns).
// W_N lookups for the pre/post twiddles of a pass.  The launcher decides
// (PassArgs::tw_smem_levels) where the table lives: 2 -- the plan's two-level
// table staged in shared memory (N <= 2^22), 3 -- its three-level table staged
// (larger N: one more complex multiply instead of global-memory latency), 0 --
// the two-level table read from global memory.  The form is a compile-time
// choice so the unrolled lookups stay branch-free.  The first (low) table is
// padded by one entry per 16 so lanes striding through it by powers of two
// spread over the banks.
__host__ __device__ __forceinline__ int tw_pad(int i) { return i + (i >> 4); }

template <int LEVELS>
struct SmemTwiddle;

template <>
struct SmemTwiddle<2> {  // two-level: staged when tw_smem_levels == 2, else global
    const float2* lo;
    const float2* hi;
    uint32_t nmask, lo_mask;
    int lo_bits;
    bool staged, split;
    TwoLevel g;

    // Every thread of the block calls it; the caller's next barrier publishes the table.
    __device__ void setup(float2* smem, const PassArgs& a) {
        g = a.tw;
        staged = a.tw_smem_levels == 2;
        lo_bits = a.tw.lo_bits < a.tw.log2n ? a.tw.lo_bits : a.tw.log2n;
        split = a.tw.log2n > lo_bits;
        lo_mask = (1u << lo_bits) - 1u;
        nmask = a.tw.log2n >= 32 ? 0xffffffffu : (1u << a.tw.log2n) - 1u;
        const int nlo = 1 << lo_bits, nhi = split ? 1 << (a.tw.log2n - lo_bits) : 0;
        lo = smem;
        hi = smem + tw_pad(nlo);
        if (staged) {
            for (int i = threadIdx.x; i < nlo; i += blockDim.x) smem[tw_pad(i)] = a.tw.lo[i];
            for (int i = threadIdx.x; i < nhi; i += blockDim.x) smem[tw_pad(nlo) + i] = a.tw.hi[i];
        }
    }
    __device__ __forceinline__ float2 operator()(uint32_t e) const {
        if (!staged) return tw_two_level(g, e);
        e &= nmask;
        const uint32_t li = e & lo_mask;
        const float2 w = lo[tw_pad((int)li)];
        return split ? cmul(w, hi[e >> lo_bits]) : w;
    }
};

template <>
struct SmemTwiddle<3> {  // three-level, always staged
    const float2* t0;
    const float2* t1;
    const float2* t2;
    uint32_t nmask, mask;
    int bits;

    __device__ void setup(float2* smem, const PassArgs& a) {
        bits = a.tw.l3_bits;
        nmask = a.tw.log2n >= 32 ? 0xffffffffu : (1u << a.tw.log2n) - 1u;
        mask = (1u << bits) - 1u;
        const int nb = 1 << bits, stride = tw_pad(nb);
        t0 = smem;
        t1 = smem + stride;
        t2 = smem + 2 * stride;
        for (int i = threadIdx.x; i < 3 * nb; i += blockDim.x)
            smem[(i >> bits) * stride + tw_pad(i & (nb - 1))] = a.tw.l3[i];
    }
    __device__ __forceinline__ float2 operator()(uint32_t e) const {
        e &= nmask;
        const float2 w0 = t0[tw_pad((int)(e & mask))];
        const float2 w1 = t1[tw_pad((int)((e >> bits) & mask))];
        const float2 w2 = t2[tw_pad((int)(e >> (2 * bits)))];
        return cmul(cmul(w0, w1), w2);
    }
};

// Shared-memory entries the staged tables of `tw` take (0: no such table).
inline int tw_smem_entries_for(const TwoLevel& tw, int levels) {
    if (levels == 2) {
        const int lob = tw.lo_bits < tw.log2n ? tw.lo_bits : tw.log2n;
        return tw_pad(1 << lob) + (tw.log2n > lob ? 1 << (tw.log2n - lob) : 0);
    }
    if (levels == 3 && tw.l3 && tw.l3_bits > 0) return 3 * tw_pad(1 << tw.l3_bits);
    return 0;
}

// Staged form for a pass whose fixed shared memory is `base` bytes: the
// two-level table when it takes <= 4096 entries, else (when the kernel has a
// three-level form, max_levels 3) the three-level one, else none.  `cls` is
// the occupancy-cache class: 0 = nothing staged, else the table rounded up to
// a multiple of kTwClassEntries entries (fine enough that the rounding never
// costs a resident CTA).
constexpr int kTwClassEntries = 64;
constexpr int kTwClasses = 4096 / kTwClassEntries + 1;  // class 0..64
inline size_t tw_class_bytes(int cls) { return (size_t)cls * kTwClassEntries * sizeof(float2); }

inline void choose_tw_staging(PassArgs& pa, size_t base, size_t cap, int& cls, int max_levels = 2) {
    pa.tw_smem_entries = 0;
    pa.tw_smem_levels = 0;
    cls = 0;
    if (pa.tw_mode == 0) return;
    for (int levels = 2; levels <= max_levels; ++levels) {
        const int n = tw_smem_entries_for(pa.tw, levels);
        if (n <= 0 || n > 4096) continue;
        const int c = (n + kTwClassEntries - 1) / kTwClassEntries;
        if (base + tw_class_bytes(c) <= cap) {
            pa.tw_smem_entries = n;
            pa.tw_smem_levels = levels;
            cls = c;
            return;
        }
    }
}

template <int LOG2L, int LAYOUT, int LMAP, int SMAP>
struct PassKGeo {
    static constexpr int L = 1 << LOG2L;
    static constexpr int E = L < 16 ? L : 16;
    static constexpr int TF = L / E;
    static constexpr int LPAD = (L + (L >> 4)) | 1;  // odd: regions start on distinct banks
    // sub-FFTs per CTA: ~256 threads; >= 16 when the sub-FFT index is the
    // coalesced dimension (128-byte runs per element index: shorter runs
    // leave HBM bursts half used); capped so two tile buffers fit in 200 KB.
    static constexpr int KMIN = (LAYOUT || SMAP == 2) ? 16 : 1;
    static constexpr int K0 = TF >= 256 ? 1 : 256 / TF;
    static constexpr int KD = K0 > KMIN ? K0 : KMIN;
    static constexpr int KCAP = floor_pow2((200 * 1024) / (2 * LPAD * 8));
    static constexpr int K = KD < KCAP ? KD : KCAP;
    static constexpr int THREADS = K * TF;
    // resident CTAs the register budget is sized for (~768 threads per SM)
    static constexpr int MINB = THREADS >= 768 ? 1 : 768 / THREADS;
    static constexpr int NP = LOG2L <= 4 ? 1 : (LOG2L + 3) / 4;
    static constexpr size_t SMEM = (size_t)2 * K * LPAD * sizeof(float2) + (size_t)K * sizeof(int64_t) +
                                   (size_t)tw_total(LOG2L) * sizeof(float2);
};

template <int LOG2L, int LAYOUT, int LMAP, int SMAP>
__global__ void __launch_bounds__(PassKGeo<LOG2L, LAYOUT, LMAP, SMAP>::THREADS,
                                  PassKGeo<LOG2L, LAYOUT, LMAP, SMAP>::MINB)
    k_pass(const float2* __restrict__ in, float2* __restrict__ out, PassArgs a) {
    using G = PassKGeo<LOG2L, LAYOUT, LMAP, SMAP>;
    extern __shared__ __align__(16) float2 smem[];
    int64_t* sbase = reinterpret_cast<int64_t*>(smem + 2 * G::K * G::LPAD);
    float2* tw_smem = reinterpret_cast<float2*>(sbase + G::K);
    fill_stockham_twiddles<LOG2L>(tw_smem);  // visible after the first in-loop barrier
    SmemTwiddle<2> twiddle;  // W_N lookups, staged in shared memory when they fit
    twiddle.setup(tw_smem + tw_total(LOG2L), a);
    if (a.tw_smem_levels) __syncthreads();
    const int tid = threadIdx.x;
    const int cl = LAYOUT ? tid % G::K : tid / G::TF;
    const int t = LAYOUT ? tid / G::K : tid % G::TF;
    const int64_t ntiles = (a.nsub + G::K - 1) / G::K;
    const int64_t imask = (int64_t(1) << a.inner_log2) - 1;
    const uint32_t in_stride = (uint32_t)a.in_stride, out_stride = (uint32_t)a.out_stride;
    const float osr = a.scale, osi = a.conj_out ? -a.scale : a.scale;
    const bool scaled = a.scale != 1.0f || a.conj_out;  // uniform: skip the epilogue multiply when it is 1

    auto issue = [&](int64_t tile, float2* buf) {
        if (LMAP == 1) {
            const float2* src = in + tile * (int64_t)(G::K * G::L);
            const int64_t lim = (a.nsub - tile * G::K) * G::L;
#pragma unroll
            for (int i = 0; i < G::E; ++i) {
                const int g = tid + i * G::THREADS;
                if (g < lim) cp_async8(buf + (g >> LOG2L) * G::LPAD + pad16(g & (G::L - 1)), src + g);
            }
        } else {
            const int64_t f = tile * G::K + cl;
            if (f < a.nsub) {
                const int64_t o = f >> a.inner_log2, c = f & imask;
                const int64_t cin = a.in_base_bits ? (int64_t)brev_bits((uint32_t)c, a.in_base_bits) : c;
                const float2* src = in + o * a.in_outer + cin * a.in_inner;
                float2* dst = buf + cl * G::LPAD;
#pragma unroll
                for (int m = 0; m < G::E; ++m) {
                    const uint32_t e = (uint32_t)(t + m * G::TF);
                    const uint32_t pe = a.in_elem_bitrev ? brev_bits(e, LOG2L) : e;
                    cp_async8(dst + pad16((int)e), src + pe * in_stride);
                }
            }
        }
    };

    int64_t tile = blockIdx.x;
    if (tile < ntiles) issue(tile, smem);
    cp_async_commit();
    for (int it = 0; tile < ntiles; ++it, tile += gridDim.x) {
        float2* cur = smem + (it & 1) * (G::K * G::LPAD);
        float2* nxt = smem + ((it & 1) ^ 1) * (G::K * G::LPAD);
        if (tile + gridDim.x < ntiles) issue(tile + gridDim.x, nxt);
        cp_async_commit();
        cp_async_wait1();  // this tile's copies have landed (the next tile's may be in flight)
        if (LMAP == 1) __syncthreads();

        const int64_t f = tile * G::K + cl;
        const bool active = f < a.nsub;
        const int64_t o = f >> a.inner_log2, c = f & imask;
        if (SMAP != 0 && t == 0) {
            const int64_t cout = a.out_base_bits ? (int64_t)brev_bits((uint32_t)c, a.out_base_bits) : c;
            sbase[cl] = active ? o * a.out_outer + cout * a.out_inner : -1;
        }
        const uint32_t cmul32 = (uint32_t)c * (uint32_t)a.tw_mul;
        float2* region = cur + cl * G::LPAD;
        float2 v[G::E];
#pragma unroll
        for (int m = 0; m < G::E; ++m) {
            const int e = t + m * G::TF;
            float2 val = region[pad16(e)];
            if (a.conj_in) val.y = -val.y;
            if (a.tw_mode == 1) val = cmul(val, twiddle((uint32_t)e * cmul32));
            v[m] = val;
        }
        if (G::NP > 1 || SMAP != 0) __syncthreads();  // buffer becomes the exchange area

        stockham_passes<LOG2L, 0, G::E, G::TF, 0, true>(v, t, region, tw_smem);  // packed adds: +0-2 %

#pragma unroll
        for (int m = 0; m < G::E; ++m) {
            const int k = t + m * G::TF;
            float2 val = v[m];
            if (a.tw_mode == 2) val = cmul(val, twiddle((uint32_t)k * cmul32));
            v[m] = scaled ? make_float2(val.x * osr, val.y * osi) : val;
        }

        if constexpr (SMAP == 0) {
            if (active) {
                const int64_t cout = a.out_base_bits ? (int64_t)brev_bits((uint32_t)c, a.out_base_bits) : c;
                float2* dst = out + o * a.out_outer + cout * a.out_inner;
#pragma unroll
                for (int m = 0; m < G::E; ++m) {
                    const uint32_t k = (uint32_t)(t + m * G::TF);
                    const uint32_t pk = a.out_elem_bitrev ? brev_bits(k, LOG2L) : k;
                    dst[pk * out_stride] = v[m];
                }
            }
        } else {
#pragma unroll
            for (int m = 0; m < G::E; ++m) region[pad16(t + m * G::TF)] = v[m];
            __syncthreads();
#pragma unroll
            for (int i = 0; i < G::E; ++i) {
                const int idx = tid + i * G::THREADS;
                const int cl2 = SMAP == 1 ? idx >> LOG2L : idx % G::K;
                const uint32_t k = SMAP == 1 ? (uint32_t)(idx & (G::L - 1)) : (uint32_t)(idx / G::K);
                const int64_t base = sbase[cl2];
                if (base >= 0) {
                    const uint32_t pk = a.out_elem_bitrev ? brev_bits(k, LOG2L) : k;
                    out[base + pk * out_stride] = cur[cl2 * G::LPAD + pad16((int)k)];
                }
            }
        }
        __syncthreads();  // `cur` is refilled two tiles from now
    }
}

// Per-device launch facts (SM count, resident CTAs or clusters per kernel
// configuration), filled on first use under a mutex and read lock-free after.
static std::mutex g_sm_mu, g_occ_mu;
static std::atomic<int> g_sm_count[64];

template <typename F>
static cudaError_t cached_value(std::mutex& mu, std::atomic<int>& slot, int* out, F fill) {
    int v = slot.load(std::memory_order_acquire);
    if (v <= 0) {
        std::lock_guard<std::mutex> lk(mu);
        v = slot.load(std::memory_order_relaxed);
        if (v <= 0) {
            int nv = 0;
            const cudaError_t e = fill(&nv);
            if (e != cudaSuccess) return e;
            v = nv > 0 ? nv : 1;
            slot.store(v, std::memory_order_release);
        }
    }
    *out = v;
    return cudaSuccess;
}

cudaError_t device_sm_count(int dev, int* sms) {
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    return cached_value(g_sm_mu, g_sm_count[dev], sms, [&](int* v) {
        return cudaDeviceGetAttribute(v, cudaDevAttrMultiProcessorCount, dev);
    });
}

// Resident CTAs per SM of `kern` with `smem` dynamic bytes (cached in `slot`).
template <typename K>
static cudaError_t cached_occupancy(std::atomic<int>& slot, K kern, int threads, size_t smem, size_t smem_attr,
                                    int* out) {
    return cached_value(g_occ_mu, slot, out, [&](int* v) {
        cudaError_t e = cudaSuccess;
        if (smem_attr > 48 * 1024) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_attr);
        if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(v, kern, threads, smem);
        return e;
    });
}

template <int LOG2L, int LAYOUT, int LMAP, int SMAP>
static cudaError_t launch_pass_t(const float2* in, float2* out, const PassArgs& a, cudaStream_t s) {
    using G = PassKGeo<LOG2L, LAYOUT, LMAP, SMAP>;
    auto kern = k_pass<LOG2L, LAYOUT, LMAP, SMAP>;
    // Shared-memory W_N tables: up to 4096 entries (N <= 2^22); occupancy
    // is cached per device and table size class.
    constexpr size_t kSmemCap = 227 * 1024;
    static std::atomic<int> blocks_per_sm[64][kTwClasses];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    PassArgs b = a;
    int cls = 0;
    choose_tw_staging(b, G::SMEM, kSmemCap, cls);
    const size_t smem_cls = G::SMEM + tw_class_bytes(cls);
    int sms = 0, nb = 0;
    e = device_sm_count(dev, &sms);
    if (e == cudaSuccess) e = cached_occupancy(blocks_per_sm[dev][cls], kern, G::THREADS, smem_cls, kSmemCap, &nb);
    if (e != cudaSuccess) return e;
    const int64_t ntiles = (b.nsub + G::K - 1) / G::K;
    int64_t grid = (int64_t)nb * sms;
    if (grid > ntiles) grid = ntiles;
    if (grid < 1) grid = 1;
    const size_t smem = G::SMEM + (size_t)b.tw_smem_entries * sizeof(float2);
    kern<<<(unsigned)grid, G::THREADS, smem, s>>>(in, out, b);
    return cudaGetLastError();
}

template <int LOG2L>
static cudaError_t launch_pass_l(int layout, int lmap, int smap, const float2* in, float2* out,
                                 const PassArgs& a, cudaStream_t s) {
    if (layout) {  // columns: per-thread loads, stores direct or staged element-fastest
        return smap == 1 ? launch_pass_t<LOG2L, 1, 0, 1>(in, out, a, s) : launch_pass_t<LOG2L, 1, 0, 0>(in, out, a, s);
    }
    if (lmap) {
        return smap == 2 ? launch_pass_t<LOG2L, 0, 1, 2>(in, out, a, s)
             : smap == 1 ? launch_pass_t<LOG2L, 0, 1, 1>(in, out, a, s)
                         : launch_pass_t<LOG2L, 0, 1, 0>(in, out, a, s);
    }
    return smap == 2 ? launch_pass_t<LOG2L, 0, 0, 2>(in, out, a, s)
         : smap == 1 ? launch_pass_t<LOG2L, 0, 0, 1>(in, out, a, s)
                     : launch_pass_t<LOG2L, 0, 0, 0>(in, out, a, s);
}

}  // namespace bfft

#include "bfft_pass_tma.cuh"
#include "bfft_pair.cuh"
#include "bfft_fused.cuh"
#include "bfft_rows_pair.cuh"
#include "bfft_tc.cuh"

namespace bfft {

// Failure-detection probe: one thread waits, through the same bounded waits the
// kernels use, on an mbarrier that nothing arrives on and on a counter that
// nothing increments.  Each wait gives up after kWaitLimitNs, records its bit
// in the status word (0: mbarrier, 1: dependency counter) and the kernel
// returns normally -- the context stays usable.
__device__ uint32_t g_probe_counter;  // never incremented

__global__ void k_wait_probe() {
    __shared__ uint64_t bar;
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    (void)mbar_wait_bounded(&bar, 0);
    (void)counter_wait_bounded(&g_probe_counter, 1u);
}

cudaError_t run_wait_probe(cudaStream_t s) {
    k_wait_probe<<<1, 1, 0, s>>>();
    return cudaGetLastError();
}

cudaError_t read_device_status(unsigned* status, bool clear) {
    cudaError_t e = cudaMemcpyFromSymbol(status, g_kernel_status, sizeof(unsigned));
    if (e == cudaSuccess && clear) {
        const unsigned zero = 0;
        e = cudaMemcpyToSymbol(g_kernel_status, &zero, sizeof(unsigned));
    }
    return e;
}

// ---- rows of 2 points: one row per thread, in registers ----
//
// A 2-point row is one 16-byte vector: each thread loads its row, runs the
// butterfly in registers and stores it -- a warp reads and writes 512
// contiguous bytes, no shared memory, no barriers.  (The same kernel for 4..16
// points, each row a few 16-byte loads of one thread, measured 0-22 % slower
// than the k_pass row tile: a warp's loads touch 32 lines at a time.)
template <int LOG2L>
__global__ void __launch_bounds__(256) k_rows_regs(const float2* __restrict__ in, float2* __restrict__ out,
                                                   PassArgs a) {
    constexpr int L = 1 << LOG2L;
    const int64_t imask = (int64_t(1) << a.inner_log2) - 1;
    const float osr = a.scale, osi = a.conj_out ? -a.scale : a.scale;
    const bool scaled = a.scale != 1.0f || a.conj_out;
    for (int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; f < a.nsub;
         f += (int64_t)gridDim.x * blockDim.x) {
        const int64_t o = f >> a.inner_log2, c = f & imask;
        const int64_t cin = a.in_base_bits ? (int64_t)brev_bits((uint32_t)c, a.in_base_bits) : c;
        const int64_t cout = a.out_base_bits ? (int64_t)brev_bits((uint32_t)c, a.out_base_bits) : c;
        const float4* src = reinterpret_cast<const float4*>(in + o * a.in_outer + cin * a.in_inner);
        float4* dst = reinterpret_cast<float4*>(out + o * a.out_outer + cout * a.out_inner);
        float2 v[L];
#pragma unroll
        for (int j = 0; j < L / 2; ++j) {
            const float4 q = __ldg(src + j);
            v[2 * j] = make_float2(q.x, a.conj_in ? -q.y : q.y);
            v[2 * j + 1] = make_float2(q.z, a.conj_in ? -q.w : q.w);
        }
        Dft<L, true>::run(v);
        if (scaled) {
#pragma unroll
            for (int m = 0; m < L; ++m) v[m] = make_float2(v[m].x * osr, v[m].y * osi);
        }
#pragma unroll
        for (int j = 0; j < L / 2; ++j) __stcs(dst + j, make_float4(v[2 * j].x, v[2 * j].y, v[2 * j + 1].x, v[2 * j + 1].y));
    }
}

template <int LOG2L>
static cudaError_t launch_rows_regs_t(const float2* in, float2* out, const PassArgs& a, cudaStream_t s) {
    k_rows_regs<LOG2L><<<flat_grid(a.nsub, 256), 256, 0, s>>>(in, out, a);
    return cudaGetLastError();
}

// ---- adjacent short rows (L = 16..64 points): shuffles instead of shared memory ----
//
// G = L/2 lanes share a row, each holding two consecutive elements (one
// 16-byte vector), so a warp's eight fully coalesced 16-byte loads cover
// 8 * 32/G adjacent rows: in load j, lane l holds elements 2i, 2i+1
// (i = l mod G) of row 8 (32/G) g + j (32/G) + l/G.  An L-point DFT is
// X[k1 + (L/2) k2] = Y0[k1] + (-1)^k2 W_L^k1 Y1[k1] with Ys the (L/2)-point
// DFT of the elements 2i + s; the row's G lanes compute both with log2 G
// radix-2 decimation-in-frequency steps across lanes (shfl_xor G/2 .. 1),
// after which lane i holds Ys[bitrev(i)].  All eight loads are in flight
// before the first shuffle; no shared memory, no barriers.  Measured against
// the shared-memory row passes on B*N = 2^24: 16 points 63.5 -> 51.5 µs,
// 32 points 59.5 -> 51.2, 64 points 57.0 -> 55.0; for 4 and 8 points the
// k_pass row tile is as fast or faster.
template <int LOG2L>
__global__ void __launch_bounds__(256) k_rows_shfl(const float2* __restrict__ in, float2* __restrict__ out,
                                                   int64_t nrows, int conj_in, int conj_out, float scale) {
    constexpr int L = 1 << LOG2L, G = L / 2, LG = LOG2L - 1, RPL = 32 / G;  // rows per load
    const int lane = threadIdx.x & 31, i = lane & (G - 1);
    const int k1 = LG ? (int)(__brev((unsigned)i) >> (32 - LG)) : 0;
    // step q (h = G >> (q + 1)), branch-free: y <- (p + sgn y) * w with
    // sgn = +1, w = 1 on the lower lane of a pair and sgn = -1,
    // w = W_{2h}^(i mod h) on the upper one
    float2 wstep[LG > 0 ? LG : 1];
    float sgn[LG > 0 ? LG : 1];
#pragma unroll
    for (int q = 0; q < LG; ++q) {
        const int h = G >> (q + 1);
        const bool upper = i & h;
        sgn[q] = upper ? -1.f : 1.f;
        wstep[q] = upper ? g_tw_levels[2 * h + (i & (h - 1))] : make_float2(1.f, 0.f);
    }
    const float2 wl = g_tw_levels[L + k1];  // W_L^k1
    const float osr = scale, osi = conj_out ? -scale : scale;
    const int64_t groups = (nrows + 8 * RPL - 1) / (8 * RPL);
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t g = warp; g < groups; g += nwarps) {
        const int64_t r0 = g * 8 * RPL;
        const float4* src = reinterpret_cast<const float4*>(in + r0 * L);
        float4 q[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            q[j] = r0 + j * RPL + lane / G < nrows ? __ldcs(src + lane + 32 * j) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t row = r0 + j * RPL + lane / G;
            float2 y[2] = {make_float2(q[j].x, conj_in ? -q[j].y : q[j].y),
                           make_float2(q[j].z, conj_in ? -q[j].w : q[j].w)};
#pragma unroll
            for (int st = 0; st < LG; ++st) {
                const int h = G >> (st + 1);
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    const float2 p = make_float2(__shfl_xor_sync(0xffffffffu, y[u].x, h, G),
                                                 __shfl_xor_sync(0xffffffffu, y[u].y, h, G));
                    const float2 d = make_float2(fmaf(sgn[st], y[u].x, p.x), fmaf(sgn[st], y[u].y, p.y));
                    y[u] = h > 1 ? cmul(d, wstep[st]) : d;
                }
            }
            const float2 t = cmul(y[1], wl);
            const float2 lo = cadd(y[0], t), hi = csub(y[0], t);
            if (row < nrows) {
                float2* d = out + row * L;
                __stcs(d + k1, make_float2(lo.x * osr, lo.y * osi));
                __stcs(d + k1 + G, make_float2(hi.x * osr, hi.y * osi));
            }
        }
    }
}

// 128-point rows: the same scheme with four elements per lane.  Lane i of
// the warp holds x[4i + s] (s < 4, two 16-byte loads), the four 32-point DFTs
// Ys over i run across all 32 lanes (five shfl_xor steps), and lane i forms
// X[k1 + 32 k2] = DFT4_s(W128^(s k1) Ys[k1])[k2] for k1 = bitrev5(i).  A warp
// takes 4 rows per iteration, eight loads in flight.
__global__ void __launch_bounds__(256) k_rows_shfl128(const float2* __restrict__ in, float2* __restrict__ out,
                                                      int64_t nrows, int conj_in, int conj_out, float scale) {
    const int i = threadIdx.x & 31;
    const int k1 = (int)(__brev((unsigned)i) >> 27);
    float2 wstep[5];
    float sgn[5];
#pragma unroll
    for (int q = 0; q < 5; ++q) {
        const int h = 16 >> q;
        const bool upper = i & h;
        sgn[q] = upper ? -1.f : 1.f;
        wstep[q] = upper ? g_tw_levels[2 * h + (i & (h - 1))] : make_float2(1.f, 0.f);
    }
    const float2 w1 = g_tw_levels[128 + k1], w2 = g_tw_levels[128 + 2 * k1], w3 = g_tw_levels[128 + 3 * k1];
    const float osr = scale, osi = conj_out ? -scale : scale;
    const int64_t groups = (nrows + 3) >> 2;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t g = warp; g < groups; g += nwarps) {
        const int64_t r0 = g << 2;
        float4 q[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int64_t row = r0 + (j >> 1);
            q[j] = row < nrows ? __ldg(reinterpret_cast<const float4*>(in + row * 128) + 2 * i + (j & 1))
                               : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const int64_t row = r0 + r;
            const float4 a = q[2 * r], b = q[2 * r + 1];
            float2 y[4] = {make_float2(a.x, conj_in ? -a.y : a.y), make_float2(a.z, conj_in ? -a.w : a.w),
                           make_float2(b.x, conj_in ? -b.y : b.y), make_float2(b.z, conj_in ? -b.w : b.w)};
#pragma unroll
            for (int st = 0; st < 5; ++st) {
                const int h = 16 >> st;
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float2 p = make_float2(__shfl_xor_sync(0xffffffffu, y[u].x, h),
                                                 __shfl_xor_sync(0xffffffffu, y[u].y, h));
                    const float2 d = make_float2(fmaf(sgn[st], y[u].x, p.x), fmaf(sgn[st], y[u].y, p.y));
                    y[u] = h > 1 ? cmul(d, wstep[st]) : d;
                }
            }
            y[1] = cmul(y[1], w1);
            y[2] = cmul(y[2], w2);
            y[3] = cmul(y[3], w3);
            Dft<4, true>::run(y);
            if (row < nrows) {
                float2* d = out + row * 128;
#pragma unroll
                for (int k2 = 0; k2 < 4; ++k2) __stcs(d + k1 + 32 * k2, make_float2(y[k2].x * osr, y[k2].y * osi));
            }
        }
    }
}

// Adjacent rows of 16..128 points (row f at f * L), 16-byte aligned, without
// W_N twiddles or bit-reversed addressing: the shuffle kernel.
static cudaError_t launch_rows_shfl(int log2l, const float2* in, float2* out, const PassArgs& a, cudaStream_t s) {
    if (log2l < 4 || log2l > 7) return cudaErrorNotSupported;
    const int64_t L = int64_t(1) << log2l;
    const int64_t inner = int64_t(1) << a.inner_log2;
    if (((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) || a.in_stride != 1 ||
        a.out_stride != 1 || a.in_elem_bitrev || a.out_elem_bitrev || a.tw_mode != 0 || a.in_base_bits ||
        a.out_base_bits)
        return cudaErrorNotSupported;
    auto adjacent = [&](int64_t outer, int64_t inner_stride) {
        return inner == 1 ? outer == L : (inner_stride == L && outer == inner * L);
    };
    if (!adjacent(a.in_outer, a.in_inner) || !adjacent(a.out_outer, a.out_inner)) return cudaErrorNotSupported;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = device_sm_count(dev, &sms);
    if (e != cudaSuccess) return e;
    const int64_t rows_per_warp = L == 128 ? 4 : 8 * (64 / L);
    int64_t blocks = ((a.nsub + rows_per_warp - 1) / rows_per_warp + 7) / 8;  // 8 warps per block
    if (blocks > (int64_t)sms * 8) blocks = (int64_t)sms * 8;
    if (blocks < 1) blocks = 1;
    switch (log2l) {
        case 4: k_rows_shfl<4><<<(unsigned)blocks, 256, 0, s>>>(in, out, a.nsub, a.conj_in, a.conj_out, a.scale); break;
        case 5: k_rows_shfl<5><<<(unsigned)blocks, 256, 0, s>>>(in, out, a.nsub, a.conj_in, a.conj_out, a.scale); break;
        case 6: k_rows_shfl<6><<<(unsigned)blocks, 256, 0, s>>>(in, out, a.nsub, a.conj_in, a.conj_out, a.scale); break;
        case 7: k_rows_shfl128<<<(unsigned)blocks, 256, 0, s>>>(in, out, a.nsub, a.conj_in, a.conj_out, a.scale); break;
        default: return cudaErrorNotSupported;
    }
    return cudaGetLastError();
}

// The register-only row kernel when the shape allows it (rows of 2
// contiguous points, every row start 16-byte aligned, no W_N twiddle).
static cudaError_t launch_rows_regs(int log2l, const float2* in, float2* out, const PassArgs& a, cudaStream_t s) {
    if (log2l != 1) return cudaErrorNotSupported;
    const int64_t inner = int64_t(1) << a.inner_log2;
    if (((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) || a.in_stride != 1 ||
        a.out_stride != 1 || a.in_elem_bitrev || a.out_elem_bitrev || a.tw_mode != 0)
        return cudaErrorNotSupported;
    if ((a.in_outer & 1) || (inner > 1 && (a.in_inner & 1)) || (a.out_outer & 1) || (inner > 1 && (a.out_inner & 1)))
        return cudaErrorNotSupported;
    return launch_rows_regs_t<1>(in, out, a, s);
}

cudaError_t launch_pass(int log2l, int layout, int lmap, int smap, const float2* in, float2* out,
                        const PassArgs& a, cudaStream_t s) {
    if (layout == 1) {  // column tiles: TMA-staged pass when the shape allows it
        const cudaError_t e = launch_pass_tma(log2l, in, out, a, s);
        if (e != cudaErrorNotSupported) return e;
    } else if (smap != 2) {  // row tiles with row outputs: bulk-copy pass when the shape allows it
        cudaError_t e = log2l == 1 ? launch_rows_regs(log2l, in, out, a, s) : launch_rows_shfl(log2l, in, out, a, s);
        if (e != cudaErrorNotSupported) return e;
        e = launch_rows_pair(log2l, in, out, a, s);
        if (e != cudaErrorNotSupported) return e;
        e = launch_pass_tma_rows(log2l, in, out, a, s);
        if (e != cudaErrorNotSupported) return e;
    }
    switch (log2l) {
        case 1: return launch_pass_l<1>(layout, lmap, smap, in, out, a, s);
        case 2: return launch_pass_l<2>(layout, lmap, smap, in, out, a, s);
        case 3: return launch_pass_l<3>(layout, lmap, smap, in, out, a, s);
        case 4: return launch_pass_l<4>(layout, lmap, smap, in, out, a, s);
        case 5: return launch_pass_l<5>(layout, lmap, smap, in, out, a, s);
        case 6: return launch_pass_l<6>(layout, lmap, smap, in, out, a, s);
        case 7: return launch_pass_l<7>(layout, lmap, smap, in, out, a, s);
        case 8: return launch_pass_l<8>(layout, lmap, smap, in, out, a, s);
        case 9: return launch_pass_l<9>(layout, lmap, smap, in, out, a, s);
        case 10: return launch_pass_l<10>(layout, lmap, smap, in, out, a, s);
        case 11: return launch_pass_l<11>(layout, lmap, smap, in, out, a, s);
        case 12: return launch_pass_l<12>(layout, lmap, smap, in, out, a, s);
        default: return cudaErrorInvalidValue;
    }
}

// ============================================================== cluster FFT
//
// One HBM round trip for 4096 < N <= 65536: the 4-step N = N1 * N2 runs on a
// thread-block cluster of P CTAs.  CTA r of the cluster owns columns
// n2 in [r*N2/P, (r+1)*N2/P) for the N1-point column FFTs (stride-N2 loads,
// coalesced across its columns), multiplies by W_N^{n2 k1} and leaves the
// result in its shared memory; after a cluster barrier every CTA gathers its
// rows k1 in [r*N1/P, (r+1)*N1/P) from all P CTAs through distributed shared
// memory, runs the N2-point row FFTs and stores X[k1 + N1 k2] (staged so the
// store is coalesced across its rows).  Persistent over the batch: the next
// transform's columns are copied in with cp.async while the current one is
// gathered, transformed and stored.  Synchronisation is the hardware cluster
// barrier only (every CTA runs the same iterations), and a final barrier keeps
// each CTA's shared memory alive until the others have finished reading it.
template <int LOG2N1, int LOG2N2, int LOG2P>
struct CluGeo {
    static constexpr int N1 = 1 << LOG2N1, N2 = 1 << LOG2N2, P = 1 << LOG2P;
    static constexpr int64_t N = (int64_t)N1 * N2;
    static constexpr int LOG2CA = LOG2N2 - LOG2P;
    static constexpr int CA = N2 / P;  // pass-A columns per CTA
    static constexpr int RB = N1 / P;  // pass-B rows per CTA
    static constexpr int M = N1 * N2 / P;
    static constexpr int E = 16;
    static constexpr int TFA = N1 / E, TFB = N2 / E;
    static constexpr int THREADS = M / E;
    static constexpr int MINB = THREADS >= 768 ? 1 : 768 / THREADS;
    static constexpr int LPADA = (N1 + (N1 >> 4)) | 1;
    static constexpr int LPADB = (N2 + (N2 >> 4)) | 1;
    static constexpr int XSZ = CA * LPADA;
    static constexpr int YSZ = M > RB * LPADB ? M : RB * LPADB;
    static constexpr int TWA = tw_total(LOG2N1), TWB = tw_total(LOG2N2);
    static constexpr size_t SMEM = (size_t)(XSZ + YSZ + TWA + TWB) * sizeof(float2);
};

__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;\n" ::: "memory"); }

template <int LOG2N1, int LOG2N2, int LOG2P>
__global__ void __launch_bounds__(CluGeo<LOG2N1, LOG2N2, LOG2P>::THREADS, CluGeo<LOG2N1, LOG2N2, LOG2P>::MINB)
    k_cluster_fft(const float2* __restrict__ in, float2* __restrict__ out, ClusterArgs a) {
    using G = CluGeo<LOG2N1, LOG2N2, LOG2P>;
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(16) float2 smem[];
    float2* X = smem;
    float2* Y = smem + G::XSZ;
    float2* twA = Y + G::YSZ;
    float2* twB = twA + G::TWA;
    fill_stockham_twiddles<LOG2N1>(twA);  // visible after the first in-loop barrier
    fill_stockham_twiddles<LOG2N2>(twB);
    const int rank = (int)cluster.block_rank();
    const int64_t cid = blockIdx.x / G::P;
    const int64_t nclu = gridDim.x / G::P;
    const int tid = threadIdx.x;
    const int clA = tid % G::CA, tA = tid / G::CA;    // pass A: column fastest
    const int rlB = tid / G::TFB, tB = tid % G::TFB;  // pass B: element fastest
    const int n2 = rank * G::CA + clA;
    const int k1 = rank * G::RB + rlB;
    float2* regA = X + clA * G::LPADA;
    float2* regB = Y + rlB * G::LPADB;
    const float osr = a.scale, osi = a.conj_out ? -a.scale : a.scale;

    auto issue = [&](int64_t b) {
        const float2* src = in + b * G::N + n2;
#pragma unroll
        for (int m = 0; m < G::E; ++m) {
            const int e = tA + m * G::TFA;
            cp_async8(regA + pad16(e), src + (int64_t)e * G::N2);
        }
    };

    int64_t b = cid;
    if (b < a.batch) issue(b);
    cp_async_commit();
    for (; b < a.batch; b += nclu) {
        cp_async_wait0();
        float2 v[G::E];
#pragma unroll
        for (int m = 0; m < G::E; ++m) {
            float2 val = regA[pad16(tA + m * G::TFA)];
            if (a.conj_in) val.y = -val.y;
            v[m] = val;
        }
        __syncthreads();
        stockham_passes<LOG2N1, 0, G::E, G::TFA, 0, true>(v, tA, regA, twA);  // packed adds: +4 %
#pragma unroll
        for (int m = 0; m < G::E; ++m) {
            const int k = tA + m * G::TFA;
            Y[k * G::CA + clA] = cmul(v[m], tw_two_level(a.tw, (uint32_t)(n2 * k)));
        }
        cluster.sync();  // every CTA's twiddled columns are in place
        if (b + nclu < a.batch) issue(b + nclu);
        cp_async_commit();
#pragma unroll
        for (int m = 0; m < G::E; ++m) {
            const int n = tB + m * G::TFB;
            const float2* rp = cluster.map_shared_rank(Y + (k1 * G::CA + (n & (G::CA - 1))), n >> G::LOG2CA);
            v[m] = *rp;
        }
        cluster.sync();  // all remote reads of Y are done
        stockham_passes<LOG2N2, 0, G::E, G::TFB, 0, true>(v, tB, regB, twB);
#pragma unroll
        for (int m = 0; m < G::E; ++m) regB[pad16(tB + m * G::TFB)] = make_float2(v[m].x * osr, v[m].y * osi);
        __syncthreads();
        float2* dst = out + b * G::N + rank * G::RB;
#pragma unroll
        for (int i = 0; i < G::E; ++i) {
            const int idx = tid + i * G::THREADS;
            const int rl2 = idx % G::RB, k2 = idx / G::RB;
            dst[rl2 + (int64_t)G::N1 * k2] = Y[rl2 * G::LPADB + pad16(k2)];
        }
        __syncthreads();
    }
    cluster.sync();
}

template <int LOG2N1, int LOG2N2, int LOG2P>
static cudaError_t launch_cluster_t(const float2* in, float2* out, const ClusterArgs& a, cudaStream_t s) {
    using G = CluGeo<LOG2N1, LOG2N2, LOG2P>;
    auto kern = k_cluster_fft<LOG2N1, LOG2N2, LOG2P>;
    static std::atomic<int> max_clusters[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = G::P;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(G::THREADS);
    cfg.dynamicSmemBytes = G::SMEM;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int sms = 0, nc = 0;
    e = device_sm_count(dev, &sms);
    if (e == cudaSuccess)
        e = cached_value(g_occ_mu, max_clusters[dev], &nc, [&](int* v) {
            cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)G::SMEM);
            if (e2 == cudaSuccess && G::P > 8)
                e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
            cudaLaunchConfig_t q = cfg;
            q.gridDim = dim3((unsigned)(G::P * sms));
            if (e2 == cudaSuccess) e2 = cudaOccupancyMaxActiveClusters(v, kern, &q);
            return e2;
        });
    if (e != cudaSuccess) return e;
    int64_t nclu = nc;
    if (nclu > a.batch) nclu = a.batch;
    cfg.gridDim = dim3((unsigned)(nclu * G::P));
    e = cudaLaunchKernelEx(&cfg, kern, in, out, a);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

bool cluster_supported(int log2n) { return log2n >= 13 && log2n <= 16; }

cudaError_t launch_cluster_fft(int log2n, const float2* in, float2* out, const ClusterArgs& a, cudaStream_t s) {
    switch (log2n) {
        case 13: return launch_cluster_t<6, 7, 1>(in, out, a, s);
        case 14: return launch_cluster_t<7, 7, 2>(in, out, a, s);
        case 15: return launch_cluster_t<7, 8, 3>(in, out, a, s);
        case 16: {
            // 16-CTA clusters (non-portable size) keep 4096 points per CTA and
            // three CTAs per SM; fall back to portable 8-CTA clusters.
            cudaError_t e = launch_cluster_t<8, 8, 4>(in, out, a, s);
            if (e == cudaErrorInvalidValue || e == cudaErrorInvalidConfiguration ||
                e == cudaErrorNotSupported || e == cudaErrorInvalidClusterSize) {
                (void)cudaGetLastError();
                e = launch_cluster_t<8, 8, 3>(in, out, a, s);
            }
            return e;
        }
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace bfft
