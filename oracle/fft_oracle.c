/*
 * fft_oracle.c -- TEST INFRASTRUCTURE ONLY.
 *
 * A plain-C, CPU-only restatement of the Kunlunxin-FFT reference arithmetic
 * for the 1-D power-of-two complex FFT hot path.  It exists to CHECK the B200
 * CUDA library; it is never linked into, loaded by, or called from the
 * product path.  Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference legs may load it (through oracle/oracle.py).
 *
 * Every function restates one reference routine and cites it (paths are
 * relative to the reference project root).  Data is interleaved complex
 * (re, im pairs), batch-major (B, N), exactly like the public complex64
 * layout; the reference's planar split is an internal detail of its Triton
 * backend and does not change any arithmetic.
 *
 * Float32 routines reproduce the reference's FP32 dataflow: the same stage
 * order, index maps, twiddle addressing and operation order (each product
 * and sum rounded separately -- build with -ffp-contract=off).  Float64
 * routines reproduce include/butterfly/fft.hpp (the reference's native C++
 * CPU path).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifndef M_PI
#define M_PI 3.14159265358979323846
#endif

/* ------------------------------------------------------------------ */
/* Index maps (must be bit-exact)                                      */
/* ------------------------------------------------------------------ */

/* Reverse the low `bits` bits of x.
 * Reference: include/butterfly/bit_reverse.hpp:15-22, src/xpu/kernels.py:27-38. */
uint32_t bfo_bit_reverse(uint32_t x, int bits) {
    uint32_t r = 0;
    for (int b = 0; b < bits; ++b) {
        r = (r << 1) | (x & 1u);
        x >>= 1;
    }
    return r;
}

/* DIT input permutation of the radix-4 cascade: radix-4 digits taken from the
 * low end, an odd top bit moves to bit 0.  Reference: src/xpu/kernels.py:41-57. */
uint32_t bfo_dit_digit_reverse(uint32_t x, int bits) {
    uint32_t r = 0;
    for (int q = 0; q < bits / 2; ++q) {
        uint32_t d = (x >> (2 * q)) & 3u;
        r |= d << (bits - 2 * q - 2);
    }
    if (bits & 1) r |= (x >> (bits - 1)) & 1u;
    return r;
}

/* DIF output permutation of the radix-4 cascade: for odd `bits` the 1-bit digit
 * sits at the bottom of the input index and takes the top output weight.
 * Reference: src/xpu/kernels.py:60-78. */
uint32_t bfo_dif_digit_reverse(uint32_t x, int bits) {
    if (!(bits & 1)) return bfo_dit_digit_reverse(x, bits);
    uint32_t r = (x & 1u) << (bits - 1);
    for (int q = 1; q <= bits / 2; ++q) {
        uint32_t d = (x >> (2 * q - 1)) & 3u;
        r |= d << (bits - 1 - 2 * q);
    }
    return r;
}

void bfo_index_table(int kind, int bits, uint32_t* out) {
    uint32_t n = 1u << bits;
    for (uint32_t i = 0; i < n; ++i) {
        out[i] = kind == 0 ? bfo_bit_reverse(i, bits)
               : kind == 1 ? bfo_dit_digit_reverse(i, bits)
                           : bfo_dif_digit_reverse(i, bits);
    }
}

static int ilog2(int64_t n) {
    int b = 0;
    while (((int64_t)1 << b) < n) ++b;
    return b;
}

/* ------------------------------------------------------------------ */
/* Twiddles                                                            */
/* ------------------------------------------------------------------ */

/* cos/sin of the FP32 angle (-2*pi*idx)/n for idx < count, formed the way the
 * reference's torch code forms it: an FP32 product then an FP32 quotient.
 * Reference: src/xpu/runner.py:93-97 (count = n/2) and :1650-1658
 * (_real_twiddle, count = n/2 + 1). */
void bfo_twiddle_f32(int64_t n, int64_t count, float* wr, float* wi) {
    const float c = (float)(-2.0 * M_PI);
    for (int64_t idx = 0; idx < count; ++idx) {
        float ang = (c * (float)idx) / (float)n;
        wr[idx] = cosf(ang);
        wi[idx] = sinf(ang);
    }
}

/* ------------------------------------------------------------------ */
/* Radix-2 global stages (M0 / M4)                                     */
/* ------------------------------------------------------------------ */

/* One radix-2 DIT stage on one row.  Reference: src/xpu/kernels.py:100-163
 * (dit_stage_kernel) and :993-1060 (dit_stage_batch_kernel):
 *   k in [0,N/2): j = k % n, i = (k/n)*2n + j
 *   a = X[i], b = X[i+n]*W[j*M];  Y[i] = a+b, Y[i+n] = a-b
 * with an optional bit-reversed read of the inputs (stage 0). */
static void dit_stage_row(const float* X, float* Y, int64_t n, int64_t M, int64_t N,
                          int bits, int bitrev_in, const float* wr, const float* wi) {
    for (int64_t k = 0; k < N / 2; ++k) {
        int64_t j = k % n;
        int64_t i = ((k / n) * 2) * n + j;
        int64_t s0 = bitrev_in ? bfo_bit_reverse((uint32_t)i, bits) : i;
        int64_t s1 = bitrev_in ? bfo_bit_reverse((uint32_t)(i + n), bits) : i + n;
        int64_t w = j * M;
        float ar = X[2 * s0], ai = X[2 * s0 + 1];
        float br = X[2 * s1], bi = X[2 * s1 + 1];
        float brw = br * wr[w] - bi * wi[w];
        float biw = br * wi[w] + bi * wr[w];
        Y[2 * i] = ar + brw;
        Y[2 * i + 1] = ai + biw;
        Y[2 * (i + n)] = ar - brw;
        Y[2 * (i + n) + 1] = ai - biw;
    }
}

/* One radix-2 DIF stage on one row; rev_mode 0 natural, 1 bit-reversed,
 * 2 DIF digit-reversed output.  Reference: src/xpu/kernels.py:166-236
 * (dif_stage_kernel), :1063-1124 (dif_stage_batch_kernel) and :813-867
 * (dif_stage2_batch_kernel). */
static void dif_stage_row(const float* X, float* Y, int64_t n, int64_t M, int64_t N,
                          int bits, int rev_mode, const float* wr, const float* wi) {
    for (int64_t k = 0; k < N / 2; ++k) {
        int64_t j = k % n;
        int64_t i = ((k / n) * 2) * n + j;
        int64_t w = j * M;
        float ar = X[2 * i], ai = X[2 * i + 1];
        float br = X[2 * (i + n)], bi = X[2 * (i + n) + 1];
        float sr = ar + br, si = ai + bi;
        float dr = ar - br, di = ai - bi;
        float drw = dr * wr[w] - di * wi[w];
        float diw = dr * wi[w] + di * wr[w];
        int64_t d0 = i, d1 = i + n;
        if (rev_mode == 1) {
            d0 = bfo_bit_reverse((uint32_t)i, bits);
            d1 = bfo_bit_reverse((uint32_t)(i + n), bits);
        } else if (rev_mode == 2) {
            d0 = bfo_dif_digit_reverse((uint32_t)i, bits);
            d1 = bfo_dif_digit_reverse((uint32_t)(i + n), bits);
        }
        Y[2 * d0] = sr;
        Y[2 * d0 + 1] = si;
        Y[2 * d1] = drw;
        Y[2 * d1 + 1] = diw;
    }
}

/* M0 / M4 radix-2 FFT of `batch` rows of length n (interleaved complex f32).
 * DIT: stages n=1..N/2, bit-reversal folded into stage 0
 *      (src/xpu/runner.py:118-163 fft_dit, :781-841 fft_dit_batch).
 * DIF: stages n=N/2..1, bit-reversal folded into the last stage
 *      (src/xpu/runner.py:166-206 fft_dif, :844-896 fft_dif_batch). */
int bfo_fft_radix2_f32(const float* x, float* y, int64_t n, int64_t batch, int dif) {
    if (n < 1 || (n & (n - 1))) return 1;
    int bits = ilog2(n);
    float* wr = (float*)malloc(sizeof(float) * (size_t)(n / 2 + 1));
    float* wi = (float*)malloc(sizeof(float) * (size_t)(n / 2 + 1));
    float* a = (float*)malloc(sizeof(float) * 2 * (size_t)n);
    float* b = (float*)malloc(sizeof(float) * 2 * (size_t)n);
    bfo_twiddle_f32(n, n / 2, wr, wi);
    for (int64_t r = 0; r < batch; ++r) {
        const float* src = x + 2 * n * r;
        memcpy(a, src, sizeof(float) * 2 * (size_t)n);
        if (n == 1) {
            memcpy(y + 2 * n * r, a, sizeof(float) * 2);
            continue;
        }
        if (!dif) {
            for (int s = 0; s < bits; ++s) {
                int64_t sn = (int64_t)1 << s;
                dit_stage_row(a, b, sn, n / (sn * 2), n, bits, s == 0, wr, wi);
                float* t = a; a = b; b = t;
            }
        } else {
            for (int s = bits - 1; s >= 0; --s) {
                int64_t sn = (int64_t)1 << s;
                dif_stage_row(a, b, sn, n / (sn * 2), n, bits, s == 0 ? 1 : 0, wr, wi);
                float* t = a; a = b; b = t;
            }
        }
        memcpy(y + 2 * n * r, a, sizeof(float) * 2 * (size_t)n);
    }
    free(wr); free(wi); free(a); free(b);
    return 0;
}

/* ------------------------------------------------------------------ */
/* Radix-4 stages (M5)                                                 */
/* ------------------------------------------------------------------ */

/* Twiddle pair for exponent e <= 3N/4: entries above N/2 fold through
 * W[N-e] = conj(W[e]).  Reference: src/xpu/kernels.py:287-296. */
static void tw_fold(const float* wr, const float* wi, int64_t e, int64_t N, float* r, float* i) {
    if (e > N / 2) {
        *r = wr[N - e];
        *i = wi[N - e] * -1.0f;
    } else {
        *r = wr[e];
        *i = wi[e];
    }
}

/* One radix-4 DIT stage (span 4n).  Reference: src/xpu/kernels.py:239-334
 * (dit_stage4_kernel) and :633-720 (dit_stage4_batch_kernel). */
static void dit_stage4_row(const float* X, float* Y, int64_t n, int64_t M, int64_t N, int bits,
                           int digrev_in, const float* wr, const float* wi) {
    for (int64_t k = 0; k < N / 4; ++k) {
        int64_t j = k % n;
        int64_t i = ((k / n) * 4) * n + j;
        int64_t s[4];
        for (int d = 0; d < 4; ++d)
            s[d] = digrev_in ? bfo_dit_digit_reverse((uint32_t)(i + d * n), bits) : i + d * n;
        float ar = X[2 * s[0]], ai = X[2 * s[0] + 1];
        float br = X[2 * s[1]], bi = X[2 * s[1] + 1];
        float cr = X[2 * s[2]], ci = X[2 * s[2] + 1];
        float dr = X[2 * s[3]], di = X[2 * s[3] + 1];
        int64_t jm = j * M, w2 = jm << 1, w3 = jm + w2;
        float w1r = wr[jm], w1i = wi[jm], w2r = wr[w2], w2i = wi[w2], w3r, w3i;
        tw_fold(wr, wi, w3, N, &w3r, &w3i);
        float b1r = br * w1r - bi * w1i, b1i = br * w1i + bi * w1r;
        float b2r = cr * w2r - ci * w2i, b2i = cr * w2i + ci * w2r;
        float b3r = dr * w3r - di * w3i, b3i = dr * w3i + di * w3r;
        float y0r = ar + b1r + b2r + b3r, y0i = ai + b1i + b2i + b3i;
        float y1r = ar + b1i - b2r - b3i, y1i = ai - b1r - b2i + b3r;
        float y2r = ar - b1r + b2r - b3r, y2i = ai - b1i + b2i - b3i;
        float y3r = ar - b1i - b2r + b3i, y3i = ai + b1r - b2i - b3r;
        Y[2 * i] = y0r; Y[2 * i + 1] = y0i;
        Y[2 * (i + n)] = y1r; Y[2 * (i + n) + 1] = y1i;
        Y[2 * (i + 2 * n)] = y2r; Y[2 * (i + 2 * n) + 1] = y2i;
        Y[2 * (i + 3 * n)] = y3r; Y[2 * (i + 3 * n) + 1] = y3i;
    }
}

/* One radix-4 DIF stage (span 4n).  Reference: src/xpu/kernels.py:337-423
 * (dif_stage4_kernel) and :723-809 (dif_stage4_batch_kernel). */
static void dif_stage4_row(const float* X, float* Y, int64_t n, int64_t M, int64_t N, int bits,
                           int digrev_out, const float* wr, const float* wi) {
    for (int64_t k = 0; k < N / 4; ++k) {
        int64_t j = k % n;
        int64_t i = ((k / n) * 4) * n + j;
        float ar = X[2 * i], ai = X[2 * i + 1];
        float br = X[2 * (i + n)], bi = X[2 * (i + n) + 1];
        float cr = X[2 * (i + 2 * n)], ci = X[2 * (i + 2 * n) + 1];
        float dr = X[2 * (i + 3 * n)], di = X[2 * (i + 3 * n) + 1];
        float y0r = ar + br + cr + dr, y0i = ai + bi + ci + di;
        float y1r = ar + bi - cr - di, y1i = ai - br - ci + dr;
        float y2r = ar - br + cr - dr, y2i = ai - bi + ci - di;
        float y3r = ar - bi - cr + di, y3i = ai + br - ci - dr;
        int64_t jm = j * M, w2 = jm << 1, w3 = jm + w2;
        float w1r = wr[jm], w1i = wi[jm], w2r = wr[w2], w2i = wi[w2], w3r, w3i;
        tw_fold(wr, wi, w3, N, &w3r, &w3i);
        float t1r = y1r * w1r - y1i * w1i, t1i = y1r * w1i + y1i * w1r;
        float t2r = y2r * w2r - y2i * w2i, t2i = y2r * w2i + y2i * w2r;
        float t3r = y3r * w3r - y3i * w3i, t3i = y3r * w3i + y3i * w3r;
        int64_t d[4];
        for (int q = 0; q < 4; ++q)
            d[q] = digrev_out ? bfo_dif_digit_reverse((uint32_t)(i + q * n), bits) : i + q * n;
        Y[2 * d[0]] = y0r; Y[2 * d[0] + 1] = y0i;
        Y[2 * d[1]] = t1r; Y[2 * d[1] + 1] = t1i;
        Y[2 * d[2]] = t2r; Y[2 * d[2] + 1] = t2i;
        Y[2 * d[3]] = t3r; Y[2 * d[3] + 1] = t3i;
    }
}

/* M5 radix-4 FFT of `batch` rows (n >= 4).  Stage sequences:
 * DIT spans 4, 16, ... plus a radix-2 tail spanning N for odd log2 N
 *   (src/xpu/runner.py:1367-1383 _r4_dit_stages, :1399-1469 fft_dit_radix4);
 * DIF groups N, N/4, ... plus a radix-2 group-2 tail storing through the DIF
 *   digit reversal (src/xpu/runner.py:1386-1396 _r4_dif_stages,
 *   :1472-1540 fft_dif_radix4). */
int bfo_fft_radix4_f32(const float* x, float* y, int64_t n, int64_t batch, int dif) {
    if (n < 4 || (n & (n - 1))) return 1;
    int bits = ilog2(n);
    float* wr = (float*)malloc(sizeof(float) * (size_t)(n / 2 + 1));
    float* wi = (float*)malloc(sizeof(float) * (size_t)(n / 2 + 1));
    float* a = (float*)malloc(sizeof(float) * 2 * (size_t)n);
    float* b = (float*)malloc(sizeof(float) * 2 * (size_t)n);
    bfo_twiddle_f32(n, n / 2, wr, wi);
    for (int64_t r = 0; r < batch; ++r) {
        memcpy(a, x + 2 * n * r, sizeof(float) * 2 * (size_t)n);
        if (!dif) {
            int64_t s = 4;
            for (;;) {
                dit_stage4_row(a, b, s >> 2, n / s, n, bits, s == 4, wr, wi);
                { float* t = a; a = b; b = t; }
                if (s == n) break;
                if (4 * s <= n) {
                    s *= 4;
                } else {
                    /* radix-2 tail spanning N: half-span N/2, stride 1 */
                    dit_stage_row(a, b, n >> 1, 1, n, bits, 0, wr, wi);
                    { float* t = a; a = b; b = t; }
                    break;
                }
            }
        } else {
            int64_t s = n;
            int nst = 0;
            int64_t spans[32];
            while (s % 4 == 0 && s >= 4) { spans[nst++] = s; s >>= 2; }
            int tail2 = (s == 2);
            for (int q = 0; q < nst; ++q) {
                int last = (q == nst - 1) && !tail2;
                dif_stage4_row(a, b, spans[q] >> 2, n / spans[q], n, bits, last, wr, wi);
                { float* t = a; a = b; b = t; }
            }
            if (tail2) {
                dif_stage_row(a, b, 1, n >> 1, n, bits, 2, wr, wi);
                { float* t = a; a = b; b = t; }
            }
        }
        memcpy(y + 2 * n * r, a, sizeof(float) * 2 * (size_t)n);
    }
    free(wr); free(wi); free(a); free(b);
    return 0;
}

/* Out-of-place bit-reversal permutation Y[i] = X[bitrev(i)] per row.
 * Reference: src/xpu/kernels.py:81-97 (bitrev_kernel), :536-561
 * (bitrev_batch_kernel), src/xpu/runner.py:1542-1552. */
int bfo_bitrev_permute(const float* x, float* y, int64_t n, int64_t batch) {
    if (n < 1 || (n & (n - 1))) return 1;
    int bits = ilog2(n);
    for (int64_t r = 0; r < batch; ++r)
        for (int64_t i = 0; i < n; ++i) {
            int64_t s = bfo_bit_reverse((uint32_t)i, bits);
            y[2 * (r * n + i)] = x[2 * (r * n + s)];
            y[2 * (r * n + i) + 1] = x[2 * (r * n + s) + 1];
        }
    return 0;
}

/* ------------------------------------------------------------------ */
/* Dedicated real-transform epilogues                                  */
/* ------------------------------------------------------------------ */

/* R2C stitch: from the N/2-point FFT Z of packed pairs, X[k] = a - i*w*c for
 * k in [0, N/2], DC/Nyquist imaginary forced to 0, scale fused.
 * Reference: src/xpu/kernels.py:1127-1177 (r2c_stitch_kernel). */
int bfo_r2c_stitch_f32(const float* z, float* x, int64_t n, int64_t batch, float scale) {
    int64_t np = n / 2, cols = np + 1;
    float* wr = (float*)malloc(sizeof(float) * (size_t)cols);
    float* wi = (float*)malloc(sizeof(float) * (size_t)cols);
    bfo_twiddle_f32(n, cols, wr, wi);
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t k = 0; k < cols; ++k) {
            int64_t jc = (np - k) % np, zk = k % np;
            const float* zb = z + 2 * b * np;
            float zr_k = zb[2 * zk], zi_k = zb[2 * zk + 1];
            float zr_j = zb[2 * jc], zi_j = zb[2 * jc + 1];
            float ar = 0.5f * (zr_k + zr_j), ai = 0.5f * (zi_k - zi_j);
            float cr = 0.5f * (zr_k - zr_j), ci = 0.5f * (zi_k + zi_j);
            float xr = ar + wr[k] * ci + wi[k] * cr;
            float xi = ai - wr[k] * cr + wi[k] * ci;
            float* o = x + 2 * (b * cols + k);
            o[0] = xr * scale;
            o[1] = (k == 0 || k == np) ? 0.0f : xi * scale;
        }
    free(wr); free(wi);
    return 0;
}

/* C2R pre-twiddle: half spectrum -> direct input Z of the N/2-point core,
 * Z[k] = a + i*w*c with w = exp(+2*pi*i*k/N), DC/Nyquist imaginary ignored.
 * Reference: src/xpu/kernels.py:1180-1229 (c2r_pre_kernel). */
int bfo_c2r_pre_f32(const float* xh, float* z, int64_t n, int64_t batch) {
    int64_t np = n / 2, cols = np + 1;
    float* wr = (float*)malloc(sizeof(float) * (size_t)cols);
    float* wi = (float*)malloc(sizeof(float) * (size_t)cols);
    bfo_twiddle_f32(n, cols, wr, wi);
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t k = 0; k < np; ++k) {
            int64_t j = np - k;
            const float* xb = xh + 2 * b * cols;
            float xk_r = xb[2 * k], xk_i = k > 0 ? xb[2 * k + 1] : 0.0f;
            float xj_r = xb[2 * j], xj_i = j < np ? xb[2 * j + 1] : 0.0f;
            float ar = 0.5f * (xk_r + xj_r), ai = 0.5f * (xk_i - xj_i);
            float cr = 0.5f * (xk_r - xj_r), ci = 0.5f * (xk_i + xj_i);
            float w_r = wr[k], w_i = -wi[k];
            float* o = z + 2 * (b * np + k);
            o[0] = ar - (w_r * ci + w_i * cr);
            o[1] = ai + (w_r * cr - w_i * ci);
        }
    free(wr); free(wi);
    return 0;
}

/* C2R unpack: out[2k] = s*Re u[m], out[2k+1] = s*Im u[m], m = (N/2-k) % (N/2).
 * Reference: src/xpu/kernels.py:1232-1258 (c2r_unpack_kernel). */
int bfo_c2r_unpack_f32(const float* u, float* out, int64_t n, int64_t batch, float scale) {
    int64_t np = n / 2;
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t k = 0; k < np; ++k) {
            int64_t m = (np - k) % np;
            const float* ub = u + 2 * b * np;
            out[b * n + 2 * k] = ub[2 * m] * scale;
            out[b * n + 2 * k + 1] = ub[2 * m + 1] * scale;
        }
    return 0;
}

/* ------------------------------------------------------------------ */
/* Float64 path (the reference's native C++ CPU FFT)                    */
/* ------------------------------------------------------------------ */

/* Radix-2 FFT in double with an exact-angle twiddle table, DIT with an explicit
 * bit-reversal first or DIF with the reversal last.  Reference:
 * include/butterfly/fft.hpp:28-97, include/butterfly/twiddle.hpp:18-36.
 * sign = -1 forward, +1 unnormalised inverse. */
int bfo_fft_f64(const double* x, double* y, int64_t n, int64_t batch, int dif, int sign) {
    if (n < 1 || (n & (n - 1))) return 1;
    int bits = ilog2(n);
    double* wr = (double*)malloc(sizeof(double) * (size_t)(n / 2 + 1));
    double* wi = (double*)malloc(sizeof(double) * (size_t)(n / 2 + 1));
    double* a = (double*)malloc(sizeof(double) * 2 * (size_t)n);
    for (int64_t idx = 0; idx < n / 2; ++idx) {
        double ang = (double)sign * 2.0 * M_PI * (double)idx / (double)n;
        wr[idx] = cos(ang);
        wi[idx] = sin(ang);
    }
    for (int64_t r = 0; r < batch; ++r) {
        const double* src = x + 2 * n * r;
        if (!dif) {
            for (int64_t i = 0; i < n; ++i) {
                int64_t s = bfo_bit_reverse((uint32_t)i, bits);
                a[2 * s] = src[2 * i];
                a[2 * s + 1] = src[2 * i + 1];
            }
            for (int64_t sn = 1; sn < n; sn *= 2) {
                int64_t M = n / (2 * sn);
                for (int64_t k = 0; k < n / 2; ++k) {
                    int64_t j = k % sn, i = (k / sn) * 2 * sn + j, w = j * M;
                    double xr = a[2 * i], xi = a[2 * i + 1];
                    double br = a[2 * (i + sn)], bi = a[2 * (i + sn) + 1];
                    double yr = br * wr[w] - bi * wi[w], yi = br * wi[w] + bi * wr[w];
                    a[2 * i] = xr + yr; a[2 * i + 1] = xi + yi;
                    a[2 * (i + sn)] = xr - yr; a[2 * (i + sn) + 1] = xi - yi;
                }
            }
            memcpy(y + 2 * n * r, a, sizeof(double) * 2 * (size_t)n);
        } else {
            memcpy(a, src, sizeof(double) * 2 * (size_t)n);
            for (int64_t sn = n / 2; sn >= 1; sn /= 2) {
                int64_t M = n / (2 * sn);
                for (int64_t k = 0; k < n / 2; ++k) {
                    int64_t j = k % sn, i = (k / sn) * 2 * sn + j, w = j * M;
                    double xr = a[2 * i], xi = a[2 * i + 1];
                    double br = a[2 * (i + sn)], bi = a[2 * (i + sn) + 1];
                    double dr = xr - br, di = xi - bi;
                    a[2 * i] = xr + br; a[2 * i + 1] = xi + bi;
                    a[2 * (i + sn)] = dr * wr[w] - di * wi[w];
                    a[2 * (i + sn) + 1] = dr * wi[w] + di * wr[w];
                }
            }
            double* o = y + 2 * n * r;
            for (int64_t i = 0; i < n; ++i) {
                int64_t s = bfo_bit_reverse((uint32_t)i, bits);
                o[2 * s] = a[2 * i];
                o[2 * s + 1] = a[2 * i + 1];
            }
        }
    }
    free(wr); free(wi); free(a);
    return 0;
}
