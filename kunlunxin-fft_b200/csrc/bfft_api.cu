// bfft_api.cu -- plans, flows and the extern "C" boundary of libbfft.so.
//
// A plan fixes everything the reference decides in plan_fft / the runner
// (src/xpu/entry.py:292-456, src/xpu/runner.py): which runner executes, its
// knobs, the inverse / norm epilogue and the real-transform wrapper.  At
// creation it validates the descriptor, builds the ordered list of kernel
// launches for the runner ("steps") and allocates the plan-owned twiddle
// tables; bfft_execute only enqueues the steps.
#include <cuda_runtime.h>

#include <atomic>
#include <mutex>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/bfft.h"
#include "bfft_kernels.cuh"

using namespace bfft;

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

bfft_status fail(bfft_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return st;
}

bfft_status cuda_fail(cudaError_t e, const char* what) {
    return fail(BFFT_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

struct DeviceGuard {
    int prev = -1;
    bool ok = true;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

bool is_pow2(int64_t v) { return v > 0 && (v & (v - 1)) == 0; }
int ilog2(int64_t v) {
    int b = 0;
    while (((int64_t)1 << b) < v) ++b;
    return b;
}

// norm epilogue scale, torch.fft semantics (src/xpu/entry.py:81-102)
double norm_scale(int64_t n, int tdir, int norm) {
    if (norm == BFFT_NORM_ORTHO) return 1.0 / std::sqrt((double)n);
    if ((norm == BFFT_NORM_FORWARD && tdir == BFFT_FORWARD) ||
        (norm == BFFT_NORM_BACKWARD && tdir == BFFT_INVERSE))
        return 1.0 / (double)n;
    return 1.0;
}

enum StepKind { S_STAGE2, S_STAGE4, S_PASS, S_CLUSTER, S_FUSED };

// A local group of the whole transform (2^13 .. 2^16 points) runs as the fused
// single-pass kernel from this batch on, as the cluster kernel below it.
constexpr int64_t kFusedMinBatch = 2;

struct Step {
    StepKind kind;
    bool dif = false;
    StageArgs st{};
    PassArgs pa{};
    ClusterArgs ca{};
    FusedArgs fa{};
    int log2l = 0, layout = 0, lmap = 0, smap = 0;
    int block = 256;
};

struct TwAlloc {
    float2* mem = nullptr;
    TwoLevel tw{};
};

}  // namespace

struct bfft_plan_s {
    bfft_plan_desc d{};
    int64_t core_n = 0;      // length of the complex core transform
    int64_t full_n = 0;      // the plan's N
    TwAlloc twc, twf;        // W_core and (real flows) W_N
    std::vector<Step> core;  // unnormalised forward core on (batch, core_n)
    size_t ws_bytes = 0;
    size_t aux_offset = 0;   // start of the fused kernel's scratch ring in the workspace
    bool has_aux = false;
    int launches = 0;
};

namespace {

cudaError_t alloc_two_level(int64_t n, TwAlloc& t) {
    int log2n = ilog2(n);
    int lo_bits = (log2n + 1) / 2;
    if (lo_bits < 1) lo_bits = 1;
    int64_t nlo = (int64_t)1 << (lo_bits < log2n ? lo_bits : log2n);
    int64_t nhi = log2n > lo_bits ? ((int64_t)1 << (log2n - lo_bits)) : 1;
    // beyond 2^22 points the two-level table no longer fits in shared
    // memory; a three-level one (3 x 2^ceil(log2 N / 3) entries) does
    const int l3_bits = log2n > 22 ? (log2n + 2) / 3 : 0;
    const int64_t n3 = l3_bits ? (int64_t)3 << l3_bits : 0;
    cudaError_t e = cudaMalloc(&t.mem, sizeof(float2) * (size_t)(nlo + nhi + n3));
    if (e != cudaSuccess) return e;
    t.tw.lo = t.mem;
    t.tw.hi = t.mem + nlo;
    t.tw.lo_bits = lo_bits;
    t.tw.log2n = log2n;
    if (log2n == 0) return cudaMemset(t.mem, 0, sizeof(float2));  // W_1 unused
    e = fill_two_level(t.mem, t.mem + nlo, lo_bits, log2n, 0);
    if (e == cudaSuccess && l3_bits) {
        t.tw.l3 = t.mem + nlo + nhi;
        t.tw.l3_bits = l3_bits;
        e = fill_three_level(t.mem + nlo + nhi, l3_bits, log2n, 0);
    }
    return e;
}

Step stage2(bool dif, int64_t n, int64_t batch, int64_t half, int in_perm, int out_perm,
            int folded, int block, const TwoLevel& tw) {
    Step s;
    s.kind = S_STAGE2;
    s.dif = dif;
    s.block = block;
    s.st.n = n;
    s.st.batch = batch;
    s.st.half = half;
    s.st.M = n / (2 * half);
    s.st.log2n = ilog2(n);
    s.st.in_perm = in_perm;
    s.st.out_perm = out_perm;
    s.st.scale = 1.0f;
    s.st.folded = folded;
    s.st.tw = tw;
    return s;
}

Step stage4(bool dif, int64_t n, int64_t batch, int64_t span, int in_perm, int out_perm,
            int folded, int block, const TwoLevel& tw) {
    Step s = stage2(dif, n, batch, span / 4, in_perm, out_perm, folded, block, tw);
    s.kind = S_STAGE4;
    s.st.M = n / span;
    return s;
}

// A pass step.  `transpose_store` asks for the store to be staged through
// shared memory in the layout opposite to the compute layout.  Rows whose
// tile is one contiguous block are copied cooperatively, and short
// contiguous rows (fewer than 32 threads per sub-FFT) are stored staged too,
// so every global access is coalesced across the warp.
Step pass_step(int log2l, int layout, int transpose_store, const PassArgs& pa) {
    Step s;
    s.kind = S_PASS;
    s.log2l = log2l;
    s.layout = layout;
    s.pa = pa;
    s.pa.scale = 1.0f;
    s.pa.inner_log2 = ilog2(pa.inner);
    const int64_t L = (int64_t)1 << log2l;
    const int64_t tf = L < 16 ? 1 : L / 16;
    s.smap = transpose_store ? (layout ? 1 : 2) : 0;
    if (!layout) {
        // sub-FFT f = o*inner + c starts at f*L  <=>  in_outer = inner*L and
        // (in_inner = L or a single sub-FFT per outer index)
        const bool contiguous_in = pa.in_stride == 1 && !pa.in_elem_bitrev && !pa.in_base_bits &&
                                   pa.in_outer == pa.inner * L && (pa.inner == 1 || pa.in_inner == L);
        s.lmap = contiguous_in ? 1 : 0;
        if (s.smap == 0 && tf < 32 && pa.out_stride == 1 && !pa.out_elem_bitrev) s.smap = 1;
    }
    return s;
}

PassArgs blank_pass(const TwoLevel& tw) {
    PassArgs p{};
    p.scale = 1.0f;
    p.tw = tw;
    p.tw_mul = 1;
    return p;
}

// Local group of the DIT flows (M1 / M2 / M3): the first log2 T DIT stages on
// the bit-reversed array.  Tile t = bitrev(c) of the bit-reversed array holds
// the natural-order T-point DFT of the stride-(N/T) subsequence starting at c,
// so one pass reads x[c + m N/T] and writes block bitrev(c).
Step dit_local(int64_t n, int64_t batch, int log2t, const TwoLevel& tw) {
    const int64_t T = (int64_t)1 << log2t, cols = n / T;
    PassArgs p = blank_pass(tw);
    p.nsub = batch * cols;
    p.inner = cols;
    p.in_outer = n;
    p.in_inner = 1;
    p.in_stride = cols;
    p.out_outer = n;
    p.out_inner = T;
    p.out_stride = 1;
    p.out_base_bits = ilog2(cols);
    const bool col = cols >= 4;
    return pass_step(log2t, col ? 1 : 0, col ? 1 : 0, p);
}

// Local group of the DIF flows plus the output bit reversal: the last
// log2 T DIF stages on tile h followed by the global bit reversal place
// output k of the natural DFT of tile h at k N/T + bitrev(h).  Enumerating
// c' = bitrev(h) makes the strided store coalesced across c'.
Step dif_local(int64_t n, int64_t batch, int log2t, const TwoLevel& tw) {
    const int64_t T = (int64_t)1 << log2t, cols = n / T;
    PassArgs p = blank_pass(tw);
    p.nsub = batch * cols;
    p.inner = cols;
    p.in_outer = n;
    p.in_inner = T;
    p.in_stride = 1;
    p.in_base_bits = ilog2(cols);
    p.out_outer = n;
    p.out_inner = 1;
    p.out_stride = cols;
    return pass_step(log2t, 0, cols >= 4 ? 1 : 0, p);
}

// DIT stages [s0, s0+g) as one pass.  With G = 2^g, S = 2^s0, group (hi, lo)
// combines the S-point DFTs held in the G blocks of super-block hi: element m
// (decimation residue) sits in block bitrev_G(m), is twiddled by W_{GS}^{m lo}
// and a G-point DFT leaves output k2 at hi GS + k2 S + lo.
Step dit_group(int64_t n, int64_t batch, int s0, int g, const TwoLevel& tw) {
    const int64_t S = (int64_t)1 << s0, G = (int64_t)1 << g;
    PassArgs p = blank_pass(tw);
    p.nsub = batch * (n / G);
    p.inner = S;
    p.in_outer = G * S;
    p.in_inner = 1;
    p.in_stride = S;
    p.in_elem_bitrev = 1;
    p.out_outer = G * S;
    p.out_inner = 1;
    p.out_stride = S;
    p.tw_mode = 1;
    p.tw_mul = n / (G * S);
    return pass_step(g, S >= 4 ? 1 : 0, 0, p);
}

// DIF stages [s0, s0+g) (applied top-down) as one pass: the first g stages
// of a GS-point DIF on each super-block -- a G-point DFT over elements
// hi GS + m S + lo, twiddle W_{GS}^{lo k2}, output k2 stored at block
// bitrev_G(k2).
Step dif_group(int64_t n, int64_t batch, int s0, int g, const TwoLevel& tw) {
    Step s = dit_group(n, batch, s0, g, tw);
    s.pa.in_elem_bitrev = 0;
    s.pa.out_elem_bitrev = 1;
    s.pa.tw_mode = 2;
    return s;
}

// Tail passes read and write strided columns; up to 2^9 points they run on
// the TMA-staged column pass (16 sub-FFTs per tile, 128-byte runs), beyond it
// on k_pass with shorter runs, which costs more than an extra pass.
constexpr int kMaxTailPassLog2 = 9;

// Split `count` consecutive stages into the fewest passes of <= kMaxTailPassLog2
// stages, as equal as possible.
std::vector<int> split_stages(int count) {
    std::vector<int> out;
    if (count <= 0) return out;
    int parts = (count + kMaxTailPassLog2 - 1) / kMaxTailPassLog2;
    for (int i = 0; i < parts; ++i) out.push_back(count / parts + (i < count % parts ? 1 : 0));
    return out;
}

// The reference's tail partition (src/xpu/matrices.py:373-405): stages
// tile..N/2 ascending; greedily take the largest group of 2..glog stages
// whose period n0 << g <= maxp, else a single stage.
void tail_groups(int log2t, int log2n, int glog, int64_t maxp,
                 std::vector<std::pair<int, int>>& units /* (s0, g) g=0: single */) {
    int i = log2t;
    while (i < log2n) {
        int take = 0;
        int avail = log2n - i;
        for (int s = (glog < avail ? glog : avail); s > 1; --s) {
            if (((int64_t)1 << (i + s)) <= maxp) {
                take = s;
                break;
            }
        }
        if (take) {
            units.push_back({i, take});
            i += take;
        } else {
            units.push_back({i, 0});
            i += 1;
        }
    }
}

// The run_hybrid flow's passes (4-step N = tile * t2, adapter_hybrid.py:224-270):
// length-t2 FFTs over x[m1 tile + m0] with the twiddle W_N^{k_t m0} fused into
// their store, then length-tile FFTs over each row k_t stored to
// out[k_r t2 + k_t].  A factor of 1 drops its pass.  Returns the number of
// steps written to `out` (0..2); both factors must be <= 2^kMaxPassLog2.
int hybrid_steps(int64_t n, int64_t B, int64_t tile, const TwoLevel& tw, Step out[2]) {
    const int64_t t2 = n / tile;
    const int lt = ilog2(tile), l2 = ilog2(t2);
    int k = 0;
    if (t2 > 1) {
        PassArgs a = blank_pass(tw);
        a.nsub = B * tile;
        a.inner = tile;
        a.in_outer = n;
        a.in_inner = 1;
        a.in_stride = tile;
        a.out_outer = n;
        a.out_inner = 1;
        a.out_stride = tile;
        a.tw_mode = 2;
        a.tw_mul = 1;
        out[k++] = pass_step(l2, tile >= 4 ? 1 : 0, 0, a);
    }
    if (tile > 1) {
        PassArgs b = blank_pass(tw);
        b.nsub = B * t2;
        b.inner = t2;
        b.in_outer = n;
        b.in_inner = tile;
        b.in_stride = 1;
        b.out_outer = n;
        b.out_inner = 1;
        b.out_stride = t2;
        out[k++] = pass_step(lt, 0, t2 >= 4 ? 1 : 0, b);
    }
    return k;
}

bfft_status build_core(bfft_plan_s& P) {
    const bfft_plan_desc& d = P.d;
    const int64_t n = P.core_n, B = d.batch;
    const int log2n = ilog2(n);
    const TwoLevel& tw = P.twc.tw;
    const int block = d.block > 0 ? d.block : 256;
    std::vector<Step>& st = P.core;
    if (n == 1) return BFFT_OK;  // identity core; epilogue handles conj/scale
    const int r = d.runner;
    const bool batch_runner = r == BFFT_RUN_FFT_DIT_BATCH || r == BFFT_RUN_FFT_DIF_BATCH;
    const int folded = (batch_runner && d.variant == BFFT_FOLDED) ? 1 : 0;
    auto tile_log2 = [&](int64_t tile, int64_t def) {
        int64_t t = tile > 0 ? tile : def;
        if (t > n) t = n;
        return ilog2(t);
    };
    switch (r) {
        case BFFT_RUN_FFT_DIT:
        case BFFT_RUN_FFT_DIT_BATCH:
            for (int s = 0; s < log2n; ++s)
                st.push_back(stage2(false, n, B, (int64_t)1 << s, s == 0 ? 1 : 0, 0, folded, block, tw));
            return BFFT_OK;
        case BFFT_RUN_FFT_DIF:
        case BFFT_RUN_FFT_DIF_BATCH:
            for (int s = log2n - 1; s >= 0; --s)
                st.push_back(stage2(true, n, B, (int64_t)1 << s, 0, s == 0 ? 1 : 0, folded, block, tw));
            return BFFT_OK;
        case BFFT_RUN_FFT_DIT_RADIX4:
        case BFFT_RUN_FFT_DIT_RADIX4_BATCH: {
            if (n < 4) return fail(BFFT_ERR_SHAPE, "radix-4 requires N >= 4, got N=%lld", (long long)n);
            int64_t s = 4;
            for (;;) {
                st.push_back(stage4(false, n, B, s, s == 4 ? 2 : 0, 0, 0, block, tw));
                if (s == n) break;
                if (4 * s <= n) {
                    s *= 4;
                } else {
                    st.push_back(stage2(false, n, B, n / 2, 0, 0, 0, block, tw));
                    break;
                }
            }
            return BFFT_OK;
        }
        case BFFT_RUN_FFT_DIF_RADIX4:
        case BFFT_RUN_FFT_DIF_RADIX4_BATCH: {
            if (n < 4) return fail(BFFT_ERR_SHAPE, "radix-4 requires N >= 4, got N=%lld", (long long)n);
            std::vector<int64_t> spans;
            int64_t s = n;
            while (s % 4 == 0 && s >= 4) {
                spans.push_back(s);
                s >>= 2;
            }
            const bool tail2 = s == 2;
            for (size_t q = 0; q < spans.size(); ++q) {
                const bool last = q + 1 == spans.size() && !tail2;
                st.push_back(stage4(true, n, B, spans[q], 0, last ? 2 : 0, 0, block, tw));
            }
            if (tail2) st.push_back(stage2(true, n, B, 1, 0, 2, 0, block, tw));
            return BFFT_OK;
        }
        case BFFT_RUN_FFT_DIT_FUSED: {
            if (d.tile <= 1) {  // runner.py:226-227: tile <= 1 is the M0 flow
                for (int s = 0; s < log2n; ++s)
                    st.push_back(stage2(false, n, B, (int64_t)1 << s, s == 0 ? 1 : 0, 0, 0, block, tw));
                return BFFT_OK;
            }
            const int lt = tile_log2(d.tile, 64);
            if (lt > kMaxPassLog2)
                return fail(BFFT_ERR_UNSUPPORTED, "fused tile 2^%d exceeds the CTA-resident limit 2^%d", lt, kMaxPassLog2);
            st.push_back(dit_local(n, B, lt, tw));
            for (int s = lt; s < log2n; ++s)
                st.push_back(stage2(false, n, B, (int64_t)1 << s, 0, 0, 0, block, tw));
            return BFFT_OK;
        }
        case BFFT_RUN_FFT_DIT_MATRIX:
        case BFFT_RUN_FFT_DIT_MATRIX_BATCH:
        case BFFT_RUN_FFT_DIF_MATRIX:
        case BFFT_RUN_FFT_DIF_MATRIX_BATCH: {
            const bool dif = r == BFFT_RUN_FFT_DIF_MATRIX || r == BFFT_RUN_FFT_DIF_MATRIX_BATCH;
            if (d.tile <= 1) {  // runner.py:401-403: tile <= 1 is the M0 / M4 flow
                for (int s = 0; s < log2n; ++s) {
                    int sd = dif ? log2n - 1 - s : s;
                    st.push_back(stage2(dif, n, B, (int64_t)1 << sd, (!dif && sd == 0) ? 1 : 0,
                                        (dif && sd == 0) ? 1 : 0, 0, block, tw));
                }
                return BFFT_OK;
            }
            const int lt = tile_log2(d.tile, 64);
            if (lt > kMaxPassLog2) {
                // A local group of the whole transform beyond one CTA: the
                // cluster kernel holds all N points on chip across its CTAs.
                if (lt == log2n && fused_supported(log2n) && B >= kFusedMinBatch) {
                    Step f;
                    f.kind = S_FUSED;
                    f.log2l = log2n;
                    f.fa.batch = B;
                    f.fa.tw = tw;
                    f.fa.scale = 1.0f;
                    st.push_back(f);
                    return BFFT_OK;
                }
                if (lt == log2n && cluster_supported(log2n)) {
                    Step c;
                    c.kind = S_CLUSTER;
                    c.log2l = log2n;
                    c.ca.batch = B;
                    c.ca.tw = tw;
                    c.ca.scale = 1.0f;
                    st.push_back(c);
                    return BFFT_OK;
                }
                return fail(BFFT_ERR_UNSUPPORTED, "matrix tile 2^%d exceeds the on-chip limit (2^%d per CTA, "
                            "whole transforms of 2^13..2^16 per cluster)", lt, kMaxPassLog2);
            }
            std::vector<int> parts = split_stages(log2n - lt);
            if (!dif) {
                st.push_back(dit_local(n, B, lt, tw));
                int s0 = lt;
                for (int g : parts) {
                    st.push_back(dit_group(n, B, s0, g, tw));
                    s0 += g;
                }
            } else {
                int top = log2n;
                for (int g : parts) {
                    st.push_back(dif_group(n, B, top - g, g, tw));
                    top -= g;
                }
                st.push_back(dif_local(n, B, lt, tw));
            }
            return BFFT_OK;
        }
        case BFFT_RUN_FFT_DIT_GROUPED:
        case BFFT_RUN_FFT_DIF_GROUPED: {
            const bool dif = r == BFFT_RUN_FFT_DIF_GROUPED;
            if (d.glog < 1) return fail(BFFT_ERR_VALUE, "glog must be >= 1, got %d", d.glog);
            if (d.cells < 1) return fail(BFFT_ERR_VALUE, "cells must be >= 1, got %d", d.cells);
            if (d.tile <= 1) {
                for (int s = 0; s < log2n; ++s) {
                    int sd = dif ? log2n - 1 - s : s;
                    st.push_back(stage2(dif, n, B, (int64_t)1 << sd, (!dif && sd == 0) ? 1 : 0,
                                        (dif && sd == 0) ? 1 : 0, 0, block, tw));
                }
                return BFFT_OK;
            }
            const int lt = tile_log2(d.tile, 64);
            if (lt > kMaxPassLog2)
                return fail(BFFT_ERR_UNSUPPORTED, "grouped tile 2^%d exceeds the CTA-resident limit 2^%d", lt, kMaxPassLog2);
            std::vector<std::pair<int, int>> units;
            tail_groups(lt, log2n, d.glog, d.maxp > 0 ? d.maxp : 4096, units);
            for (auto& u : units)
                if (u.second > kMaxPassLog2)
                    return fail(BFFT_ERR_UNSUPPORTED, "group of %d stages exceeds 2^%d points", u.second, kMaxPassLog2);
            if (!dif) {
                st.push_back(dit_local(n, B, lt, tw));
                for (auto& u : units)
                    st.push_back(u.second ? dit_group(n, B, u.first, u.second, tw)
                                          : stage2(false, n, B, (int64_t)1 << u.first, 0, 0, 0, block, tw));
            } else {
                for (auto it = units.rbegin(); it != units.rend(); ++it)
                    st.push_back(it->second ? dif_group(n, B, it->first, it->second, tw)
                                            : stage2(true, n, B, (int64_t)1 << it->first, 0, 0, 0, block, tw));
                st.push_back(dif_local(n, B, lt, tw));
            }
            return BFFT_OK;
        }
        case BFFT_RUN_RUN_HYBRID: {
            int64_t tile = d.tile > 0 ? d.tile : 64;
            if (!is_pow2(tile) || tile > n || n % tile)
                return fail(BFFT_ERR_VALUE, "tile %lld must be a power of two dividing N=%lld", (long long)tile, (long long)n);
            const int64_t t2 = n / tile;
            if (ilog2(tile) > kMaxPassLog2 || ilog2(t2) > kMaxPassLog2)
                return fail(BFFT_ERR_UNSUPPORTED, "4-step factors %lld x %lld exceed the CTA-resident limit 2^%d",
                            (long long)t2, (long long)tile, kMaxPassLog2);
            Step hs[2];
            const int k = hybrid_steps(n, B, tile, tw, hs);
            for (int i = 0; i < k; ++i) st.push_back(hs[i]);
            return BFFT_OK;
        }
        default:
            return fail(BFFT_ERR_VALUE, "unknown runner id %d", r);
    }
}

void set_first_conj(Step& s) {
    if (s.kind == S_PASS) s.pa.conj_in = 1;
    else if (s.kind == S_CLUSTER) s.ca.conj_in = 1;
    else if (s.kind == S_FUSED) s.fa.conj_in = 1;
    else s.st.conj_in = 1;
}
void set_last_epilogue(Step& s, int conj, float scale) {
    if (s.kind == S_PASS) {
        s.pa.conj_out = conj;
        s.pa.scale = scale;
    } else if (s.kind == S_CLUSTER) {
        s.ca.conj_out = conj;
        s.ca.scale = scale;
    } else if (s.kind == S_FUSED) {
        s.fa.conj_out = conj;
        s.fa.scale = scale;
    } else {
        s.st.conj_out = conj;
        s.st.scale = scale;
    }
}

// after_pass: the previous kernel on the stream is a pass of this flow, so a
// TMA pass may be launched as its programmatic dependent.
cudaError_t launch_step(const Step& s, const float2* in, float2* out, cudaStream_t stream, bool after_pass = false,
                        void* aux = nullptr) {
    g_launches.fetch_add(1, std::memory_order_relaxed);
    switch (s.kind) {
        case S_STAGE2: return launch_radix2_stage(s.dif, in, out, s.st, s.block, stream);
        case S_STAGE4: return launch_radix4_stage(s.dif, in, out, s.st, s.block, stream);
        case S_PASS: {
            PassArgs pa = s.pa;
            pa.pdl = after_pass ? 1 : 0;
            return launch_pass(s.log2l, s.layout, s.lmap, s.smap, in, out, pa, stream);
        }
        case S_CLUSTER: return launch_cluster_fft(s.log2l, in, out, s.ca, stream);
        case S_FUSED: {
            // TMA needs 16-byte aligned buffers; otherwise the cluster kernel runs the same transform
            const cudaError_t e = aux ? launch_fused_fft(s.log2l, in, out, aux, s.fa, stream) : cudaErrorNotSupported;
            if (e != cudaErrorNotSupported) return e;
            ClusterArgs c{};
            c.batch = s.fa.batch;
            c.tw = s.fa.tw;
            c.scale = s.fa.scale;
            c.conj_in = s.fa.conj_in;
            c.conj_out = s.fa.conj_out;
            return launch_cluster_fft(s.log2l, in, out, c, stream);
        }
        default: return cudaErrorInvalidValue;
    }
}

// Runs the core steps from `src` into `dst`, ping-ponging through `scratch`;
// neither `src` nor its aliases are ever written.
cudaError_t run_core(const Step* st, size_t L, const float2* src, float2* dst, float2* scratch,
                     cudaStream_t stream, void* aux = nullptr) {
    const float2* cur = src;
    for (size_t i = 0; i < L; ++i) {
        float2* tgt = ((L - 1 - i) % 2 == 0) ? dst : scratch;
        cudaError_t e = launch_step(st[i], cur, tgt, stream, i > 0 && st[i - 1].kind == S_PASS, aux);
        if (e != cudaSuccess) return e;
        cur = tgt;
    }
    return cudaSuccess;
}

}  // namespace

// Shared with the other translation units of the library (bfft_noalloc.cu).
namespace bfft {
void set_last_error(const char* msg) { g_last_error = msg; }
void count_launches(int k) { g_launches.fetch_add((uint64_t)k, std::memory_order_relaxed); }

cudaError_t run_hybrid_flow(const float2* in, float2* out, float2* scratch, int64_t n, int64_t batch,
                            int64_t tile, const TwoLevel& tw, int conj, float scale, cudaStream_t s) {
    Step st[2];
    const int k = hybrid_steps(n, batch, tile, tw, st);
    if (k == 0) {
        g_launches.fetch_add(1, std::memory_order_relaxed);
        return launch_scale(in, out, batch * n, scale, 0, s);
    }
    if (conj) set_first_conj(st[0]);
    set_last_epilogue(st[k - 1], conj, scale);
    return run_core(st, (size_t)k, in, out, scratch, s);
}
}  // namespace bfft

// ================================================================ C ABI

extern "C" {

int bfft_api_version(void) { return BFFT_API_VERSION; }

const char* bfft_last_error(void) { return g_last_error.c_str(); }

uint64_t bfft_launch_counter(void) { return g_launches.load(); }

bfft_status bfft_plan_create(const bfft_plan_desc* desc, bfft_plan_t* plan) {
    if (!desc || !plan) return fail(BFFT_ERR_VALUE, "null descriptor or plan pointer");
    *plan = nullptr;
    const bfft_plan_desc& d = *desc;
    if (d.runner < BFFT_RUN_FFT_DIT || d.runner > BFFT_RUN_RUN_HYBRID)
        return fail(BFFT_ERR_VALUE, "unknown runner id %d", d.runner);
    if (d.direction != BFFT_DIT && d.direction != BFFT_DIF)
        return fail(BFFT_ERR_VALUE, "direction must be dit/dif, got %d", d.direction);
    if (d.transform_type < BFFT_C2C || d.transform_type > BFFT_C2R)
        return fail(BFFT_ERR_VALUE, "bad transform_type %d", d.transform_type);
    if (d.transform_direction != BFFT_FORWARD && d.transform_direction != BFFT_INVERSE)
        return fail(BFFT_ERR_VALUE, "bad transform_direction %d", d.transform_direction);
    if (d.norm < BFFT_NORM_NONE || d.norm > BFFT_NORM_ORTHO) return fail(BFFT_ERR_VALUE, "bad norm %d", d.norm);
    if (d.transform_type == BFFT_R2C && d.transform_direction != BFFT_FORWARD)
        return fail(BFFT_ERR_VALUE, "r2c is a forward transform");
    if (d.transform_type == BFFT_C2R && d.transform_direction != BFFT_INVERSE)
        return fail(BFFT_ERR_VALUE, "c2r is an inverse transform");
    if (!is_pow2(d.n)) return fail(BFFT_ERR_SHAPE, "size must be a positive power of two, got %lld", (long long)d.n);
    if (d.n > ((int64_t)1 << 30)) return fail(BFFT_ERR_SHAPE, "N=%lld exceeds 2^30", (long long)d.n);
    if (d.batch < 1) return fail(BFFT_ERR_SHAPE, "batch must be >= 1, got %lld", (long long)d.batch);
    if (d.block <= 0 || !is_pow2(d.block)) return fail(BFFT_ERR_VALUE, "block must be a positive power of two, got %d", d.block);
    if (d.tile < 0 || (d.tile > 1 && !is_pow2(d.tile))) return fail(BFFT_ERR_VALUE, "tile must be a power of two, got %d", d.tile);
    if (d.rows < 0 || (d.rows > 1 && !is_pow2(d.rows))) return fail(BFFT_ERR_VALUE, "rows must be a power of two, got %d", d.rows);
    if (d.variant != BFFT_SPREAD && d.variant != BFFT_FOLDED)
        return fail(BFFT_ERR_VALUE, "variant must be spread/folded, got %d", d.variant);
    const bool spread_only = d.runner == BFFT_RUN_FFT_DIT_MATRIX_BATCH || d.runner == BFFT_RUN_FFT_DIF_MATRIX_BATCH ||
                             d.runner == BFFT_RUN_FFT_DIT_RADIX4_BATCH || d.runner == BFFT_RUN_FFT_DIF_RADIX4_BATCH;
    if (spread_only && d.variant != BFFT_SPREAD)
        return fail(BFFT_ERR_VALUE, "this runner lowers variant='spread' (Ud=B) only");
    const bool dedicated = d.transform_type != BFFT_C2C && d.real_flow == BFFT_REAL_DEDICATED;
    if (dedicated && d.n < 4) return fail(BFFT_ERR_SHAPE, "dedicated real flow needs N >= 4, got %lld", (long long)d.n);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
        return fail(BFFT_ERR_CUDA, "no CUDA device available");
    if (d.device < 0 || d.device >= ndev) return fail(BFFT_ERR_VALUE, "device %d out of range", d.device);

    bfft_plan_s* P = new bfft_plan_s();
    P->d = d;
    P->full_n = d.n;
    P->core_n = dedicated ? d.n / 2 : d.n;
    DeviceGuard g(d.device);
    if (!g.ok) {
        delete P;
        return fail(BFFT_ERR_CUDA, "cannot select device %d", d.device);
    }
    cudaError_t e = ensure_unit_twiddles(d.device, 0);
    if (e == cudaSuccess) e = alloc_two_level(P->core_n, P->twc);
    if (e == cudaSuccess && d.transform_type != BFFT_C2C) e = alloc_two_level(P->full_n, P->twf);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        if (P->twc.mem) cudaFree(P->twc.mem);
        if (P->twf.mem) cudaFree(P->twf.mem);
        delete P;
        return e == cudaErrorMemoryAllocation ? fail(BFFT_ERR_ALLOC, "twiddle allocation failed")
                                              : cuda_fail(e, "plan setup");
    }
    bfft_status st = build_core(*P);
    if (st != BFFT_OK) {
        std::string msg = g_last_error;
        bfft_plan_destroy(P);
        g_last_error = msg;
        return st;
    }
    const int64_t B = d.batch, n = d.n, c = P->core_n;
    const size_t cbytes = sizeof(float2) * (size_t)(B * c);
    const int L = (int)P->core.size();
    if (d.transform_type == BFFT_C2C) {
        P->ws_bytes = L > 1 ? cbytes : 0;
        P->launches = L == 0 ? 1 : L;
    } else if (dedicated) {
        // r2c: core (in -> F via A) + stitch; c2r: pre (in -> C) + core (C -> out via A,
        // the unpack fused; a one-point core keeps the scale + unpack kernels)
        P->ws_bytes = (d.transform_type == BFFT_R2C ? 2 : 3) * cbytes;
        P->launches = d.transform_type == BFFT_R2C ? (L == 0 ? 1 : L) + 1 : (L == 0 ? 3 : L + 1);
    } else {
        P->ws_bytes = 3 * sizeof(float2) * (size_t)(B * n);
        P->launches = (L == 0 ? 1 : L) + 2;
    }
    for (const Step& stp : P->core)
        if (stp.kind == S_FUSED) P->has_aux = true;
    if (P->has_aux) {  // the fused kernel's L2-resident scratch ring follows the flow's buffers
        P->aux_offset = (P->ws_bytes + 255) & ~(size_t)255;
        P->ws_bytes = P->aux_offset + fused_workspace_bytes(c, B);
    }
    *plan = P;
    return BFFT_OK;
}

bfft_status bfft_plan_workspace_size(bfft_plan_t plan, size_t* bytes) {
    if (!plan || !bytes) return fail(BFFT_ERR_VALUE, "null plan or output pointer");
    *bytes = plan->ws_bytes;
    return BFFT_OK;
}

bfft_status bfft_plan_launches(bfft_plan_t plan, int* launches) {
    if (!plan || !launches) return fail(BFFT_ERR_VALUE, "null plan or output pointer");
    *launches = plan->launches;
    return BFFT_OK;
}

bfft_status bfft_plan_destroy(bfft_plan_t plan) {
    if (!plan) return BFFT_OK;
    {
        DeviceGuard g(plan->d.device);
        if (plan->twc.mem) cudaFree(plan->twc.mem);
        if (plan->twf.mem) cudaFree(plan->twf.mem);
    }
    delete plan;
    return BFFT_OK;
}

bfft_status bfft_execute(bfft_plan_t plan, const void* in, void* out, void* workspace,
                         size_t workspace_bytes, void* stream_) {
    if (!plan) return fail(BFFT_ERR_VALUE, "null plan");
    if (!in || !out) return fail(BFFT_ERR_VALUE, "null input or output pointer");
    if (in == out) return fail(BFFT_ERR_VALUE, "input and output must not alias");
    if (((uintptr_t)in | (uintptr_t)out | (uintptr_t)workspace) & 7u)
        return fail(BFFT_ERR_VALUE, "input, output and workspace must be 8-byte aligned");
    if (plan->ws_bytes && (!workspace || workspace_bytes < plan->ws_bytes))
        return fail(BFFT_ERR_WORKSPACE, "workspace of %zu bytes required, got %zu", plan->ws_bytes,
                    workspace ? workspace_bytes : (size_t)0);
    const bfft_plan_desc& d = plan->d;
    DeviceGuard g(d.device);
    if (!g.ok) return fail(BFFT_ERR_CUDA, "cannot select device %d", d.device);
    cudaStream_t s = (cudaStream_t)stream_;
    const int64_t B = d.batch, n = d.n, c = plan->core_n;
    const bool inverse = d.transform_direction == BFFT_INVERSE;
    cudaError_t e = cudaSuccess;
    std::vector<Step> core = plan->core;  // epilogue flags are per call
    float2* ws = static_cast<float2*>(workspace);
    void* aux = plan->has_aux ? static_cast<void*>(static_cast<unsigned char*>(workspace) + plan->aux_offset) : nullptr;

    if (d.transform_type == BFFT_C2C) {
        const float scale = (float)norm_scale(n, d.transform_direction, d.norm);
        if (core.empty()) {
            g_launches.fetch_add(1, std::memory_order_relaxed);
            e = launch_scale((const float2*)in, (float2*)out, B * n, scale, 0, s);
        } else {
            if (inverse) set_first_conj(core.front());
            set_last_epilogue(core.back(), inverse ? 1 : 0, scale);
            e = run_core(core.data(), core.size(), (const float2*)in, (float2*)out, ws, s, aux);
        }
    } else if (d.real_flow == BFFT_REAL_DEDICATED) {
        float2* F = ws;
        float2* A = ws + B * c;
        if (d.transform_type == BFFT_R2C) {
            // pack: the float32 (B, N) input IS the complex64 (B, N/2) z
            const float scale = (float)norm_scale(n, BFFT_FORWARD, d.norm);
            e = core.empty() ? launch_scale((const float2*)in, F, B * c, 1.0f, 0, s)
                             : run_core(core.data(), core.size(), (const float2*)in, F, A, s, aux);
            if (core.empty()) g_launches.fetch_add(1, std::memory_order_relaxed);
            if (e == cudaSuccess) {
                g_launches.fetch_add(1, std::memory_order_relaxed);
                e = launch_r2c_stitch(F, (float2*)out, n, B, scale, plan->twf.tw, s);
            }
        } else {
            float2* C = ws + 2 * B * c;
            const float scale = (float)(2.0 * norm_scale(n, BFFT_INVERSE, d.norm));
            g_launches.fetch_add(1, std::memory_order_relaxed);
            e = launch_c2r_pre((const float2*)in, C, n, B, plan->twf.tw, s);
            if (e == cudaSuccess && !core.empty()) {
                // The reference's unpack reads the core DFT reversed, u[(N/2 - k) mod N/2]
                // = conj(DFT(conj z))[k]: with the conjugates and the scale fused into
                // the first and last pass, the core writes the real output itself
                // (float32 pairs = complex64 (B, N/2)) and the unpack pass goes away.
                set_first_conj(core.front());
                set_last_epilogue(core.back(), 1, scale);
                e = run_core(core.data(), core.size(), C, (float2*)out, A, s, aux);
            } else if (e == cudaSuccess) {
                g_launches.fetch_add(2, std::memory_order_relaxed);
                e = launch_scale(C, F, B * c, 1.0f, 0, s);
                if (e == cudaSuccess) e = launch_c2r_unpack(F, (float*)out, n, B, scale, s);
            }
        }
    } else {
        float2* C = ws;
        float2* F = ws + B * n;
        float2* A = ws + 2 * B * n;
        if (d.transform_type == BFFT_R2C) {
            const float scale = (float)norm_scale(n, BFFT_FORWARD, d.norm);
            g_launches.fetch_add(1, std::memory_order_relaxed);
            e = launch_real_to_complex((const float*)in, C, B * n, s);
            if (e == cudaSuccess) {
                e = core.empty() ? launch_scale(C, F, B * n, 1.0f, 0, s) : run_core(core.data(), core.size(), C, F, A, s, aux);
                if (core.empty()) g_launches.fetch_add(1, std::memory_order_relaxed);
            }
            if (e == cudaSuccess) {
                g_launches.fetch_add(1, std::memory_order_relaxed);
                e = launch_crop(F, (float2*)out, n, B, scale, s);
            }
        } else {
            const float scale = (float)norm_scale(n, BFFT_INVERSE, d.norm);
            g_launches.fetch_add(1, std::memory_order_relaxed);
            e = launch_hermitian_conj((const float2*)in, C, n, B, s);
            if (e == cudaSuccess) {
                e = core.empty() ? launch_scale(C, F, B * n, 1.0f, 0, s) : run_core(core.data(), core.size(), C, F, A, s, aux);
                if (core.empty()) g_launches.fetch_add(1, std::memory_order_relaxed);
            }
            if (e == cudaSuccess) {
                g_launches.fetch_add(1, std::memory_order_relaxed);
                e = launch_real_part(F, (float*)out, B * n, scale, s);
            }
        }
    }
    if (e != cudaSuccess) return cuda_fail(e, "bfft_execute launch");
    return BFFT_OK;
}

bfft_status bfft_bit_reverse_permute(const void* x, void* y, int64_t n, int64_t batch, int32_t device,
                                     void* stream) {
    if (!x || !y) return fail(BFFT_ERR_VALUE, "null pointer");
    if (x == y) return fail(BFFT_ERR_VALUE, "input and output must not alias");
    if (!is_pow2(n) || n > ((int64_t)1 << 30)) return fail(BFFT_ERR_SHAPE, "size must be a positive power of two, got %lld", (long long)n);
    if (batch < 1) return fail(BFFT_ERR_SHAPE, "batch must be >= 1");
    DeviceGuard g(device);
    if (!g.ok) return fail(BFFT_ERR_CUDA, "cannot select device %d", device);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = launch_bitrev((const float2*)x, (float2*)y, n, batch, 256, (cudaStream_t)stream);
    return e == cudaSuccess ? BFFT_OK : cuda_fail(e, "bit_reverse_permute");
}

static bfft_status real_epilogue_checks(const void* a, const void* b, int64_t n, int64_t batch) {
    if (!a || !b) return fail(BFFT_ERR_VALUE, "null pointer");
    if (a == b) return fail(BFFT_ERR_VALUE, "input and output must not alias");
    if (((uintptr_t)a | (uintptr_t)b) & 7u) return fail(BFFT_ERR_VALUE, "pointers must be 8-byte aligned");
    if (!is_pow2(n)) return fail(BFFT_ERR_SHAPE, "size must be a positive power of two, got %lld", (long long)n);
    if (n < 4) return fail(BFFT_ERR_SHAPE, "dedicated real flow needs N >= 4, got %lld", (long long)n);
    if (batch < 1) return fail(BFFT_ERR_SHAPE, "batch must be >= 1");
    return BFFT_OK;
}

// Two-level W_N tables for the stand-alone epilogues, cached per (device, N).
static std::mutex g_epi_mu;
static std::vector<std::pair<std::pair<int, int64_t>, TwAlloc>> g_epi_tw;

static bfft_status epi_table(int device, int64_t n, TwoLevel* out) {
    std::lock_guard<std::mutex> lk(g_epi_mu);
    for (auto& kv : g_epi_tw)
        if (kv.first.first == device && kv.first.second == n) {
            *out = kv.second.tw;
            return BFFT_OK;
        }
    TwAlloc t;
    cudaError_t e = alloc_two_level(n, t);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "epilogue twiddle table");
    g_epi_tw.push_back({{device, n}, t});
    *out = t.tw;
    return BFFT_OK;
}

bfft_status bfft_r2c_stitch(const void* z, void* x, int64_t n, int64_t batch, float scale, int32_t device,
                            void* stream) {
    bfft_status st = real_epilogue_checks(z, x, n, batch);
    if (st) return st;
    DeviceGuard g(device);
    if (!g.ok) return fail(BFFT_ERR_CUDA, "cannot select device %d", device);
    TwoLevel tw;
    if ((st = epi_table(device, n, &tw))) return st;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = launch_r2c_stitch((const float2*)z, (float2*)x, n, batch, scale, tw, (cudaStream_t)stream);
    return e == cudaSuccess ? BFFT_OK : cuda_fail(e, "r2c_stitch");
}

bfft_status bfft_c2r_pre(const void* xh, void* z, int64_t n, int64_t batch, int32_t device, void* stream) {
    bfft_status st = real_epilogue_checks(xh, z, n, batch);
    if (st) return st;
    DeviceGuard g(device);
    if (!g.ok) return fail(BFFT_ERR_CUDA, "cannot select device %d", device);
    TwoLevel tw;
    if ((st = epi_table(device, n, &tw))) return st;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = launch_c2r_pre((const float2*)xh, (float2*)z, n, batch, tw, (cudaStream_t)stream);
    return e == cudaSuccess ? BFFT_OK : cuda_fail(e, "c2r_pre");
}

bfft_status bfft_c2r_unpack(const void* u, void* out, int64_t n, int64_t batch, float scale, int32_t device,
                            void* stream) {
    bfft_status st = real_epilogue_checks(u, out, n, batch);
    if (st) return st;
    DeviceGuard g(device);
    if (!g.ok) return fail(BFFT_ERR_CUDA, "cannot select device %d", device);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = launch_c2r_unpack((const float2*)u, (float*)out, n, batch, scale, (cudaStream_t)stream);
    return e == cudaSuccess ? BFFT_OK : cuda_fail(e, "c2r_unpack");
}

bfft_status bfft_index_map(int32_t kind, int32_t bits, void* out, int32_t device, void* stream) {
    if (!out) return fail(BFFT_ERR_VALUE, "null pointer");
    if (kind < 0 || kind > 2) return fail(BFFT_ERR_VALUE, "index map kind must be 0, 1 or 2, got %d", kind);
    if (bits < 0 || bits > 30) return fail(BFFT_ERR_VALUE, "bits must be in [0, 30], got %d", bits);
    DeviceGuard g(device);
    if (!g.ok) return fail(BFFT_ERR_CUDA, "cannot select device %d", device);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = launch_index_map(kind, bits, (uint32_t*)out, (cudaStream_t)stream);
    return e == cudaSuccess ? BFFT_OK : cuda_fail(e, "index_map");
}

bfft_status bfft_device_status(int32_t device, uint32_t* status, int32_t clear) {
    if (!status) return fail(BFFT_ERR_VALUE, "null pointer");
    DeviceGuard g(device);
    if (!g.ok) return fail(BFFT_ERR_CUDA, "cannot select device %d", device);
    unsigned v = 0;
    cudaError_t e = read_device_status(&v, clear != 0);
    if (e != cudaSuccess) return cuda_fail(e, "device_status");
    *status = v;
    return BFFT_OK;
}

bfft_status bfft_probe_bounded_waits(int32_t device, void* stream) {
    DeviceGuard g(device);
    if (!g.ok) return fail(BFFT_ERR_CUDA, "cannot select device %d", device);
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = run_wait_probe(s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return cuda_fail(e, "probe_bounded_waits");
    return BFFT_OK;
}

bfft_status bfft_tc_dft16_rows(const void* in, void* out, int64_t rows, int32_t transform_direction, float scale,
                               int32_t device, void* stream) {
    if (!in || !out) return fail(BFFT_ERR_VALUE, "null pointer");
    if (in == out) return fail(BFFT_ERR_VALUE, "input and output must not alias");
    if (((uintptr_t)in | (uintptr_t)out) & 15u) return fail(BFFT_ERR_VALUE, "pointers must be 16-byte aligned");
    if (rows < 1 || rows > 0x7fffffffLL) return fail(BFFT_ERR_SHAPE, "rows must be in [1, 2^31), got %lld", (long long)rows);
    if (transform_direction != BFFT_FORWARD && transform_direction != BFFT_INVERSE)
        return fail(BFFT_ERR_VALUE, "bad transform_direction %d", transform_direction);
    DeviceGuard g(device);
    if (!g.ok) return fail(BFFT_ERR_CUDA, "cannot select device %d", device);
    const int inv = transform_direction == BFFT_INVERSE;
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = launch_tc_dft16_rows((const float2*)in, (float2*)out, rows, scale, inv, inv, (cudaStream_t)stream);
    return e == cudaSuccess ? BFFT_OK : cuda_fail(e, "tc_dft16_rows");
}

bfft_status bfft_twiddle_table(void* w, int64_t n, int64_t count, int32_t device, void* stream) {
    if (!w) return fail(BFFT_ERR_VALUE, "null pointer");
    if (!is_pow2(n)) return fail(BFFT_ERR_SHAPE, "size must be a positive power of two, got %lld", (long long)n);
    if (count < 0) return fail(BFFT_ERR_VALUE, "count must be >= 0");
    if (count == 0) return BFFT_OK;
    DeviceGuard g(device);
    if (!g.ok) return fail(BFFT_ERR_CUDA, "cannot select device %d", device);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    cudaError_t e = launch_twiddle_table((float2*)w, n, count, (cudaStream_t)stream);
    return e == cudaSuccess ? BFFT_OK : cuda_fail(e, "twiddle_table");
}

}  // extern "C"
