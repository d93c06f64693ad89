// bfft_dist.cu -- device phases of the distributed 4-step C2C FFT.
//
// One 1-D transform of N = N1 * N2 points is spread over P ranks as
// contiguous slabs: rank r holds x[r N/P, (r+1) N/P), i.e. rows
// n1 in [r M1, (r+1) M1) of the row-major N1 x N2 view (M1 = N1/P,
// M2 = N2/P).  The transform is the 4-step decomposition the reference's
// hybrid adapter applies on one device (src/xpu/adapter_hybrid.py:224-270:
// stride gather, length-N1 sub-FFTs, twiddle W_N^{n2 k1}, length-N2
// sub-FFTs, digit-reversal transpose), with each transpose that crosses
// ranks done as an all-to-all between the phases below:
//
//   phase 0: x_r[i][n2]            -> send[s][n2'][i]     transpose (conj for inverse)
//   --- all-to-all 1: recv[p][n2'][i], n1 = p M1 + i, n2 = r M2 + n2'
//   phase 1: chunk permute -> [n2'][n1]; length-N1 row FFTs -> [n2'][k1];
//            transpose x W_N^{n2 k1} -> send[t][k1'][n2']
//   --- all-to-all 2: recv[s][k1'][n2'], k1 = r M1 + k1', n2 = s M2 + n2'
//   phase 2: chunk permute -> [k1'][n2]; length-N2 row FFTs -> [k1'][k2];
//            transpose -> send[u][k2'][k1']
//   --- all-to-all 3: recv[s][k2'][k1'], k2 = r M2 + k2', k1 = s M1 + k1'
//   phase 3: chunk permute -> out[k2'][k1] (conj and norm scale), which is
//            X[k2 N1 + k1] for the rank's output slab k2 in [r M2, (r+1) M2)
//
// Transposed-output mode replaces phase 2, all-to-all 3 and phase 3 by
//   phase 4: chunk permute -> [k1'][n2]; length-N2 row FFTs -> out[k1'][k2]
//            (conj and norm scale), i.e. X[k2 N1 + k1] for k1 = r M1 + k1'
// so the rank ends holding M1 whole columns k1 of the N1 x N2 output view
// instead of a contiguous slab: one exchange and two local passes fewer.
//
// The exchanges themselves are NCCL all-to-alls issued by the host layer
// between these calls (bfft/dist.py); every phase only touches this rank's
// device memory.
#include <cmath>
#include <cstring>
#include <cstdarg>
#include <cstdio>
#include <cstdint>
#include <string>
#include <vector>

#include "../../include/bfft.h"
#include "bfft_kernels.cuh"

using namespace bfft;

namespace {

constexpr int kTT = 32;  // transpose tile edge (complex64 elements)

// out[c][r] = scale * tw(r, c) * (conj?) in[r][c] over a rows x cols
// row-major matrix; tw(r, c) = W_N^{(row0 + r) c} when use_tw.
__global__ void __launch_bounds__(256) k_transpose(const float2* __restrict__ in, float2* __restrict__ out,
                                                   int64_t rows, int64_t cols, int64_t tiles_c, TwoLevel tw,
                                                   int use_tw, uint32_t row0, int conj, float scale) {
    __shared__ float2 t[kTT][kTT + 1];
    const int64_t tile = blockIdx.x;
    const int64_t r0 = (tile / tiles_c) * kTT, c0 = (tile % tiles_c) * kTT;
    const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
    for (int j = ty; j < kTT; j += 8) {
        const int64_t r = r0 + j, c = c0 + tx;
        if (r < rows && c < cols) {
            float2 v = in[r * cols + c];
            if (conj) v.y = -v.y;
            if (use_tw) v = cmul(v, tw_two_level(tw, (row0 + (uint32_t)r) * (uint32_t)c));
            t[j][tx] = v;
        }
    }
    __syncthreads();
#pragma unroll
    for (int j = ty; j < kTT; j += 8) {
        const int64_t c = c0 + j, r = r0 + tx;
        if (r < rows && c < cols) {
            const float2 v = t[tx][j];
            out[c * rows + r] = make_float2(v.x * scale, v.y * scale);
        }
    }
}

// out[b][a][c] = scale * (conj?) in[a][b][c] with A = 2^la, B = 2^lb and
// chunks of 2^lc vector elements V (float4 = two complex64, or float2).
template <typename V>
__global__ void __launch_bounds__(256) k_chunk_permute(const V* __restrict__ in, V* __restrict__ out, int la,
                                                       int lb, int lc, int64_t total, int conj, float scale) {
    const int64_t cmask = ((int64_t)1 << lc) - 1, amask = ((int64_t)1 << la) - 1;
    for (int64_t o = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; o < total;
         o += (int64_t)gridDim.x * blockDim.x) {
        const int64_t c = o & cmask, rest = o >> lc;
        const int64_t a = rest & amask, b = rest >> la;
        V v = in[(((a << lb) + b) << lc) | c];
        if constexpr (sizeof(V) == 16) {
            if (conj) { v.y = -v.y; v.w = -v.w; }
            v.x *= scale; v.y *= scale; v.z *= scale; v.w *= scale;
        } else {
            if (conj) v.y = -v.y;
            v.x *= scale; v.y *= scale;
        }
        out[o] = v;
    }
}

// Transpose fused with the exchange: element (r, c) of the local rows x cols
// matrix goes to rank d = c >> log2_dc, at offset
// (c & (dc - 1)) * dst_ld + dst_off + r of that rank's exchange buffer
// (peers[d], mapped into this process), optionally times W_N^{(row0 + r) c},
// conjugated and scaled.  A 64 x 32 tile is read row-wise (256-byte runs),
// held transposed in shared memory, and written as 16-byte stores, 512-byte
// runs of consecutive r per warp, over NVLink (remote ranks) or locally.
// Persistent: a CTA walks tiles with a grid stride, the next tile's loads
// issued before this tile's stores, and every thread fences at system scope
// once, after its last store, so the host-ordered barrier that follows
// publishes them (a fence per tile halved the kernel's rate).
constexpr int kSR = 64, kSC = 32;  // scatter tile: rows x cols
__global__ void __launch_bounds__(256) k_scatter_transpose(const float2* __restrict__ in, float2* const* peers,
                                                           int64_t rows, int64_t cols, int64_t tiles_c,
                                                           int64_t ntiles, int log2_dc, int64_t dst_ld,
                                                           int64_t dst_off, TwoLevel tw, int use_tw, uint32_t row0,
                                                           int conj, float scale) {
    __shared__ __align__(16) float2 t[kSC][kSR + 2];  // [col][row], rows 16-byte aligned
    const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
    const int64_t dmask = ((int64_t)1 << log2_dc) - 1;
    float2 v[kSR / 8];
    auto load = [&](int64_t tile) {
        const int64_t r0 = (tile / tiles_c) * kSR, c0 = (tile % tiles_c) * kSC;
#pragma unroll
        for (int j = 0; j < kSR / 8; ++j) {
            const int64_t r = r0 + ty + 8 * j, c = c0 + tx;
            v[j] = (r < rows && c < cols) ? in[r * cols + c] : make_float2(0.f, 0.f);
        }
    };
    int64_t tile = blockIdx.x;
    if (tile < ntiles) load(tile);
    for (; tile < ntiles; tile += gridDim.x) {
        const int64_t r0 = (tile / tiles_c) * kSR, c0 = (tile % tiles_c) * kSC;
#pragma unroll
        for (int j = 0; j < kSR / 8; ++j) {
            const int rl = ty + 8 * j;
            float2 w = v[j];
            if (conj) w.y = -w.y;
            if (use_tw) w = cmul(w, tw_two_level(tw, (row0 + (uint32_t)(r0 + rl)) * (uint32_t)(c0 + tx)));
            t[tx][rl] = make_float2(w.x * scale, w.y * scale);
        }
        __syncthreads();
        if (tile + gridDim.x < ntiles) load(tile + gridDim.x);  // in flight during the stores
#pragma unroll
        for (int j = 0; j < kSC / 8; ++j) {
            const int cl = ty + 8 * j;
            const int64_t c = c0 + cl, r = r0 + 2 * tx;
            if (c >= cols || r >= rows) continue;
            float2* dst = peers[c >> log2_dc] + (c & dmask) * dst_ld + dst_off + r;
            if (r + 1 < rows && !(reinterpret_cast<uintptr_t>(dst) & 15)) {
                *reinterpret_cast<float4*>(dst) = *reinterpret_cast<const float4*>(&t[cl][2 * tx]);
            } else {
                dst[0] = t[cl][2 * tx];
                if (r + 1 < rows) dst[1] = t[cl][2 * tx + 1];
            }
        }
        __syncthreads();  // the tile buffer is rewritten by the next iteration
    }
    __threadfence_system();
}


cudaError_t launch_transpose(const float2* in, float2* out, int64_t rows, int64_t cols, const TwoLevel& tw,
                             int use_tw, uint32_t row0, int conj, float scale, cudaStream_t s) {
    const int64_t tr = (rows + kTT - 1) / kTT, tc = (cols + kTT - 1) / kTT;
    k_transpose<<<(unsigned)(tr * tc), dim3(kTT, 8), 0, s>>>(in, out, rows, cols, tc, tw, use_tw, row0, conj, scale);
    count_launches(1);
    return cudaGetLastError();
}

int ilog2(int64_t v) {
    int b = 0;
    while (((int64_t)1 << b) < v) ++b;
    return b;
}

cudaError_t launch_scatter(const float2* in, float2* const* peers, int64_t rows, int64_t cols, int64_t dc,
                           int64_t dst_ld, int64_t dst_off, const TwoLevel& tw, int use_tw, uint32_t row0, int conj,
                           float scale, cudaStream_t s) {
    const int64_t tr = (rows + kSR - 1) / kSR, tc = (cols + kSC - 1) / kSC, ntiles = tr * tc;
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = device_sm_count(dev, &sms);
    if (e != cudaSuccess) return e;
    // 8 CTAs of 256 threads fill an SM (warp limit); a few tiles per CTA
    int64_t grid = (int64_t)sms * 8;
    if (grid > ntiles) grid = ntiles;
    k_scatter_transpose<<<(unsigned)grid, dim3(32, 8), 0, s>>>(in, peers, rows, cols, tc, ntiles, ilog2(dc), dst_ld,
                                                               dst_off, tw, use_tw, row0, conj, scale);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_chunk_permute(const float2* in, float2* out, int64_t A, int64_t B, int64_t C, int conj,
                                 float scale, cudaStream_t s) {
    int dev = 0, sms = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e == cudaSuccess) e = device_sm_count(dev, &sms);
    if (e != cudaSuccess) return e;
    const int64_t total_c = A * B * C;
    const int blocks_cap = sms * 8;
    if (C % 2 == 0) {
        const int64_t total = total_c / 2;
        int64_t grid = (total + 255) / 256;
        if (grid > blocks_cap) grid = blocks_cap;
        k_chunk_permute<float4><<<(unsigned)grid, 256, 0, s>>>(reinterpret_cast<const float4*>(in),
                                                               reinterpret_cast<float4*>(out), ilog2(A), ilog2(B),
                                                               ilog2(C) - 1, total, conj, scale);
    } else {
        int64_t grid = (total_c + 255) / 256;
        if (grid > blocks_cap) grid = blocks_cap;
        k_chunk_permute<float2><<<(unsigned)grid, 256, 0, s>>>(in, out, ilog2(A), ilog2(B), ilog2(C), total_c, conj,
                                                               scale);
    }
    count_launches(1);
    return cudaGetLastError();
}

bfft_status dfail(bfft_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    set_last_error(buf);
    return st;
}

bfft_status dcuda(cudaError_t e, const char* what) {
    return dfail(BFFT_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool pow2(int64_t v) { return v > 0 && (v & (v - 1)) == 0; }

struct DevGuard {
    int prev = -1;
    bool ok = true;
    explicit DevGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~DevGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

struct bfft_dist_plan_s {
    int64_t n = 0, n1 = 0, n2 = 0, m1 = 0, m2 = 0;
    int32_t nranks = 1, rank = 0, tdir = BFFT_FORWARD, norm = BFFT_NORM_BACKWARD, device = 0;
    float2* twmem = nullptr;
    TwoLevel tw{};
    bfft_plan_t row1 = nullptr, row2 = nullptr;
    size_t row_ws = 0;
    float scale = 1.0f;
    // peer-to-peer mode: this rank's two exchange buffers (X1 [M2][N1] and
    // X2 [M1][N2]), every rank's buffers as mapped here, and the device tables
    float2* xbuf = nullptr;
    std::vector<void*> opened;     // peer allocations opened through CUDA IPC (closed on destroy)
    float2** d_peers_x1 = nullptr;  // nranks entries
    float2** d_peers_x2 = nullptr;
    bool attached = false;
};

namespace {

bfft_status make_row_plan(int64_t n, int64_t batch, int32_t tile, int32_t device, bfft_plan_t* out) {
    bfft_plan_desc d{};
    d.runner = BFFT_RUN_FFT_DIT_MATRIX_BATCH;
    d.direction = BFFT_DIT;
    d.n = n;
    d.batch = batch;
    d.transform_type = BFFT_C2C;
    d.transform_direction = BFFT_FORWARD;
    d.norm = BFFT_NORM_NONE;
    d.real_flow = BFFT_REAL_DEDICATED;
    d.block = 256;
    if (tile > 0) {
        d.tile = tile;
    } else {
        // Whole rows on chip up to 2^12 points (one CTA); 2^13..2^16 with a
        // batch: tile = N, the fused single-pass kernel (one HBM round trip);
        // else a 256-point local group and tail passes of <= 2^9 points,
        // every pass on the TMA-staged kernels.
        const int l = ilog2(n);
        d.tile = (l <= kMaxPassLog2 || (l <= 16 && batch >= 2)) ? (int32_t)n : 256;
    }
    d.rows = 1;
    d.glog = 4;
    d.maxp = 4096;
    d.cells = 1;
    d.variant = BFFT_SPREAD;
    d.device = device;
    return bfft_plan_create(&d, out);
}

// The transposed-output phase ends with the row FFTs; conjugation (inverse)
// and a norm scale other than 1 take one more elementwise pass.
bool dist_epilogue(const bfft_dist_plan_s* p) { return p->tdir == BFFT_INVERSE || p->scale != 1.0f; }

}  // namespace

extern "C" {

bfft_status bfft_dist_batch_shard(int64_t batch, int32_t nranks, int32_t rank, int64_t* first, int64_t* count) {
    if (!first || !count) return dfail(BFFT_ERR_VALUE, "NULL output pointer");
    if (batch < 0) return dfail(BFFT_ERR_SHAPE, "batch must be >= 0, got %lld", (long long)batch);
    if (nranks < 1) return dfail(BFFT_ERR_VALUE, "nranks must be >= 1, got %d", nranks);
    if (rank < 0 || rank >= nranks) return dfail(BFFT_ERR_VALUE, "rank %d outside [0, %d)", rank, nranks);
    const int64_t base = batch / nranks, extra = batch % nranks;
    *count = base + (rank < extra ? 1 : 0);
    *first = rank * base + (rank < extra ? rank : extra);
    return BFFT_OK;
}

bfft_status bfft_dist_plan_create(int64_t n1, int64_t n2, int32_t nranks, int32_t rank,
                                  int32_t transform_direction, int32_t norm, int32_t row_tile1,
                                  int32_t row_tile2, int32_t device, bfft_dist_plan_t* plan) {
    if (!plan) return dfail(BFFT_ERR_VALUE, "plan output pointer is NULL");
    *plan = nullptr;
    if (!pow2(n1) || !pow2(n2) || n1 < 2 || n2 < 2)
        return dfail(BFFT_ERR_SHAPE, "factors must be powers of two >= 2, got n1=%lld n2=%lld", (long long)n1,
                     (long long)n2);
    const int64_t n = n1 * n2;
    if (ilog2(n) > 32) return dfail(BFFT_ERR_SHAPE, "N=%lld exceeds 2^32", (long long)n);
    if (nranks < 1 || !pow2(nranks)) return dfail(BFFT_ERR_VALUE, "nranks must be a power of two >= 1, got %d", nranks);
    if (rank < 0 || rank >= nranks) return dfail(BFFT_ERR_VALUE, "rank %d outside [0, %d)", rank, nranks);
    if (n1 % nranks || n2 % nranks)
        return dfail(BFFT_ERR_SHAPE, "nranks=%d must divide both factors n1=%lld and n2=%lld", nranks,
                     (long long)n1, (long long)n2);
    if (transform_direction != BFFT_FORWARD && transform_direction != BFFT_INVERSE)
        return dfail(BFFT_ERR_VALUE, "transform_direction must be 0 (forward) or 1 (inverse), got %d",
                     transform_direction);
    if (norm < BFFT_NORM_NONE || norm > BFFT_NORM_ORTHO) return dfail(BFFT_ERR_VALUE, "bad norm %d", norm);
    DevGuard g(device);
    if (!g.ok) return dfail(BFFT_ERR_CUDA, "cannot select device %d", device);

    auto* p = new bfft_dist_plan_s;
    p->n = n;
    p->n1 = n1;
    p->n2 = n2;
    p->m1 = n1 / nranks;
    p->m2 = n2 / nranks;
    p->nranks = nranks;
    p->rank = rank;
    p->tdir = transform_direction;
    p->norm = norm;
    p->device = device;
    double sc = 1.0;
    if (norm == BFFT_NORM_ORTHO) sc = 1.0 / std::sqrt((double)n);
    else if ((norm == BFFT_NORM_FORWARD && transform_direction == BFFT_FORWARD) ||
             (norm == BFFT_NORM_BACKWARD && transform_direction == BFFT_INVERSE))
        sc = 1.0 / (double)n;
    p->scale = (float)sc;

    const int log2n = ilog2(n);
    const int lo_bits = (log2n + 1) / 2;
    const int64_t nlo = (int64_t)1 << lo_bits, nhi = (int64_t)1 << (log2n - lo_bits);
    cudaError_t e = cudaMalloc(&p->twmem, sizeof(float2) * (size_t)(nlo + nhi));
    if (e == cudaSuccess) e = fill_two_level(p->twmem, p->twmem + nlo, lo_bits, log2n, 0);
    if (e == cudaSuccess) e = cudaStreamSynchronize(0);
    if (e != cudaSuccess) {
        bfft_dist_plan_destroy(p);
        return dcuda(e, "twiddle table");
    }
    p->tw.lo = p->twmem;
    p->tw.hi = p->twmem + nlo;
    p->tw.lo_bits = lo_bits;
    p->tw.log2n = log2n;

    bfft_status st = make_row_plan(n1, p->m2, row_tile1, device, &p->row1);
    if (st == BFFT_OK) st = make_row_plan(n2, p->m1, row_tile2, device, &p->row2);
    if (st != BFFT_OK) {
        std::string msg = bfft_last_error();
        bfft_dist_plan_destroy(p);
        return dfail(st, "row plan: %s", msg.c_str());
    }
    size_t w1 = 0, w2 = 0;
    bfft_plan_workspace_size(p->row1, &w1);
    bfft_plan_workspace_size(p->row2, &w2);
    p->row_ws = w1 > w2 ? w1 : w2;
    *plan = p;
    return BFFT_OK;
}

bfft_status bfft_dist_workspace_size(bfft_dist_plan_t plan, size_t* bytes) {
    if (!plan || !bytes) return dfail(BFFT_ERR_VALUE, "NULL plan or output pointer");
    const size_t slab = sizeof(float2) * (size_t)(plan->n / plan->nranks);
    *bytes = slab + ((plan->row_ws + 255) / 256) * 256;
    return BFFT_OK;
}

bfft_status bfft_dist_phase(bfft_dist_plan_t plan, int32_t phase, const void* in, void* out, void* workspace,
                            size_t workspace_bytes, void* stream) {
    if (!plan) return dfail(BFFT_ERR_VALUE, "NULL plan");
    if (phase < 0 || phase > 4) return dfail(BFFT_ERR_VALUE, "phase must be 0..4, got %d", phase);
    if (!in || !out) return dfail(BFFT_ERR_VALUE, "NULL data pointer");
    if (in == out) return dfail(BFFT_ERR_VALUE, "in and out must not alias");
    if (((uintptr_t)in | (uintptr_t)out | (uintptr_t)workspace) & 15)
        return dfail(BFFT_ERR_VALUE, "buffers must be 16-byte aligned");
    size_t need = 0;
    bfft_dist_workspace_size(plan, &need);
    if ((phase == 1 || phase == 2 || phase == 4) && (!workspace || workspace_bytes < need))
        return dfail(BFFT_ERR_WORKSPACE, "phase %d needs %zu workspace bytes, got %zu", phase, need,
                     workspace ? workspace_bytes : (size_t)0);
    DevGuard g(plan->device);
    if (!g.ok) return dfail(BFFT_ERR_CUDA, "cannot select device %d", plan->device);
    cudaStream_t s = (cudaStream_t)stream;
    const float2* x = (const float2*)in;
    float2* y = (float2*)out;
    const int64_t P = plan->nranks, m1 = plan->m1, m2 = plan->m2, n1 = plan->n1, n2 = plan->n2;
    const int inv = plan->tdir == BFFT_INVERSE;
    float2* a = (float2*)workspace;
    const size_t slab_bytes = sizeof(float2) * (size_t)(plan->n / P);
    void* row_ws = workspace ? (char*)workspace + slab_bytes : nullptr;
    const size_t row_ws_bytes = workspace_bytes > slab_bytes ? workspace_bytes - slab_bytes : 0;
    cudaError_t e = cudaSuccess;
    bfft_status st = BFFT_OK;
    switch (phase) {
        case 0:  // x_r (M1 x N2) -> (N2 x M1) = send[s][n2'][i]
            e = launch_transpose(x, y, m1, n2, plan->tw, 0, 0, inv, 1.0f, s);
            break;
        case 1: {
            const float2* rows = x;
            if (P > 1) {  // recv[p][n2'][i] -> [n2'][p][i]
                e = launch_chunk_permute(x, y, P, m2, m1, 0, 1.0f, s);
                rows = y;
            }
            if (e == cudaSuccess) st = bfft_execute(plan->row1, rows, a, row_ws, row_ws_bytes, stream);
            if (st == BFFT_OK && e == cudaSuccess)  // [n2'][k1] -> [k1][n2'] x W_N^{n2 k1}
                e = launch_transpose(a, y, m2, n1, plan->tw, 1, (uint32_t)(plan->rank * m2), 0, 1.0f, s);
            break;
        }
        case 2: {
            const float2* rows = x;
            if (P > 1) {  // recv[s][k1'][n2'] -> [k1'][s][n2']
                e = launch_chunk_permute(x, y, P, m1, m2, 0, 1.0f, s);
                rows = y;
            }
            if (e == cudaSuccess) st = bfft_execute(plan->row2, rows, a, row_ws, row_ws_bytes, stream);
            if (st == BFFT_OK && e == cudaSuccess)  // [k1'][k2] -> [k2][k1']
                e = launch_transpose(a, y, m1, n2, plan->tw, 0, 0, 0, 1.0f, s);
            break;
        }
        case 3:  // recv[s][k2'][k1'] -> out[k2'][s][k1'], conj / norm epilogue
            e = launch_chunk_permute(x, y, P, m2, m1, inv, plan->scale, s);
            break;
        case 4: {  // transposed output: recv[s][k1'][n2'] -> [k1'][n2] -> out[k1'][k2], conj / norm
            const float2* rows = x;
            if (P > 1) {
                e = launch_chunk_permute(x, a, P, m1, m2, 0, 1.0f, s);
                rows = a;
            }
            if (e == cudaSuccess) st = bfft_execute(plan->row2, rows, y, row_ws, row_ws_bytes, stream);
            if (st == BFFT_OK && e == cudaSuccess && dist_epilogue(plan))
                e = launch_scale(y, y, m1 * n2, plan->scale, inv, s);
            break;
        }
    }
    if (st != BFFT_OK) return st;
    if (e != cudaSuccess) return dcuda(e, "distributed phase launch");
    return BFFT_OK;
}

bfft_status bfft_dist_plan_launches(bfft_dist_plan_t plan, int32_t phase, int* launches) {
    if (!plan || !launches) return dfail(BFFT_ERR_VALUE, "NULL plan or output pointer");
    if (phase < 0 || phase > 4) return dfail(BFFT_ERR_VALUE, "phase must be 0..4, got %d", phase);
    int k = 0;
    if (phase == 0 || phase == 3) {
        k = 1;
    } else {
        int r = 0;
        bfft_plan_launches(phase == 1 ? plan->row1 : plan->row2, &r);
        if (phase == 4) k = r + (plan->nranks > 1 ? 1 : 0) + (dist_epilogue(plan) ? 1 : 0);
        else k = r + 1 + (plan->nranks > 1 ? 1 : 0);
    }
    *launches = k;
    return BFFT_OK;
}

bfft_status bfft_dist_plan_destroy(bfft_dist_plan_t plan) {
    if (!plan) return BFFT_OK;
    DevGuard g(plan->device);
    if (plan->row1) bfft_plan_destroy(plan->row1);
    if (plan->row2) bfft_plan_destroy(plan->row2);
    if (plan->twmem) cudaFree(plan->twmem);
    for (void* ptr : plan->opened) cudaIpcCloseMemHandle(ptr);
    if (plan->d_peers_x1) cudaFree(plan->d_peers_x1);
    if (plan->d_peers_x2) cudaFree(plan->d_peers_x2);
    if (plan->xbuf) cudaFree(plan->xbuf);
    delete plan;
    return BFFT_OK;
}

static bfft_status p2p_attach_bases(bfft_dist_plan_t plan, void* const* bases) {
    const size_t slab = (size_t)(plan->n / plan->nranks);
    std::vector<float2*> x1(plan->nranks), x2(plan->nranks);
    for (int p = 0; p < plan->nranks; ++p) {
        if (!bases[p]) return dfail(BFFT_ERR_VALUE, "NULL exchange buffer for rank %d", p);
        x1[p] = static_cast<float2*>(bases[p]);
        x2[p] = x1[p] + slab;
    }
    const size_t tb = sizeof(float2*) * (size_t)plan->nranks;
    cudaError_t e = cudaSuccess;
    if (!plan->d_peers_x1) e = cudaMalloc(&plan->d_peers_x1, tb);
    if (e == cudaSuccess && !plan->d_peers_x2) e = cudaMalloc(&plan->d_peers_x2, tb);
    if (e == cudaSuccess) e = cudaMemcpy(plan->d_peers_x1, x1.data(), tb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(plan->d_peers_x2, x2.data(), tb, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return dcuda(e, "peer tables");
    plan->attached = true;
    return BFFT_OK;
}

bfft_status bfft_dist_p2p_prepare(bfft_dist_plan_t plan, void* exchange_base, void* ipc_handle,
                                  size_t* handle_bytes) {
    if (!plan) return dfail(BFFT_ERR_VALUE, "NULL plan");
    if (handle_bytes) *handle_bytes = sizeof(cudaIpcMemHandle_t);
    DevGuard g(plan->device);
    if (!g.ok) return dfail(BFFT_ERR_CUDA, "cannot select device %d", plan->device);
    if (!plan->xbuf) {
        cudaError_t e = cudaMalloc(&plan->xbuf, sizeof(float2) * 2 * (size_t)(plan->n / plan->nranks));
        if (e != cudaSuccess)
            return e == cudaErrorMemoryAllocation ? dfail(BFFT_ERR_ALLOC, "exchange buffers: out of device memory")
                                                  : dcuda(e, "exchange buffers");
    }
    if (exchange_base) *(void**)exchange_base = plan->xbuf;
    if (ipc_handle) {
        cudaIpcMemHandle_t h;
        cudaError_t e = cudaIpcGetMemHandle(&h, plan->xbuf);
        if (e != cudaSuccess) return dcuda(e, "cudaIpcGetMemHandle");
        memcpy(ipc_handle, &h, sizeof h);
    }
    return BFFT_OK;
}

bfft_status bfft_dist_p2p_attach(bfft_dist_plan_t plan, const void* handles) {
    if (!plan || !handles) return dfail(BFFT_ERR_VALUE, "NULL plan or handles");
    if (!plan->xbuf) return dfail(BFFT_ERR_VALUE, "bfft_dist_p2p_prepare first");
    DevGuard g(plan->device);
    if (!g.ok) return dfail(BFFT_ERR_CUDA, "cannot select device %d", plan->device);
    std::vector<void*> bases(plan->nranks, nullptr);
    const char* hb = static_cast<const char*>(handles);
    for (int p = 0; p < plan->nranks; ++p) {
        if (p == plan->rank) {
            bases[p] = plan->xbuf;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + (size_t)p * sizeof h, sizeof h);
        void* ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) return dcuda(e, "cudaIpcOpenMemHandle");
        plan->opened.push_back(ptr);
        bases[p] = ptr;
    }
    return p2p_attach_bases(plan, bases.data());
}

bfft_status bfft_dist_p2p_attach_pointers(bfft_dist_plan_t plan, void* const* exchange_bases) {
    if (!plan || !exchange_bases) return dfail(BFFT_ERR_VALUE, "NULL plan or pointer table");
    DevGuard g(plan->device);
    if (!g.ok) return dfail(BFFT_ERR_CUDA, "cannot select device %d", plan->device);
    return p2p_attach_bases(plan, exchange_bases);
}

bfft_status bfft_dist_p2p_phase(bfft_dist_plan_t plan, int32_t phase, const void* in, void* out, void* workspace,
                                size_t workspace_bytes, void* stream) {
    if (!plan) return dfail(BFFT_ERR_VALUE, "NULL plan");
    if (!plan->attached) return dfail(BFFT_ERR_VALUE, "peer-to-peer phases need bfft_dist_p2p_attach first");
    if (phase < 0 || phase > 4) return dfail(BFFT_ERR_VALUE, "phase must be 0..4, got %d", phase);
    if ((phase == 0 && !in) || ((phase == 3 || phase == 4) && !out))
        return dfail(BFFT_ERR_VALUE, "NULL data pointer");
    if (((uintptr_t)in | (uintptr_t)out | (uintptr_t)workspace) & 15)
        return dfail(BFFT_ERR_VALUE, "buffers must be 16-byte aligned");
    size_t need = 0;
    bfft_dist_workspace_size(plan, &need);
    if ((phase == 1 || phase == 2 || phase == 4) && (!workspace || workspace_bytes < need))
        return dfail(BFFT_ERR_WORKSPACE, "phase %d needs %zu workspace bytes, got %zu", phase, need,
                     workspace ? workspace_bytes : (size_t)0);
    DevGuard g(plan->device);
    if (!g.ok) return dfail(BFFT_ERR_CUDA, "cannot select device %d", plan->device);
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t P = plan->nranks, m1 = plan->m1, m2 = plan->m2, n1 = plan->n1, n2 = plan->n2, r = plan->rank;
    const int inv = plan->tdir == BFFT_INVERSE;
    const size_t slab = (size_t)(plan->n / P);
    float2* x1 = plan->xbuf;  // [M2][N1]: exchange 1 (and 3) lands here
    float2* x2 = plan->xbuf + slab;  // [M1][N2]: exchange 2
    float2* tmp = (float2*)workspace;
    void* row_ws = workspace ? (char*)workspace + sizeof(float2) * slab : nullptr;
    const size_t row_ws_bytes = workspace_bytes > sizeof(float2) * slab ? workspace_bytes - sizeof(float2) * slab : 0;
    cudaError_t e = cudaSuccess;
    bfft_status st = BFFT_OK;
    switch (phase) {
        case 0:  // x_r[i][n2] -> rank n2 / M2: X1[n2 % M2][r M1 + i]
            e = launch_scatter((const float2*)in, plan->d_peers_x1, m1, n2, m2, n1, r * m1, plan->tw, 0, 0, inv, 1.0f, s);
            break;
        case 1:  // rows of X1 -> [n2'][k1] -> rank k1 / M1: X2[k1 % M1][r M2 + n2'] x W_N^{n2 k1}
            st = bfft_execute(plan->row1, x1, tmp, row_ws, row_ws_bytes, stream);
            if (st == BFFT_OK)
                e = launch_scatter(tmp, plan->d_peers_x2, m2, n1, m1, n2, r * m2, plan->tw, 1, (uint32_t)(r * m2), 0,
                                   1.0f, s);
            break;
        case 2:  // rows of X2 -> [k1'][k2] -> rank k2 / M2: X1[k2 % M2][r M1 + k1'], conj / norm
            st = bfft_execute(plan->row2, x2, tmp, row_ws, row_ws_bytes, stream);
            if (st == BFFT_OK)
                e = launch_scatter(tmp, plan->d_peers_x1, m1, n2, m2, n1, r * m1, plan->tw, 0, 0, inv, plan->scale, s);
            break;
        case 3:  // X1 holds X[k2 N1 + k1] for k2 in this rank's slab
            e = cudaMemcpyAsync(out, x1, sizeof(float2) * slab, cudaMemcpyDeviceToDevice, s);
            break;
        case 4:  // transposed output: rows of X2 -> out[k1'][k2], conj / norm
            st = bfft_execute(plan->row2, x2, out, row_ws, row_ws_bytes, stream);
            if (st == BFFT_OK && dist_epilogue(plan))
                e = launch_scale((float2*)out, (float2*)out, m1 * n2, plan->scale, inv, s);
            break;
    }
    if (st != BFFT_OK) return st;
    if (e != cudaSuccess) return dcuda(e, "peer-to-peer phase");
    return BFFT_OK;
}

}  // extern "C"
