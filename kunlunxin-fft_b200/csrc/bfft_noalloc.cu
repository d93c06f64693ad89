// bfft_noalloc.cu -- the 4-step C2C transform without any device allocation.
//
// Some callers cannot allocate device memory while they run: code executing
// inside another framework's memory budget (a pre-sized pool that owns every
// byte of the GPU), real-time or capture-sensitive loops where cudaMalloc /
// cudaFree would synchronise the device, or an FFI host that has no allocator
// bound to the CUDA context at all.  bfft_hybrid_c2c_noalloc serves them: the
// caller passes the input and output buffers, and the one scratch buffer the
// two-pass flow needs lives in a fixed-size device array of this library
// instead of a workspace or a cudaMalloc.
//
// The array is file-scope, so every GPU that loads libbfft.so holds it
// (kNoAllocMaxElems complex64 = 32 MiB, plus a 32 KiB twiddle table) until the
// process exits.  All calls share it and it keeps the last call's contents:
// calls whose executions overlap on the GPU (two streams, or two host
// threads) race on it; serialise them on one stream.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>

#include "../../include/bfft.h"
#include "bfft_kernels.cuh"

using namespace bfft;

namespace {

constexpr int64_t kNoAllocMaxElems = BFFT_NOALLOC_MAX_ELEMS;
constexpr int kNoAllocLoBits = 11;  // two-level W_N table: N <= 2^22 -> at most 2^11 + 2^11 entries

// Intermediate of the two passes: pass 1 writes every element that pass 2
// reads, so nothing in it has to start at zero.
static __device__ __align__(256) float2 g_noalloc_scratch[kNoAllocMaxElems];
// W_N two-level table of the current call (rewritten by every call).
static __device__ __align__(256) float2 g_noalloc_twiddle[2 << kNoAllocLoBits];

struct DeviceSymbols {
    float2* scratch = nullptr;
    float2* twiddle = nullptr;
};

std::mutex g_mu;
DeviceSymbols g_syms[64];

bfft_status fail(bfft_status st, const char* fmt, ...) {
    char buf[384];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    set_last_error(buf);  // reported by bfft_last_error()
    return st;
}

// One-time set-up on `device` (which must be current): the device addresses
// of the file-scope arrays (host code may not use the symbols themselves) and
// the library's unit twiddle tables.
bfft_status setup(int device, DeviceSymbols* out) {
    std::lock_guard<std::mutex> lk(g_mu);
    DeviceSymbols& s = g_syms[device];
    if (!s.scratch) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess)
            return fail(BFFT_ERR_CUDA, "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
        void* q = nullptr;
        e = cudaGetSymbolAddress(&q, g_noalloc_twiddle);
        if (e != cudaSuccess)
            return fail(BFFT_ERR_CUDA, "cudaGetSymbolAddress(twiddle): %s", cudaGetErrorString(e));
        e = ensure_unit_twiddles(device, 0);
        if (e != cudaSuccess)
            return fail(BFFT_ERR_CUDA, "unit twiddle set-up: %s", cudaGetErrorString(e));
        s.scratch = static_cast<float2*>(p);
        s.twiddle = static_cast<float2*>(q);
    }
    *out = s;
    return BFFT_OK;
}

int ilog2_exact(int64_t v) {
    if (v <= 0 || (v & (v - 1))) return -1;
    int b = 0;
    while (((int64_t)1 << b) < v) ++b;
    return b;
}

}  // namespace

extern "C" bfft_status bfft_hybrid_c2c_noalloc(const void* in, void* out, int64_t n, int64_t batch,
                                               int64_t tile, int32_t transform_direction, int32_t norm,
                                               int32_t device, void* stream) {
    if (!in || !out) return fail(BFFT_ERR_VALUE, "null input or output pointer");
    if (in == out) return fail(BFFT_ERR_VALUE, "input and output must not alias");
    if (((uintptr_t)in | (uintptr_t)out) & 7u) return fail(BFFT_ERR_VALUE, "pointers must be 8-byte aligned");
    if (transform_direction != BFFT_FORWARD && transform_direction != BFFT_INVERSE)
        return fail(BFFT_ERR_VALUE, "bad transform_direction %d", transform_direction);
    if (norm < BFFT_NORM_NONE || norm > BFFT_NORM_ORTHO) return fail(BFFT_ERR_VALUE, "bad norm %d", norm);
    const int log2n = ilog2_exact(n), log2t = ilog2_exact(tile);
    if (log2n < 1) return fail(BFFT_ERR_SHAPE, "N must be a power of two >= 2, got %lld", (long long)n);
    if (log2t < 0 || tile > n) return fail(BFFT_ERR_VALUE, "tile %lld must be a power of two dividing N=%lld",
                                           (long long)tile, (long long)n);
    if (batch < 1) return fail(BFFT_ERR_SHAPE, "batch must be >= 1");
    const int64_t t2 = n / tile;
    // Only the two-pass shapes use the scratch array; every shape uses the
    // twiddle array, sized for N <= kNoAllocMaxElems.
    if (n > kNoAllocMaxElems || (tile > 1 && t2 > 1 && batch > kNoAllocMaxElems / n))
        return fail(BFFT_ERR_SHAPE,
                    "batch*N = %lld*%lld exceeds the fixed scratch of %lld complex64 elements "
                    "(32 MiB); use bfft_execute with a caller workspace for larger transforms",
                    (long long)batch, (long long)n, (long long)kNoAllocMaxElems);
    if (log2t > kMaxPassLog2 || log2n - log2t > kMaxPassLog2)
        return fail(BFFT_ERR_UNSUPPORTED, "4-step factors %lld x %lld exceed 4096", (long long)t2, (long long)tile);
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || device < 0 || device >= ndev || device >= 64)
        return fail(BFFT_ERR_VALUE, "device %d out of range", device);

    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != device && cudaSetDevice(device) != cudaSuccess)
        return fail(BFFT_ERR_CUDA, "cannot select device %d", device);
    DeviceSymbols sym;
    bfft_status st = setup(device, &sym);
    cudaStream_t s = (cudaStream_t)stream;
    cudaError_t e = cudaSuccess;
    if (st == BFFT_OK) {
        // the split a plan's own table uses (ceil(log2 N / 2) low bits), so
        // the values are the ones bfft_execute would read
        const int lo_bits = (log2n + 1) / 2;
        const int64_t nlo = (int64_t)1 << (lo_bits < log2n ? lo_bits : log2n);
        TwoLevel tw{sym.twiddle, sym.twiddle + nlo, lo_bits, log2n};
        e = fill_two_level(sym.twiddle, sym.twiddle + nlo, lo_bits, log2n, s);
        const bool inverse = transform_direction == BFFT_INVERSE;
        double scale = 1.0;
        if (norm == BFFT_NORM_ORTHO) scale = 1.0 / std::sqrt((double)n);
        else if ((norm == BFFT_NORM_FORWARD && !inverse) || (norm == BFFT_NORM_BACKWARD && inverse))
            scale = 1.0 / (double)n;
        count_launches(1);  // the twiddle fill
        // the same passes (kernels, launch shapes, programmatic dependent
        // launch of the second pass) as a run_hybrid plan through bfft_execute
        if (e == cudaSuccess)
            e = run_hybrid_flow((const float2*)in, (float2*)out, sym.scratch, n, batch, tile, tw, inverse ? 1 : 0,
                                (float)scale, s);
    }
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    if (st != BFFT_OK) return st;
    if (e != cudaSuccess) return fail(BFFT_ERR_CUDA, "bfft_hybrid_c2c_noalloc: %s", cudaGetErrorString(e));
    return BFFT_OK;
}
