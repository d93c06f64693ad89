// bfft_stream.cu -- host-to-host execution of a batched plan, pipelined.
//
// The reference's operator API takes device tensors; a caller whose data
// lives in host memory pays the PCIe copies on top of the transform.  This
// runtime piece splits the batch into chunks and overlaps, on three internal
// streams, the host->device copy of chunk k+1, the transform of chunk k and the
// device->host copy of chunk k-1 (PCIe is full duplex), with two device
// buffers per direction.  Built only on the public C ABI (a plan for one
// chunk, bfft_execute), so every flow the library plans can be streamed.
#include <cstdarg>
#include <cstdio>
#include <cstdint>
#include <string>

#include "../../include/bfft.h"
#include "bfft_kernels.cuh"

using namespace bfft;

namespace {

bfft_status sfail(bfft_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    set_last_error(buf);
    return st;
}

bfft_status scuda(cudaError_t e, const char* what) {
    return sfail(BFFT_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

struct SDevGuard {
    int prev = -1;
    bool ok = true;
    explicit SDevGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) ok = cudaSetDevice(dev) == cudaSuccess;
    }
    ~SDevGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

}  // namespace

struct bfft_stream_plan_s {
    bfft_plan_t plan = nullptr;  // one chunk
    int64_t chunks = 0;
    size_t in_bytes = 0, out_bytes = 0, ws_bytes = 0;  // per chunk
    int32_t device = 0;
    void* din[2] = {nullptr, nullptr};
    void* dout[2] = {nullptr, nullptr};
    void* ws = nullptr;
    cudaStream_t s_in = nullptr, s_cmp = nullptr, s_out = nullptr;
    cudaEvent_t in_done[2] = {}, cmp_done[2] = {}, out_done[2] = {}, start = nullptr, end_in = nullptr,
                end_cmp = nullptr, end_out = nullptr;
};

extern "C" {

bfft_status bfft_stream_plan_destroy(bfft_stream_plan_t sp) {
    if (!sp) return BFFT_OK;
    SDevGuard g(sp->device);
    for (auto* s : {&sp->s_in, &sp->s_cmp, &sp->s_out})
        if (*s) cudaStreamSynchronize(*s);
    for (int j = 0; j < 2; ++j) {
        if (sp->din[j]) cudaFree(sp->din[j]);
        if (sp->dout[j]) cudaFree(sp->dout[j]);
        for (auto e : {sp->in_done[j], sp->cmp_done[j], sp->out_done[j]})
            if (e) cudaEventDestroy(e);
    }
    if (sp->ws) cudaFree(sp->ws);
    for (auto e : {sp->start, sp->end_in, sp->end_cmp, sp->end_out})
        if (e) cudaEventDestroy(e);
    for (auto s : {sp->s_in, sp->s_cmp, sp->s_out})
        if (s) cudaStreamDestroy(s);
    if (sp->plan) bfft_plan_destroy(sp->plan);
    delete sp;
    return BFFT_OK;
}

bfft_status bfft_stream_plan_create(const bfft_plan_desc* chunk_desc, int64_t chunks, bfft_stream_plan_t* out) {
    if (!chunk_desc || !out) return sfail(BFFT_ERR_VALUE, "NULL descriptor or output pointer");
    *out = nullptr;
    if (chunks < 1) return sfail(BFFT_ERR_VALUE, "chunks must be >= 1, got %lld", (long long)chunks);
    auto* sp = new bfft_stream_plan_s;
    sp->chunks = chunks;
    sp->device = chunk_desc->device;
    bfft_status st = bfft_plan_create(chunk_desc, &sp->plan);
    if (st != BFFT_OK) {
        std::string msg = bfft_last_error();
        delete sp;
        return sfail(st, "chunk plan: %s", msg.c_str());
    }
    const int64_t n = chunk_desc->n, b = chunk_desc->batch;
    const int tt = chunk_desc->transform_type;
    const size_t cplx_row = sizeof(float) * 2 * (size_t)n, half_row = sizeof(float) * 2 * (size_t)(n / 2 + 1);
    const size_t real_row = sizeof(float) * (size_t)n;
    sp->in_bytes = (size_t)b * (tt == BFFT_R2C ? real_row : tt == BFFT_C2R ? half_row : cplx_row);
    sp->out_bytes = (size_t)b * (tt == BFFT_R2C ? half_row : tt == BFFT_C2R ? real_row : cplx_row);
    bfft_plan_workspace_size(sp->plan, &sp->ws_bytes);
    SDevGuard g(sp->device);
    if (!g.ok) {
        bfft_stream_plan_destroy(sp);
        return sfail(BFFT_ERR_CUDA, "cannot select device %d", chunk_desc->device);
    }
    cudaError_t e = cudaSuccess;
    for (int j = 0; j < 2 && e == cudaSuccess; ++j) {
        e = cudaMalloc(&sp->din[j], sp->in_bytes);
        if (e == cudaSuccess) e = cudaMalloc(&sp->dout[j], sp->out_bytes);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sp->in_done[j], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sp->cmp_done[j], cudaEventDisableTiming);
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(&sp->out_done[j], cudaEventDisableTiming);
    }
    if (e == cudaSuccess && sp->ws_bytes) e = cudaMalloc(&sp->ws, sp->ws_bytes);
    for (auto* ev : {&sp->start, &sp->end_in, &sp->end_cmp, &sp->end_out})
        if (e == cudaSuccess) e = cudaEventCreateWithFlags(ev, cudaEventDisableTiming);
    for (auto* s : {&sp->s_in, &sp->s_cmp, &sp->s_out})
        if (e == cudaSuccess) e = cudaStreamCreateWithFlags(s, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        bfft_stream_plan_destroy(sp);
        return e == cudaErrorMemoryAllocation ? sfail(BFFT_ERR_ALLOC, "stream plan buffers: out of device memory")
                                              : scuda(e, "stream plan set-up");
    }
    *out = sp;
    return BFFT_OK;
}

bfft_status bfft_stream_plan_info(bfft_stream_plan_t sp, size_t* in_bytes_per_chunk, size_t* out_bytes_per_chunk,
                                  int* launches_per_chunk) {
    if (!sp) return sfail(BFFT_ERR_VALUE, "NULL stream plan");
    if (in_bytes_per_chunk) *in_bytes_per_chunk = sp->in_bytes;
    if (out_bytes_per_chunk) *out_bytes_per_chunk = sp->out_bytes;
    if (launches_per_chunk) bfft_plan_launches(sp->plan, launches_per_chunk);
    return BFFT_OK;
}

bfft_status bfft_stream_execute(bfft_stream_plan_t sp, const void* host_in, void* host_out, void* stream) {
    if (!sp) return sfail(BFFT_ERR_VALUE, "NULL stream plan");
    if (!host_in || !host_out) return sfail(BFFT_ERR_VALUE, "NULL host buffer");
    SDevGuard g(sp->device);
    if (!g.ok) return sfail(BFFT_ERR_CUDA, "cannot select device %d", sp->device);
    cudaStream_t caller = (cudaStream_t)stream;
    const char* hin = static_cast<const char*>(host_in);
    char* hout = static_cast<char*>(host_out);
    cudaError_t e = cudaEventRecord(sp->start, caller);  // work the caller enqueued before comes first
    for (auto s : {sp->s_in, sp->s_cmp, sp->s_out})
        if (e == cudaSuccess) e = cudaStreamWaitEvent(s, sp->start, 0);
    for (int64_t k = 0; k < sp->chunks && e == cudaSuccess; ++k) {
        const int j = (int)(k & 1);
        // copy in: buffer j was last read by the transform of chunk k-2
        if (k >= 2) e = cudaStreamWaitEvent(sp->s_in, sp->cmp_done[j], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(sp->din[j], hin + (size_t)k * sp->in_bytes, sp->in_bytes, cudaMemcpyHostToDevice,
                                sp->s_in);
        if (e == cudaSuccess) e = cudaEventRecord(sp->in_done[j], sp->s_in);
        // transform: needs chunk k in, and its output buffer copied out (chunk k-2)
        if (e == cudaSuccess) e = cudaStreamWaitEvent(sp->s_cmp, sp->in_done[j], 0);
        if (e == cudaSuccess && k >= 2) e = cudaStreamWaitEvent(sp->s_cmp, sp->out_done[j], 0);
        if (e != cudaSuccess) break;
        bfft_status st = bfft_execute(sp->plan, sp->din[j], sp->dout[j], sp->ws, sp->ws_bytes, sp->s_cmp);
        if (st != BFFT_OK) return st;
        e = cudaEventRecord(sp->cmp_done[j], sp->s_cmp);
        // copy out
        if (e == cudaSuccess) e = cudaStreamWaitEvent(sp->s_out, sp->cmp_done[j], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(hout + (size_t)k * sp->out_bytes, sp->dout[j], sp->out_bytes, cudaMemcpyDeviceToHost,
                                sp->s_out);
        if (e == cudaSuccess) e = cudaEventRecord(sp->out_done[j], sp->s_out);
    }
    // the caller's stream continues after all three streams have drained
    if (e == cudaSuccess) e = cudaEventRecord(sp->end_in, sp->s_in);
    if (e == cudaSuccess) e = cudaEventRecord(sp->end_cmp, sp->s_cmp);
    if (e == cudaSuccess) e = cudaEventRecord(sp->end_out, sp->s_out);
    for (auto ev : {sp->end_in, sp->end_cmp, sp->end_out})
        if (e == cudaSuccess) e = cudaStreamWaitEvent(caller, ev, 0);
    return e == cudaSuccess ? BFFT_OK : scuda(e, "stream execute");
}

}  // extern "C"
