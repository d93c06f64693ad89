// bfft_pass_tma.cuh -- the Stockham pass with TMA-staged column tiles.
//
// Included by bfft_kernels.cu (one translation unit: it shares the unit
// twiddle levels and the Stockham helpers).  Same transform as k_pass for the
// pass shapes whose sub-FFT index is the contiguous dimension of the input
// (every tail pass of a multi-pass flow, the strided local group, the 4-step
// column pass): a tile of K sub-FFTs x L elements is one 3-D box of a tensor
// map [outer][element][sub-FFT], copied by the Tensor Memory Accelerator into
// a dense [element][sub-FFT] shared-memory tile.  With K >= 16 that layout is
// bank-conflict free for the column thread mapping (sub-FFT index fastest)
// without padding, so the same tile is the landing buffer, the Stockham
// exchange area and the staging buffer of the store -- a TMA tensor store for
// column outputs, one bulk copy per sub-FFT for row outputs.  No thread
// computes a global address per element; the copies are asynchronous and
// tracked by mbarriers (loads) and bulk groups (stores).
//
// Pipeline: S stages per CTA (2 for 256-thread CTAs, three of which share an
// SM; 3 for the 512-thread CTAs of L = 512), persistent over tiles.  While
// tile i is transformed in stage i % S, the load of tile i+1 is in flight into
// stage (i+1) % S, whose previous contents (tile i+1-S) the store engine has
// finished reading.  No multicast: each CTA loads only its own tiles.
//
// Every wait on an mbarrier is bounded (kWaitLimitNs of %globaltimer); on
// expiry the kernel records a status bit (bfft_device_status), waits once
// more (bounded) for its copy in flight and returns.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>

namespace bfft {

__device__ unsigned int g_kernel_status;  // bit 0: a bounded mbarrier wait expired

constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
// `p` (a pointer into dynamic shared memory) rounded up to an A-byte boundary
// by pointer arithmetic, so the result keeps its shared-memory provenance and
// the compiler emits shared-memory loads and stores (LDS / STS) through it.
// (Rounding through an integer cast loses that: every access through the
// result became a generic load or store, tracked by the long scoreboard.)
template <int A>
__device__ __forceinline__ unsigned char* align_smem(unsigned char* p) {
    return p + ((A - (smem_u32(p) & (A - 1))) & (A - 1));
}
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint64_t* b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity)
        : "memory");
    return ok != 0;
}
// try_wait with a suspend-time hint: the thread may sleep until the phase
// completes or about `hint_ns` pass, instead of spinning on the barrier (a
// spinning producer warp takes issue slots from the computing warps).
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* b, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(smem_u32(b)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
// Wait for phase `parity` of `b` to complete; false (and status bit 0) when
// it has not completed within kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* b, uint32_t parity) {
    if (mbar_try_wait(b, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (mbar_try_wait_sleep(b, parity, 20000u)) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            atomicOr(&g_kernel_status, 1u);
            return false;
        }
    }
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, int c0, int c1, int c2, const void* src) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3}], [%4];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src))
                 : "memory");
}
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(reinterpret_cast<uint64_t>(dst)),
                 "r"(smem_u32(src)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}
// Programmatic dependent launch: launch_dependents lets the next kernel on
// the stream (if launched as a programmatic dependent) be scheduled once
// every CTA of this grid has issued it or exited -- its CTAs then take the
// SMs this grid's finished CTAs free and fill their tables; griddep_wait
// blocks until the previous kernel has completed and its writes are visible
// (at once for an ordinary launch).
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Generic-proxy writes to shared memory become visible to the async proxy
// (the TMA store engine) after this fence and a barrier.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__host__ __device__ constexpr uint32_t rev4(int m) {
    return static_cast<uint32_t>(((m & 1) << 3) | ((m & 2) << 1) | ((m & 4) >> 1) | ((m & 8) >> 3));
}

// ROWS 0: outputs are columns too (one tensor store per tile);
// ROWS 1: each sub-FFT's output is a contiguous row (one bulk copy each).
template <int LOG2L, int ROWS>
struct PassTGeo {
    static constexpr int L = 1 << LOG2L;
    static constexpr int E = 16;
    static constexpr int TF = L / E;
    static constexpr int K = (256 / TF) > 16 ? 256 / TF : 16;
    static constexpr int THREADS = K * TF;
    static constexpr int LB = L < 256 ? L : 256;  // TMA box extent along the element index
    static constexpr int RPAD = ROWS ? 2 : 0;     // row staging: 16-byte aligned rows, 2-way conflicts at most
    // stages start on 128-byte boundaries (TMA destinations without swizzle)
    static constexpr int SB = ((K * (L + RPAD) * 8) + 127) / 128 * 128;
    // 256-thread CTAs: two stages and <= 85 registers, three CTAs (24 warps)
    // per SM; 512-thread CTAs (L = 512): one per SM, three stages.
    static constexpr int STAGES = THREADS >= 512 ? 3 : 2;
    static constexpr int MINB = THREADS >= 512 ? 1 : 3;
    // W_N column factors shared by the TF threads of a sub-FFT (TF >= 4):
    // a [m][sub-FFT] table of 16 x K entries
    static constexpr bool COLTW = TF >= 4;
    static constexpr int COLTW_ENTRIES = COLTW ? 16 * K : 0;
    static constexpr int CPT = TF >= 16 ? 1 : 16 / TF;  // column factors per thread
    static constexpr size_t SMEM =
        128 + (size_t)STAGES * SB + 64 + (size_t)(tw_total(LOG2L) + COLTW_ENTRIES) * sizeof(float2);
    static_assert(L >= 16 && K <= 256 && LB <= 256, "TMA box limits");
};

// TW3: the pass's W_N twiddles come from the plan's three-level table (N > 2^22).
template <int LOG2L, int ROWS, bool TW3>
__global__ void __launch_bounds__(PassTGeo<LOG2L, ROWS>::THREADS, PassTGeo<LOG2L, ROWS>::MINB)
    k_pass_tma(const __grid_constant__ CUtensorMap tin, const __grid_constant__ CUtensorMap tout,
               float2* __restrict__ out, PassArgs a) {
    using G = PassTGeo<LOG2L, ROWS>;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = align_smem<128>(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + G::STAGES * G::SB);
    float2* tw_smem = reinterpret_cast<float2*>(full + 8);
    float2* coltw = tw_smem + tw_total(LOG2L);
    auto stage = [&](int s) { return reinterpret_cast<float2*>(base + s * G::SB); };

    const int tid = threadIdx.x;
    const int cl = tid % G::K, t = tid / G::K;
    constexpr int NST = ROWS ? G::K : 1;  // threads that issue (and wait for) stores
    const int64_t ntiles = a.nsub / G::K;
    const int64_t imask = (int64_t(1) << a.inner_log2) - 1;
    const float osr = a.scale, osi = a.conj_out ? -a.scale : a.scale;
    const bool scaled = a.scale != 1.0f || a.conj_out;  // uniform: skip the epilogue multiply when it is 1

    auto issue = [&](int64_t tl, int s) {  // thread 0 only
        const int64_t f0 = tl * G::K;
        const int o = static_cast<int>(f0 >> a.inner_log2), c0 = static_cast<int>(f0 & imask);
        float2* dst = stage(s);
        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(G::K * G::L * sizeof(float2)));
#pragma unroll
        for (int j = 0; j < G::L / G::LB; ++j) tma_load_3d(dst + j * G::LB * G::K, &tin, c0, j * G::LB, o, &full[s]);
    };
    int64_t tile = blockIdx.x;
    if (tile >= ntiles) griddep_launch_dependents();  // no tile for this CTA
    if (tid == 0) {  // the first tile is in flight while the tables are filled
        for (int s = 0; s < G::STAGES; ++s) mbar_init(&full[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_proxy_async_smem();
        griddep_wait();  // every read and write of the flow's buffers follows this (tables are plan-owned)
        if (tile < ntiles) issue(tile, 0);
    }
    fill_stockham_twiddles<LOG2L>(tw_smem);
    SmemTwiddle<TW3 ? 3 : 2> twiddle;  // W_N lookups, staged in shared memory when they fit
    twiddle.setup(coltw + G::COLTW_ENTRIES, a);
    __syncthreads();

    // The W_N twiddle of element e = t + m TF of sub-FFT c is W^{e C} with
    // C = c tw_mul, i.e. W^{t C} W^{m TF C}.  With TF >= 4 the 16 column
    // factors W^{m TF C} of a sub-FFT are shared by its TF threads: each
    // thread computes its share (m = t, t + TF, ...) into the [m][sub-FFT]
    // table while the tile is still in flight, plus its own W^{t C}: 1 +
    // max(1, 16/TF) W_N lookups per thread and tile instead of 16.  Thread
    // t = 0 has W^0 = 1 exactly, so its twiddles are the table's.  The table
    // is read only between the tile's first barrier and its last one, and
    // written only before the first.
    const bool twiddled = a.tw_mode != 0;  // uniform

    // bit reversal over log2 L bits of e = t + m TF (t < TF, m < 16) is
    // rev(t) * 16 + rev4(m): a per-thread base plus a constant per element
    const uint32_t rt16 = LOG2L > 4 ? (brev_bits(static_cast<uint32_t>(t), LOG2L - 4) << 4) : 0u;

    int it = 0;
    bool aborted = false;
    for (; tile < ntiles; ++it, tile += gridDim.x) {
        // the next pass may be scheduled once every CTA is on its last tile
        // (measured: as fast as triggering at the start on short flows, no
        // interference with long ones)
        if (tile + gridDim.x >= ntiles) griddep_launch_dependents();
        const int s = it % G::STAGES;
        float2* buf = stage(s);
        const int64_t f = tile * G::K + cl;
        const int64_t o = f >> a.inner_log2, c = f & imask;
        const uint32_t cmul32 = static_cast<uint32_t>(c) * static_cast<uint32_t>(a.tw_mul);
        const float2* cf = coltw + cl;  // this sub-FFT's column factors
        float2 tb = make_float2(1.f, 0.f);
        if constexpr (G::COLTW) {
            if (twiddled) {
#pragma unroll
                for (int j = 0; j < G::CPT; ++j) {
                    const int m = t + j * G::TF;
                    if (m < 16) coltw[m * G::K + cl] = twiddle(static_cast<uint32_t>(m * G::TF) * cmul32);
                }
                tb = twiddle(static_cast<uint32_t>(t) * cmul32);
            }
        }
        // W^{(t + m TF) C}
        auto wn = [&](int m) {
            if constexpr (G::COLTW) return cmul(tb, cf[m * G::K]);
            else return twiddle(static_cast<uint32_t>(t + m * G::TF) * cmul32);
        };
        // the stores that read the stage the next load will fill (tile it+1-STAGES) are done reading
        if (tid < NST) bulk_wait_read<G::STAGES - 2>();
        const bool ok = mbar_wait_bounded(&full[s], static_cast<uint32_t>((it / G::STAGES) & 1));

        float2 v[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            const uint32_t e = static_cast<uint32_t>(t + m * G::TF);
            const uint32_t pe = a.in_elem_bitrev ? rt16 + rev4(m) : e;
            float2 val = ok ? buf[pe * G::K + cl] : make_float2(0.f, 0.f);
            if (a.conj_in) val.y = -val.y;
            if constexpr (!G::COLTW) {
                if (a.tw_mode == 1) val = cmul(val, wn(m));
            }
            v[m] = val;
        }
        if (__syncthreads_or(!ok)) {  // the tile is now the exchange area; the column factors are published
            aborted = true;
            break;
        }
        if (tid == 0 && tile + gridDim.x < ntiles) issue(tile + gridDim.x, (it + 1) % G::STAGES);
        if constexpr (G::COLTW) {
            if (a.tw_mode == 1) {
#pragma unroll
                for (int m = 0; m < 16; ++m) v[m] = cmul(v[m], wn(m));
            }
        }

        stockham_passes<LOG2L, 0, 16, G::TF, G::K>(v, t, buf + cl, tw_smem);

#pragma unroll
        for (int m = 0; m < 16; ++m) {
            const uint32_t k = static_cast<uint32_t>(t + m * G::TF);
            float2 val = v[m];
            if (a.tw_mode == 2) val = cmul(val, wn(m));
            if (scaled) val = make_float2(val.x * osr, val.y * osi);
            if constexpr (ROWS) {
                buf[cl * (G::L + G::RPAD) + k] = val;
            } else {
                const uint32_t pk = a.out_elem_bitrev ? rt16 + rev4(m) : k;
                buf[pk * G::K + cl] = val;
            }
        }
        fence_proxy_async_smem();
        __syncthreads();
        if constexpr (ROWS) {
            if (tid < G::K) {  // t == 0: this thread's sub-FFT is f
                const int64_t cout = a.out_base_bits ? static_cast<int64_t>(brev_bits(static_cast<uint32_t>(c), a.out_base_bits)) : c;
                bulk_store(out + o * a.out_outer + cout * a.out_inner, buf + tid * (G::L + G::RPAD),
                           static_cast<uint32_t>(G::L * sizeof(float2)));
                bulk_commit();
            }
        } else {
            if (tid == 0) {
                const int64_t f0 = tile * G::K;
                const int oo = static_cast<int>(f0 >> a.inner_log2), c0 = static_cast<int>(f0 & imask);
#pragma unroll
                for (int j = 0; j < G::L / G::LB; ++j) tma_store_3d(&tout, c0, j * G::LB, oo, buf + j * G::LB * G::K);
                bulk_commit();
            }
        }
    }
    if (aborted && tid == 0)  // the copy this tile waited for may still land: wait (bounded) before leaving
        mbar_wait_bounded(&full[it % G::STAGES], static_cast<uint32_t>((it / G::STAGES) & 1));
    if (tid < NST) bulk_wait<0>();
}

// ---- row tiles: sub-FFTs whose elements are contiguous (L >= 32) ----
//
// A tile is K rows of L points; every row is one bulk copy (one copy for the
// whole tile when its rows are adjacent and unpadded) into a [row][element]
// stage of row stride RS, read with the element-fastest thread mapping
// (thread t of a row holds elements t + m TF).  For L >= 256 a half-warp
// reads within one row and RS = L (dense); shorter rows put 16 / TF rows in a
// half-warp, and RS = L + TF (= TF mod 16, 16-byte aligned) spreads them over
// all banks.  The Stockham exchanges then use a padded per-row layout in the
// same stage, and the outputs are staged with row stride RS again for bulk
// copies out.  A partial last tile copies only its rows.
template <int LOG2L>
struct PassRGeo {
    static constexpr int L = 1 << LOG2L;
    static constexpr int E = 16;
    static constexpr int TF = L / E;
    static constexpr int K = 256 / TF;  // 256 threads
    static constexpr int THREADS = 256;
    static constexpr int RS = L >= 256 ? L : L + TF;
    // exchange row stride: odd for L >= 256; = TF mod 16 below (L + L/16)
    static constexpr int LPAD = L >= 256 ? (L + (L >> 4)) | 1 : L + (L >> 4);
    static constexpr int ROWW = RS > LPAD ? RS : LPAD;
    // bulk copies need 16-byte alignment only: 128-byte rounding, not 1 KB
    static constexpr int SB = ((K * ROWW * 8) + 127) / 128 * 128;
    static constexpr int STAGES = 2;
    static constexpr int MINB = 3;
    static constexpr size_t SMEM = 128 + (size_t)STAGES * SB + 64 + (size_t)tw_total(LOG2L) * sizeof(float2);
    static_assert(L >= 32 && K >= 1 && (RS * 8) % 16 == 0, "row tile geometry");
};

template <int LOG2L>
__global__ void __launch_bounds__(PassRGeo<LOG2L>::THREADS, PassRGeo<LOG2L>::MINB)
    k_pass_tma_rows(const float2* __restrict__ in, float2* __restrict__ out, PassArgs a, int in_contig,
                    int out_contig) {
    using G = PassRGeo<LOG2L>;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = align_smem<128>(smem_raw);
    uint64_t* full = reinterpret_cast<uint64_t*>(base + G::STAGES * G::SB);
    float2* tw_smem = reinterpret_cast<float2*>(full + 8);
    auto stage = [&](int s) { return reinterpret_cast<float2*>(base + s * G::SB); };

    const int tid = threadIdx.x;
    const int cl = tid / G::TF, t = tid % G::TF;
    const int64_t ntiles = (a.nsub + G::K - 1) / G::K;
    const int64_t imask = (int64_t(1) << a.inner_log2) - 1;
    const float osr = a.scale, osi = a.conj_out ? -a.scale : a.scale;
    const bool scaled = a.scale != 1.0f || a.conj_out;  // uniform: skip the epilogue multiply when it is 1
    const int NST = out_contig ? 1 : G::K;  // threads that issue (and wait for) stores

    auto row_in = [&](int64_t f) -> const float2* {
        const int64_t o = f >> a.inner_log2, c = f & imask;
        const int64_t cin = a.in_base_bits ? (int64_t)brev_bits((uint32_t)c, a.in_base_bits) : c;
        return in + o * a.in_outer + cin * a.in_inner;
    };
    auto row_out = [&](int64_t f) -> float2* {
        const int64_t o = f >> a.inner_log2, c = f & imask;
        const int64_t cout = a.out_base_bits ? (int64_t)brev_bits((uint32_t)c, a.out_base_bits) : c;
        return out + o * a.out_outer + cout * a.out_inner;
    };
    // Called by every thread for L < 256, else by thread 0.  Thread 0 posts
    // the tile's byte count; the row copies are spread over threads tid < K
    // when there are many (L < 256) -- a copy may complete before the count
    // is posted, the phase cannot (its one arrival is thread 0's).
    auto issue = [&](int64_t tl, int s) {
        const int64_t f0 = tl * G::K;
        const int rows = static_cast<int>(a.nsub - f0 < G::K ? a.nsub - f0 : G::K);
        float2* dst = stage(s);
        const uint32_t row_bytes = static_cast<uint32_t>(G::L * sizeof(float2));
        if (tid == 0) mbar_arrive_expect_tx(&full[s], row_bytes * rows);
        if (in_contig) {
            if (tid == 0) bulk_load(dst, row_in(f0), row_bytes * rows, &full[s]);
        } else if constexpr (G::L >= 256) {
            if (tid == 0)
                for (int r = 0; r < rows; ++r) bulk_load(dst + r * G::RS, row_in(f0 + r), row_bytes, &full[s]);
        } else {
            if (tid < rows) bulk_load(dst + tid * G::RS, row_in(f0 + tid), row_bytes, &full[s]);
        }
    };

    int64_t tile = blockIdx.x;
    if (tile >= ntiles) griddep_launch_dependents();  // no tile for this CTA
    if (tid == 0) {
        for (int s = 0; s < G::STAGES; ++s) mbar_init(&full[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_proxy_async_smem();
        griddep_wait();  // every read and write of the flow's buffers follows this (tables are plan-owned)
        // one issuing thread: the first tile is in flight while the tables are filled
        if (G::L >= 256 && tile < ntiles) issue(tile, 0);
    }
    fill_stockham_twiddles<LOG2L>(tw_smem);
    SmemTwiddle<2> twiddle;  // W_N lookups, staged in shared memory when they fit
    twiddle.setup(tw_smem + tw_total(LOG2L), a);
    __syncthreads();
    if (G::L < 256 && tile < ntiles) issue(tile, 0);  // the barriers are initialised now
    int it = 0;
    bool aborted = false;
    for (; tile < ntiles; ++it, tile += gridDim.x) {
        // the next pass may be scheduled once every CTA is on its last tile
        // (measured: as fast as triggering at the start on short flows, no
        // interference with long ones)
        if (tile + gridDim.x >= ntiles) griddep_launch_dependents();
        const int s = it % G::STAGES;
        float2* buf = stage(s);
        const int64_t f = tile * G::K + cl;
        const bool active = f < a.nsub;
        const int64_t c = f & imask;
        if (tid < NST) bulk_wait_read<G::STAGES - 2>();
        const bool ok = mbar_wait_bounded(&full[s], static_cast<uint32_t>((it / G::STAGES) & 1));

        const uint32_t cmul32 = static_cast<uint32_t>(c) * static_cast<uint32_t>(a.tw_mul);
        float2 v[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            const uint32_t e = static_cast<uint32_t>(t + m * G::TF);
            float2 val = ok ? buf[cl * G::RS + e] : make_float2(0.f, 0.f);
            if (a.conj_in) val.y = -val.y;
            if (a.tw_mode == 1) val = cmul(val, twiddle(e * cmul32));
            v[m] = val;
        }
        if (__syncthreads_or(!ok)) {
            aborted = true;
            break;
        }
        if ((G::L < 256 || tid == 0) && tile + gridDim.x < ntiles) issue(tile + gridDim.x, (it + 1) % G::STAGES);

        // packed FP32x2 adds: +7-9 % on these passes (measured; not on the column pass)
        stockham_passes<LOG2L, 0, 16, G::TF, 0, true>(v, t, buf + cl * G::LPAD, tw_smem);

#pragma unroll
        for (int m = 0; m < 16; ++m) {
            const uint32_t k = static_cast<uint32_t>(t + m * G::TF);
            float2 val = v[m];
            if (a.tw_mode == 2) val = cmul(val, twiddle(k * cmul32));
            buf[cl * G::RS + k] = scaled ? make_float2(val.x * osr, val.y * osi) : val;
        }
        fence_proxy_async_smem();
        __syncthreads();
        const int64_t f0 = tile * G::K;
        const int rows = static_cast<int>(a.nsub - f0 < G::K ? a.nsub - f0 : G::K);
        const uint32_t row_bytes = static_cast<uint32_t>(G::L * sizeof(float2));
        if (out_contig) {
            if (tid == 0) {
                bulk_store(row_out(f0), buf, row_bytes * rows);
                bulk_commit();
            }
        } else if (tid < G::K) {
            if (tid < rows) bulk_store(row_out(f0 + tid), buf + tid * G::RS, row_bytes);
            bulk_commit();  // an empty group keeps every storing thread's group count in step
        }
        (void)active;
    }
    if (aborted && tid == 0)
        mbar_wait_bounded(&full[it % G::STAGES], static_cast<uint32_t>((it / G::STAGES) & 1));
    if (tid < NST) bulk_wait<0>();
}

// ---- host side ----

// An ordinary launch, or (pdl) one with programmatic stream serialisation.
template <typename... KArgs, typename... Args>
static cudaError_t launch_maybe_pdl(void (*kern)(KArgs...), unsigned grid, unsigned threads, size_t smem,
                                    cudaStream_t s, int pdl, Args... args) {
    if (!pdl) {
        kern<<<grid, threads, smem, s>>>(args...);
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, args...);
    return e != cudaSuccess ? e : cudaGetLastError();
}

using EncodeTiledFn = PFN_cuTensorMapEncodeTiled_v12000;

static EncodeTiledFn tensor_map_encoder() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

// 3-D map of complex64 (8-byte elements) [d2][d1][d0] with byte strides s1, s2.
static bool encode_map_3d(CUtensorMap* m, const void* ptr, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                          uint64_t s2, uint32_t b0, uint32_t b1) {
    EncodeTiledFn enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[3] = {d0, d1, d2};
    cuuint64_t strides[2] = {s1, s2};
    cuuint32_t box[3] = {b0, b1, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT64, 3, const_cast<void*>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int LOG2L, int ROWS>
static cudaError_t launch_pass_tma_t(const float2* in, float2* out, const PassArgs& a, cudaStream_t s) {
    using G = PassTGeo<LOG2L, ROWS>;
    constexpr size_t kSmemCap = 227 * 1024;
    static std::atomic<int> blocks_per_sm[64][2][kTwClasses];  // [device][three-level][class]
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const uint64_t inner = 1ull << a.inner_log2, nouter = static_cast<uint64_t>(a.nsub) >> a.inner_log2;
    CUtensorMap tin, tout;
    if (!encode_map_3d(&tin, in, inner, G::L, nouter, static_cast<uint64_t>(a.in_stride) * 8,
                       static_cast<uint64_t>(a.in_outer) * 8, G::K, G::LB))
        return cudaErrorNotSupported;
    if (ROWS) {
        tout = tin;  // unused: row outputs are bulk copies
    } else if (!encode_map_3d(&tout, out, inner, G::L, nouter, static_cast<uint64_t>(a.out_stride) * 8,
                              static_cast<uint64_t>(a.out_outer) * 8, G::K, G::LB)) {
        return cudaErrorNotSupported;
    }
    PassArgs b = a;
    int cls = 0;
    choose_tw_staging(b, G::SMEM, kSmemCap, cls, 3);
    const bool tw3 = b.tw_smem_levels == 3;
    const size_t smem_cls = G::SMEM + tw_class_bytes(cls);
    int sms = 0, nb = 0;
    e = device_sm_count(dev, &sms);
    if (e == cudaSuccess)
        e = tw3 ? cached_occupancy(blocks_per_sm[dev][1][cls], k_pass_tma<LOG2L, ROWS, true>, G::THREADS, smem_cls,
                                   kSmemCap, &nb)
                : cached_occupancy(blocks_per_sm[dev][0][cls], k_pass_tma<LOG2L, ROWS, false>, G::THREADS, smem_cls,
                                   kSmemCap, &nb);
    if (e != cudaSuccess) return e;
    const int64_t ntiles = b.nsub / G::K;
    int64_t grid = (int64_t)nb * sms;
    if (grid > ntiles) grid = ntiles;
    if (grid < 1) grid = 1;
    const size_t smem = G::SMEM + (size_t)b.tw_smem_entries * sizeof(float2);
    if (tw3)
        return launch_maybe_pdl(k_pass_tma<LOG2L, ROWS, true>, (unsigned)grid, G::THREADS, smem, s, b.pdl, tin, tout,
                                out, b);
    return launch_maybe_pdl(k_pass_tma<LOG2L, ROWS, false>, (unsigned)grid, G::THREADS, smem, s, b.pdl, tin, tout,
                            out, b);
}

template <int LOG2L>
static cudaError_t launch_pass_tma_rows_t(const float2* in, float2* out, const PassArgs& a, int in_contig,
                                          int out_contig, cudaStream_t s) {
    using G = PassRGeo<LOG2L>;
    auto kern = k_pass_tma_rows<LOG2L>;
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
    return launch_maybe_pdl(kern, (unsigned)grid, G::THREADS, smem, s, b.pdl, in, out, b, in_contig, out_contig);
}

// Row tiles through bulk copies when the shapes allow it.
static cudaError_t launch_pass_tma_rows(int log2l, const float2* in, float2* out, const PassArgs& a,
                                        cudaStream_t s) {
    // 16-point rows (one thread per row, 256 copies per tile) measured faster on k_pass
    if (log2l < 5 || log2l > 12) return cudaErrorNotSupported;
    const int64_t L = int64_t(1) << log2l;
    const int k = 256 / (int)(L / 16);
    const int64_t inner = int64_t(1) << a.inner_log2;
    if (((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) || a.in_stride != 1 ||
        a.out_stride != 1 || a.in_elem_bitrev || a.out_elem_bitrev)
        return cudaErrorNotSupported;
    // every row start 16-byte aligned
    if ((a.in_outer & 1) || (inner > 1 && (a.in_inner & 1)) || (a.out_outer & 1) || (inner > 1 && (a.out_inner & 1)))
        return cudaErrorNotSupported;
    // a tile's rows are adjacent in memory: one copy per tile
    auto contiguous = [&](int64_t outer, int64_t inner_stride, int base_bits) {
        if (inner == 1) return outer == L;
        return !base_bits && inner_stride == L && outer == inner * L && inner % k == 0;
    };
    // padded stages (L < 256) take one copy per row
    const int in_contig = log2l >= 8 && contiguous(a.in_outer, a.in_inner, a.in_base_bits) ? 1 : 0;
    const int out_contig = log2l >= 8 && contiguous(a.out_outer, a.out_inner, a.out_base_bits) ? 1 : 0;
    switch (log2l) {
        case 5: return launch_pass_tma_rows_t<5>(in, out, a, in_contig, out_contig, s);
        case 6: return launch_pass_tma_rows_t<6>(in, out, a, in_contig, out_contig, s);
        case 7: return launch_pass_tma_rows_t<7>(in, out, a, in_contig, out_contig, s);
        case 8: return launch_pass_tma_rows_t<8>(in, out, a, in_contig, out_contig, s);
        case 9: return launch_pass_tma_rows_t<9>(in, out, a, in_contig, out_contig, s);
        case 10: return launch_pass_tma_rows_t<10>(in, out, a, in_contig, out_contig, s);
        case 11: return launch_pass_tma_rows_t<11>(in, out, a, in_contig, out_contig, s);
        case 12: return launch_pass_tma_rows_t<12>(in, out, a, in_contig, out_contig, s);
        default: return cudaErrorNotSupported;
    }
}

// The TMA pass when the shapes allow it; cudaErrorNotSupported otherwise
// (the caller then runs k_pass).
static cudaError_t launch_pass_tma(int log2l, const float2* in, float2* out, const PassArgs& a, cudaStream_t s) {
    if (log2l < 4 || log2l > 9) return cudaErrorNotSupported;
    const int tf = (1 << log2l) / 16;
    const int k = (256 / tf) > 16 ? 256 / tf : 16;
    int lk = 0;
    while ((1 << lk) < k) ++lk;
    const bool aligned = ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
    if (!aligned || a.inner_log2 < lk || a.inner_log2 > 30 || (a.nsub & ((int64_t(1) << a.inner_log2) - 1)) ||
        (a.nsub >> a.inner_log2) >= (int64_t(1) << 31))
        return cudaErrorNotSupported;
    if (a.in_inner != 1 || a.in_base_bits || (a.in_stride & 1) || (a.in_outer & 1) || a.in_stride <= 0)
        return cudaErrorNotSupported;
    const bool col_out = a.out_inner == 1 && !a.out_base_bits && !(a.out_stride & 1) && !(a.out_outer & 1) &&
                         a.out_stride > 0;
    const bool row_out = a.out_stride == 1 && !a.out_elem_bitrev && !(a.out_inner & 1) && !(a.out_outer & 1);
    if (!col_out && !row_out) return cudaErrorNotSupported;
#define BFFT_TMA_CASE(L)                                                                             \
    case L:                                                                                          \
        return col_out ? launch_pass_tma_t<L, 0>(in, out, a, s) : launch_pass_tma_t<L, 1>(in, out, a, s);
    switch (log2l) {
        BFFT_TMA_CASE(4)
        BFFT_TMA_CASE(5)
        BFFT_TMA_CASE(6)
        BFFT_TMA_CASE(7)
        BFFT_TMA_CASE(8)
        BFFT_TMA_CASE(9)
        default: return cudaErrorNotSupported;
    }
#undef BFFT_TMA_CASE
}

}  // namespace bfft
