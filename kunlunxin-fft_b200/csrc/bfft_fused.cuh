// bfft_fused.cuh -- whole transforms of N = N1 * N2 points (2^13 .. 2^20) in
// one HBM round trip, as one persistent kernel.
//
// Included by bfft_kernels.cu after bfft_pass_tma.cuh (it uses the TMA /
// mbarrier helpers, the Stockham passes and the column-tile geometry).
//
// The 4-step decomposition X[k1 + N1 k2] = sum_n2 W_N2^{n2 k2} W_N^{n2 k1}
// sum_n1 x[n1 N2 + n2] W_N1^{n1 k1} splits every transform into
//   phase A: N2 column FFTs of N1 points (x read with stride N2), the twiddle
//            W_N^{k1 n2} applied to their outputs, each column's N1 outputs
//            written as one row n2 of a scratch slot S[n2][k1];
//   phase B: N1 FFTs of N2 points over n2 for each k1 (columns of S), written
//            to X[k1 + N1 k2] (out read as [k2][k1], k1 contiguous).
// Both phases are tiles of K sub-FFTs (FusedTile: 8..64 columns) loaded by
// TMA boxes into a dense [element][sub-FFT] shared tile, so the same tile is
// the landing buffer, the Stockham exchange area and the store staging.
//
// The intermediate never goes to HBM on purpose: scratch slots form a ring of
// S transforms (tens of MiB) whose stores and loads carry an L2 evict_last
// policy while the input and output streams carry evict_first, so the ring
// stays in the 126 MB L2 and HBM sees one read of x and one write of X.
//
// Scheduling: tickets from one global counter, in rounds of TA + TB tickets:
// round r holds the TA phase-A tiles of transform r and the TB phase-B tiles
// of transform r - D (the lag D lets phase A of a transform finish before its
// phase-B tickets come up).  Dependencies point only to earlier tickets:
//   B(b, i) needs the TA phase-A tiles of b completed (a_done[slot]);
//   A(b, j) needs the TB phase-B tiles of b - S (the slot's previous user)
//           to have read the slot (b_done[slot]), and S > D.
// A CTA processes its tickets in order and claims the next one while working
// on the current one, so the smallest unfinished ticket can always proceed:
// no co-residency is assumed.  Every wait is bounded (kWaitLimitNs of
// %globaltimer); an expired wait sets bit 1 (dependency) or bit 0 (mbarrier)
// of bfft_device_status and the CTA stops after its copies in flight land.
#pragma once

namespace bfft {

// Tile of one phase: NC consumer threads, each carrying 16 elements of two
// sub-FFTs (a pair); TF threads share a pair of L-point sub-FFTs, so a tile
// holds K = 2 NC / TF sub-FFTs (columns) -- 16 for L = 256 with 128 consumers,
// 8 for L = 1024 with 256.  Loaded by TMA boxes of K columns x LB elements into
// a dense [element][column] stage (the landing buffer, the Stockham exchange
// area and the store staging); ROWS 1 stages each output sub-FFT as a row
// (padded) for one bulk copy each.
template <int LOG2L, int ROWS, int NC>
struct FusedTile {
    static constexpr int L = 1 << LOG2L;
    static constexpr int TF = L / 16;
    static constexpr int NP = NC / TF;  // column pairs per tile
    static constexpr int K = 2 * NP;
    static constexpr int LB = L < 256 ? L : 256;  // TMA box extent along the element index
    static constexpr int RPAD = ROWS ? 2 : 0;     // row staging: 16-byte aligned rows
    static constexpr int SB = ((K * (L + RPAD) * 8) + 127) / 128 * 128;
    // W_N column factors shared by the TF threads of a sub-FFT pair: [m][pair], 16 x NP
    static constexpr bool COLTW = TF >= 4;
    static constexpr int CPT = TF >= 16 ? 1 : 16 / TF;  // column factors per thread
    static_assert(L >= 64 && NP >= 1 && K <= 256 && (K * 8) % 16 == 0, "fused tile geometry");
};

// 128 consumers (two CTAs per SM, 32 KiB stages) for sub-FFTs of <= 256
// points (N = 2^13..2^16); 256 consumers (one CTA per SM, 64 KiB stages) when
// a phase has 512- or 1024-point sub-FFTs (N = 2^17..2^20).
template <int LA, int LB>
struct FusedGeo {
    static constexpr bool WIDE = LA > 8 || LB > 8;
    static constexpr int CONSUMERS = WIDE ? 256 : 128;
    using GA = FusedTile<LA, 1, CONSUMERS>;  // phase A: column FFTs of N1, rows out (bulk copies)
    using GB = FusedTile<LB, 0, CONSUMERS>;  // phase B: column FFTs of N2 over the slot, columns out (TMA store)
    static constexpr int N1 = 1 << LA, N2 = 1 << LB;
    static constexpr int THREADS = CONSUMERS + 64;  // + the loader and the storer warps
    static constexpr int MINB = WIDE ? 1 : 2;
    static constexpr int NPA = GA::NP, NPB = GB::NP;  // column pairs per tile
    static constexpr int SB = GA::SB > GB::SB ? GA::SB : GB::SB;
    static constexpr int STAGES = 3;
    static constexpr int TA = N2 / GA::K;  // phase-A tiles per transform
    static constexpr int TB = N1 / GB::K;  // phase-B tiles per transform
    static_assert(TA >= 1 && TB >= 1, "N1 * N2 >= 4096");
    // pair twiddle tables (16 bytes an entry), one table when both phases have the same length
    static constexpr bool SHARED_TW = LA == LB;
    static constexpr int TWA = tw_total(LA), TWB = SHARED_TW ? 0 : tw_total(LB);
    static constexpr int COLTW = GA::COLTW ? 16 * NPA : 0;  // column-factor pairs of phase A
    // alignment slack, stages, control block (mbarriers, the stage items), tables; no static
    // shared memory, so the launcher may raise the dynamic limit to the full 227 KiB
    static constexpr int CTRL = 256;
    static constexpr size_t SMEM = 128 + (size_t)STAGES * SB + CTRL + (size_t)(TWA + TWB + COLTW) * sizeof(CPair);
    static_assert(SMEM <= 220 * 1024, "fused stages");
};

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const CUtensorMap* map, int c0, int c1, int c2,
                                                 uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void tma_store_3d_hint(const CUtensorMap* map, int c0, int c1, int c2, const void* src,
                                                  uint64_t pol) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group.L2::cache_hint"
                 " [%0, {%1, %2, %3}], [%4], %5;" ::"l"(reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src)), "l"(pol)
                 : "memory");
}
__device__ __forceinline__ void bulk_store_hint(void* dst, const void* src, uint32_t bytes, uint64_t pol) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group.L2::cache_hint [%0], [%1], %2, %3;" ::"l"(
                     reinterpret_cast<uint64_t>(dst)),
                 "r"(smem_u32(src)), "r"(bytes), "l"(pol)
                 : "memory");
}
// Order this thread's generic-proxy accesses (an acquire just made) with its
// later async-proxy (TMA / bulk) accesses of global memory, and the reverse.
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Wait (bounded) until *p >= target; false and status bit 1 on expiry.
__device__ __forceinline__ bool counter_wait_bounded(const uint32_t* p, uint32_t target) {
    if (ld_acquire_u32(p) >= target) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        __nanosleep(64);
        if (ld_acquire_u32(p) >= target) return true;
        if (global_timer_ns() - t0 > kWaitLimitNs) {
            atomicOr(&g_kernel_status, 2u);
            return false;
        }
    }
}

// One claimed work item.  kind: 0 none (no tickets left), 1 phase A, 2 phase B.
struct FusedItem {
    int kind;
    int idx;      // tile within the phase
    int64_t b;    // transform
};

__device__ __forceinline__ void mbar_arrive(uint64_t* b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(b)) : "memory");
}

// Warp-specialised: the consumer warps (threads 0 .. CONSUMERS-1) compute
// tiles and meet only at named barrier 1; lane 0 of the next warp (the
// loader) claims tickets, waits on dependencies and starts the TMA loads;
// lane 0 of the last warp (the storer) stores finished tiles and publishes
// them.  Consumers never wait for a global
// atomic or a store to complete.  The q-th item of the CTA uses stage q % ST:
//   full[s]   loader    -> consumers, storer: the tile landed (s_item[s] set);
//   staged[s] consumers -> storer: the results are staged in the stage;
//   empty[s]  storer    -> loader: the stores have read the stage.
// The storer publishes a phase-A tile (a_done) as soon as its row stores are
// complete (after releasing the stage), a phase-B tile (b_done) as soon as it
// has landed.  An issued item therefore finishes without the
// loader, and the loader may block on a dependency (always an earlier ticket)
// without closing a cycle.
template <int LA, int LB>
__global__ void __launch_bounds__(FusedGeo<LA, LB>::THREADS, FusedGeo<LA, LB>::MINB)
    k_fused_fft(const __grid_constant__ CUtensorMap ta_in, const __grid_constant__ CUtensorMap tb_in,
                const __grid_constant__ CUtensorMap tb_out, FusedArgs a) {
    using G = FusedGeo<LA, LB>;
    using GA = typename G::GA;
    using GB = typename G::GB;
    constexpr int ST = G::STAGES;
    constexpr int NC = G::CONSUMERS;
    static_assert(8 * 3 * ST + ST * sizeof(FusedItem) + sizeof(int) <= G::CTRL, "control block");
    static_assert(G::CONSUMERS % 32 == 0, "whole consumer warps");
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = align_smem<128>(smem_raw);
    unsigned char* ctrl = base + ST * G::SB;
    uint64_t* full = reinterpret_cast<uint64_t*>(ctrl);
    uint64_t* staged = full + ST;
    uint64_t* empty = staged + ST;
    FusedItem* s_item = reinterpret_cast<FusedItem*>(ctrl + 8 * 3 * ST);
    volatile int* s_abort = reinterpret_cast<volatile int*>(ctrl + 8 * 3 * ST + ST * sizeof(FusedItem));
    CPair* twA = reinterpret_cast<CPair*>(ctrl + G::CTRL);
    CPair* twB = G::SHARED_TW ? twA : twA + G::TWA;
    CPair* coltw = twA + G::TWA + G::TWB;
    auto stage = [&](int s) { return reinterpret_cast<float2*>(base + s * G::SB); };

    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&staged[s], 1);
            mbar_init(&empty[s], 1);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        fence_proxy_async_smem();
        *s_abort = 0;
    }
    fill_pair_twiddles<LA>(twA);
    if constexpr (!G::SHARED_TW) fill_pair_twiddles<LB>(twB);
    SmemTwiddle<2> twiddle;  // W_N lookups (phase-A post-twiddle), staged in shared memory when they fit
    {
        PassArgs pa{};
        pa.tw = a.tw;
        pa.tw_smem_entries = a.tw_smem_entries;
        pa.tw_smem_levels = a.tw_smem_levels;
        twiddle.setup(reinterpret_cast<float2*>(coltw + G::COLTW), pa);
    }
    __syncthreads();  // the last CTA-wide barrier: the warps part ways here

    const int S = a.slots;
    uint32_t* a_done = a.counters + 1;
    uint32_t* b_done = a.counters + 1 + S;
    if (tid == NC) {
        // ================================================ loader
        uint32_t* ticket = a.counters;
        const int64_t round_len = G::TA + G::TB;
        const int64_t ntickets = (a.batch + a.lag) * round_len;
        const uint64_t pol_stream = policy_evict_first(), pol_keep = policy_evict_last();
        griddep_wait();
        auto decode = [&](uint32_t t) -> FusedItem {  // kind -1: a ticket of no work (ring edges)
            if ((int64_t)t >= ntickets) return FusedItem{0, 0, 0};
            const int64_t r = (int64_t)t / round_len;
            const int j = (int)((int64_t)t - r * round_len);
            if (j < G::TA) return r < a.batch ? FusedItem{1, j, r} : FusedItem{-1, 0, 0};
            return (r >= a.lag && r - a.lag < a.batch) ? FusedItem{2, j - G::TA, r - a.lag} : FusedItem{-1, 0, 0};
        };
        auto ready = [&](const FusedItem& it, bool block) -> bool {
            const int slot = (int)(it.b % S);
            const uint32_t gen = (uint32_t)(it.b / S);
            const uint32_t* p = it.kind == 1 ? b_done + slot : a_done + slot;
            const uint32_t target = it.kind == 1 ? gen * (uint32_t)G::TB : (gen + 1) * (uint32_t)G::TA;
            return block ? counter_wait_bounded(p, target) : ld_acquire_u32(p) >= target;
        };
        bool failed = false;
        uint32_t next_ticket = atomicAdd(ticket, 1u);
        int64_t q = 0;
        for (;; ++q) {
            FusedItem nx = decode(next_ticket);
            while (nx.kind < 0) nx = decode(atomicAdd(ticket, 1u));
            if (nx.kind == 0) break;
            next_ticket = atomicAdd(ticket, 1u);  // the next claim's latency hides behind this item
            const int s = (int)(q % ST);
            if (q >= ST && !mbar_wait_bounded(&empty[s], (uint32_t)(((q - ST) / ST) & 1))) {
                failed = true;
                break;
            }
            // Items already issued finish without the loader (consumers compute them, the
            // storer stores and publishes them, flushing before it blocks), so blocking here
            // cannot close a cycle: every dependency is an earlier ticket.
            if (!ready(nx, true)) {
                failed = true;
                break;
            }
            s_item[s] = nx;
            fence_proxy_async_global();
            float2* dst = stage(s);
            if (nx.kind == 1) {
                mbar_arrive_expect_tx(&full[s], (uint32_t)(GA::K * GA::L * sizeof(float2)));
#pragma unroll
                for (int j = 0; j < GA::L / GA::LB; ++j)
                    tma_load_3d_hint(dst + j * GA::LB * GA::K, &ta_in, nx.idx * GA::K, j * GA::LB, (int)nx.b,
                                     &full[s], pol_stream);
            } else {
                mbar_arrive_expect_tx(&full[s], (uint32_t)(GB::K * GB::L * sizeof(float2)));
#pragma unroll
                for (int j = 0; j < GB::L / GB::LB; ++j)
                    tma_load_3d_hint(dst + j * GB::LB * GB::K, &tb_in, nx.idx * GB::K, j * GB::LB,
                                     (int)(nx.b % S), &full[s], pol_keep);
            }
            if (*s_abort) {
                ++q;
                failed = true;
                break;
            }
        }
        if (failed) {
            *s_abort = 1;
            atomicOr(&g_kernel_status, 2u);
        }
        // the end item, in the next stage once it is free
        const int s = (int)(q % ST);
        if (q < ST || mbar_wait_bounded(&empty[s], (uint32_t)(((q - ST) / ST) & 1))) {
            s_item[s] = FusedItem{0, 0, 0};
            mbar_arrive(&full[s]);
        }
        // loads this CTA started land before it leaves (bounded); item q - ST's stage holds the end item
        for (int64_t r = q - ST + 1 > 0 ? q - ST + 1 : 0; r < q; ++r)
            mbar_wait_bounded(&full[r % ST], (uint32_t)((r / ST) & 1));
        return;
    }
    if (tid == NC + 32) {
        // ================================================ storer
        const uint64_t pol_stream = policy_evict_first(), pol_keep = policy_evict_last();
        // phase-A slots whose row stores were committed but not yet published, oldest first
        int pend[4];
        int npend = 0;
        auto publish = [&](bool all) {  // all: every pending group; else all but the newest group
            if (npend == 0 || (!all && npend == 1)) return;
            if (all) bulk_wait<0>();
            else bulk_wait<1>();
            fence_proxy_async_global();
            const int n = all ? npend : npend - 1;
            for (int i = 0; i < n; ++i) red_release_add(a_done + pend[i], 1u);
            for (int i = n; i < npend; ++i) pend[i - n] = pend[i];
            npend -= n;
        };
        // wait for a phase; before blocking, publish everything pending (another CTA may wait on it)
        auto wait_phase = [&](uint64_t* bar, uint32_t par) -> bool {
            if (mbar_try_wait(bar, par)) return true;
            publish(true);
            return mbar_wait_bounded(bar, par);
        };
        for (int64_t q = 0;; ++q) {
            const int s = (int)(q % ST);
            const uint32_t par = (uint32_t)((q / ST) & 1);
            if (!wait_phase(&full[s], par)) {
                *s_abort = 1;
                break;
            }
            const FusedItem it = s_item[s];
            if (it.kind == 0) break;
            const int slot = (int)(it.b % S);
            if (it.kind == 2) red_release_add(b_done + slot, 1u);  // its tile has left the slot
            if (!wait_phase(&staged[s], par)) {
                *s_abort = 1;
                break;
            }
            float2* buf = stage(s);
            if (it.kind == 1) {
                float2* dst = a.scratch + (int64_t)slot * (G::N1 * G::N2) + (int64_t)(it.idx * GA::K) * G::N1;
#pragma unroll 1
                for (int r = 0; r < GA::K; ++r)
                    bulk_store_hint(dst + (int64_t)r * G::N1, buf + r * (GA::L + GA::RPAD),
                                    (uint32_t)(GA::L * sizeof(float2)), pol_keep);
                bulk_commit();
                pend[npend++] = slot;
            } else {
                const int c0 = it.idx * GB::K;
#pragma unroll
                for (int j = 0; j < GB::L / GB::LB; ++j)
                    tma_store_3d_hint(&tb_out, c0, j * GB::LB, (int)it.b, buf + j * GB::LB * GB::K, pol_stream);
                bulk_commit();
            }
            bulk_wait_read<0>();  // the stage may be refilled
            mbar_arrive(&empty[s]);
            publish(true);        // phase B of that transform may be waiting for these rows
        }
        publish(true);
        bulk_wait<0>();
        return;
    }
    if (tid >= NC) return;

    // ==================================================== consumers (a column pair per TF threads)
    const u64 zero = 0;
    const u64 sre = f2splat(a.scale), sim = f2splat(a.conj_out ? -a.scale : a.scale);
    const bool scaled = a.scale != 1.0f || a.conj_out;
    for (int64_t q = 0;; ++q) {
        const int s = (int)(q % ST);
        const bool ok = mbar_wait_bounded(&full[s], (uint32_t)((q / ST) & 1));
        // one decision for all consumers (the flag may change between their reads)
        const bool stop = group_sync_or<NC>(!ok || *s_abort);
        if (!ok) *s_abort = 1;
        const FusedItem cur = s_item[s];
        if (cur.kind == 0 || stop) break;
        float2* buf = stage(s);
        const float4* buf4 = reinterpret_cast<const float4*>(buf);
        if (cur.kind == 1) {
            // ---------------- phase A: column FFTs of N1, post-twiddle W_N^{k1 n2}, staged as rows
            constexpr int NP = G::NPA;
            const int p = tid % NP, t = tid / NP;  // columns 2p, 2p + 1 of the tile
            const uint32_t nA = (uint32_t)(cur.idx * GA::K + 2 * p), nB = nA + 1;
            CPair tb{};
            if constexpr (GA::COLTW) {
#pragma unroll
                for (int j = 0; j < GA::CPT; ++j) {
                    const int m = t + j * GA::TF;
                    const uint32_t e = static_cast<uint32_t>(m * GA::TF);
                    if (m < 16) coltw[m * NP + p] = cp_make(twiddle(e * nA), twiddle(e * nB));
                }
                tb = cp_make(twiddle(static_cast<uint32_t>(t) * nA), twiddle(static_cast<uint32_t>(t) * nB));
            }
            CPair v[16];
#pragma unroll
            for (int m = 0; m < 16; ++m) {
                const float4 x = buf4[(t + m * GA::TF) * NP + p];
                v[m] = CPair{f2pack(x.x, x.z), f2pack(x.y, x.w)};
                if (a.conj_in) v[m].im = f2sub(zero, v[m].im);
            }
            group_sync<NC>();  // the tile is now the exchange area; the column factors are published
            pair_passes<LA, 0, GA::TF, NP, NC>(v, t, reinterpret_cast<ulonglong2*>(buf) + p, twA);
#pragma unroll
            for (int m = 0; m < 16; ++m) {
                const uint32_t k = static_cast<uint32_t>(t + m * GA::TF);
                CPair w;
                if constexpr (GA::COLTW) w = cp_mul(tb, coltw[m * NP + p]);
                else w = cp_make(twiddle(k * nA), twiddle(k * nB));
                const CPair y = cp_mul(v[m], w);
                buf[(2 * p) * (GA::L + GA::RPAD) + k] = cp_first(y);
                buf[(2 * p + 1) * (GA::L + GA::RPAD) + k] = cp_second(y);
            }
        } else {
            // ---------------- phase B: column FFTs of N2 over the slot, epilogue, staged as columns of X
            constexpr int NP = G::NPB;
            const int p = tid % NP, t = tid / NP;
            CPair v[16];
#pragma unroll
            for (int m = 0; m < 16; ++m) {
                const float4 x = buf4[(t + m * GB::TF) * NP + p];
                v[m] = CPair{f2pack(x.x, x.z), f2pack(x.y, x.w)};
            }
            group_sync<NC>();
            pair_passes<LB, 0, GB::TF, NP, NC>(v, t, reinterpret_cast<ulonglong2*>(buf) + p, twB);
            float4* out4 = reinterpret_cast<float4*>(buf);
#pragma unroll
            for (int m = 0; m < 16; ++m) {
                CPair y = v[m];
                if (scaled) y = CPair{f2mul(y.re, sre), f2mul(y.im, sim)};
                out4[(t + m * GB::TF) * NP + p] = make_float4(f2lo(y.re), f2lo(y.im), f2hi(y.re), f2hi(y.im));
            }
        }
        fence_proxy_async_smem();
        group_sync<NC>();  // staged; also: every consumer has read s_item[s] and the column factors
        if (tid == 0) mbar_arrive(&staged[s]);
    }
}

// ---- host side ----

template <int LA, int LB>
static cudaError_t launch_fused_t(const float2* in, float2* out, const FusedArgs& a0, cudaStream_t s) {
    using G = FusedGeo<LA, LB>;
    using GA = typename G::GA;
    using GB = typename G::GB;
    constexpr size_t kSmemCap = 227 * 1024;
    static std::atomic<int> blocks_per_sm[64][kTwClasses];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const uint64_t N1 = G::N1, N2 = G::N2, N = N1 * N2;
    CUtensorMap ta_in, tb_in, tb_out;
    // x as [b][n1][n2]: sub-FFT (column) index n2 fastest
    if (!encode_map_3d(&ta_in, in, N2, N1, (uint64_t)a0.batch, N2 * 8, N * 8, GA::K, GA::LB)) return cudaErrorNotSupported;
    // slots as [slot][n2][k1]: phase B's sub-FFT index k1 fastest, element n2
    if (!encode_map_3d(&tb_in, a0.scratch, N1, N2, (uint64_t)a0.slots, N1 * 8, N * 8, GB::K, GB::LB))
        return cudaErrorNotSupported;
    // X as [b][k2][k1]
    if (!encode_map_3d(&tb_out, out, N1, N2, (uint64_t)a0.batch, N1 * 8, N * 8, GB::K, GB::LB))
        return cudaErrorNotSupported;
    FusedArgs a = a0;
    PassArgs pa{};
    pa.tw = a.tw;
    pa.tw_mode = 2;
    int cls = 0;
    choose_tw_staging(pa, G::SMEM, kSmemCap, cls);
    a.tw_smem_entries = pa.tw_smem_entries;
    a.tw_smem_levels = pa.tw_smem_levels;
    auto kern = k_fused_fft<LA, LB>;
    int sms = 0, nb = 0;
    e = device_sm_count(dev, &sms);
    if (e == cudaSuccess) e = cached_occupancy(blocks_per_sm[dev][cls], kern, G::THREADS, G::SMEM + tw_class_bytes(cls),
                                               kSmemCap, &nb);
    if (e != cudaSuccess) return e;
    const int64_t items = a.batch * (G::TA + G::TB);
    int64_t grid = (int64_t)nb * sms;
    if (grid > items) grid = items;
    if (grid < 1) grid = 1;
    const size_t smem = G::SMEM + (size_t)a.tw_smem_entries * sizeof(float2);
    e = cudaMemsetAsync(a.counters, 0, sizeof(uint32_t) * (1 + 2 * (size_t)a.slots), s);
    if (e != cudaSuccess) return e;
    return launch_maybe_pdl(kern, (unsigned)grid, G::THREADS, smem, s, 0, ta_in, tb_in, tb_out, a);
}

// Scratch ring sizing, in tickets (the tiles of one transform form one round
// of TA + TB tickets): phase-B tiles come up kLagTickets after their
// transform's phase-A tiles, and a slot is reused kSlackTickets after its
// phase-B tiles came up, so S > D.  A ticket stands for 16 KiB of ring with
// 128 consumers and 32 KiB with 256 (N >= 2^17), so the ring is 48 MiB either
// way.  Measured on B200 (N = 2^16, B = 8192; N = 2^13, B = 65536): lag/slack
// 768/768 leaves the loaders blocked on dependencies (2.96 ms), 1024/1024
// 2.69 ms, 1536/1536 2.56 ms (a 48 MiB ring), 2048/2048 2.82 ms and 3072/1536
// 2.98 ms -- the larger rings no longer stay in L2.  After the kernel got
// faster (shared-memory accesses as such, sleeping waits) the optimum moved
// for long runs: N = 2^16, B = 8192 (4 GiB) takes 2.29 ms at 1280/1280 (a
// 40 MiB ring) against 2.36 ms at 1536/1536 (1408/1408 2.30, 1152/1152 2.33,
// 1280/1024 2.31, 1280/1536 2.34, 1152/1280 2.34, 1024/1024 2.40, 1792/1792
// 2.53), while a 128 MiB batch (B N = 2^24) stays
// faster at 1536/1536 (N = 2^13: 99-102 against 105 us; N = 2^16: 97 against
// 103 us).  Batches of 2^26 points (512 MiB) or more use the smaller ring.
constexpr int kLagTickets = 1536, kSlackTickets = 1536;
constexpr int kLagTicketsLong = 1280, kSlackTicketsLong = 1280;
constexpr int64_t kLongRunPoints = int64_t(1) << 26;

inline void fused_round(int log2n, int* round_len, int* ticket_kib) {
    switch (log2n) {
        case 13: *round_len = FusedGeo<7, 6>::TA + FusedGeo<7, 6>::TB; break;
        case 14: *round_len = FusedGeo<7, 7>::TA + FusedGeo<7, 7>::TB; break;
        case 15: *round_len = FusedGeo<8, 7>::TA + FusedGeo<8, 7>::TB; break;
        case 16: *round_len = FusedGeo<8, 8>::TA + FusedGeo<8, 8>::TB; break;
        case 17: *round_len = FusedGeo<9, 8>::TA + FusedGeo<9, 8>::TB; break;
        case 18: *round_len = FusedGeo<9, 9>::TA + FusedGeo<9, 9>::TB; break;
        case 19: *round_len = FusedGeo<10, 9>::TA + FusedGeo<10, 9>::TB; break;
        default: *round_len = FusedGeo<10, 10>::TA + FusedGeo<10, 10>::TB; break;
    }
    *ticket_kib = (int)(((int64_t(8) << log2n) / 1024) / *round_len);
}

inline void fused_ring(int64_t n, int64_t batch, int* slots, int* lag) {
    int log2n = 0;
    while ((int64_t(1) << log2n) < n) ++log2n;
    int rl = 0, kib = 16;
    fused_round(log2n, &rl, &kib);
    const bool long_run = n * batch >= kLongRunPoints;
    const int lag0 = long_run ? kLagTicketsLong : kLagTickets;
    const int slack0 = long_run ? kSlackTicketsLong : kSlackTickets;
    // the same ring bytes whatever the ticket size
    const int lag_t = kib > 16 ? lag0 * 16 / kib : lag0;
    const int slack_t = kib > 16 ? slack0 * 16 / kib : slack0;
    const int D = (lag_t + rl - 1) / rl;
    const int64_t want = D + (slack_t + rl - 1) / rl;
    *lag = D;
    *slots = (int)(batch < want ? batch : want);  // batch <= S: no slot is reused
}

bool fused_supported(int log2n) { return log2n >= 13 && log2n <= 20; }

size_t fused_workspace_bytes(int64_t n, int64_t batch) {
    int slots = 0, lag = 0;
    fused_ring(n, batch, &slots, &lag);
    return (size_t)slots * (size_t)n * sizeof(float2) + 256 + sizeof(uint32_t) * (1 + 2 * (size_t)slots);
}

cudaError_t launch_fused_fft(int log2n, const float2* in, float2* out, void* workspace, const FusedArgs& a0,
                             cudaStream_t s) {
    FusedArgs a = a0;
    const int64_t n = int64_t(1) << log2n;
    fused_ring(n, a.batch, &a.slots, &a.lag);
    a.scratch = static_cast<float2*>(workspace);
    a.counters = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(workspace) +
                                             (size_t)a.slots * (size_t)n * sizeof(float2) + 128);
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(workspace)) & 15)
        return cudaErrorNotSupported;
    switch (log2n) {
        case 13: return launch_fused_t<7, 6>(in, out, a, s);
        case 14: return launch_fused_t<7, 7>(in, out, a, s);
        case 15: return launch_fused_t<8, 7>(in, out, a, s);
        case 16: return launch_fused_t<8, 8>(in, out, a, s);
        case 17: return launch_fused_t<9, 8>(in, out, a, s);
        case 18: return launch_fused_t<9, 9>(in, out, a, s);
        case 19: return launch_fused_t<10, 9>(in, out, a, s);
        case 20: return launch_fused_t<10, 10>(in, out, a, s);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace bfft
