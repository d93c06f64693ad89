// bfft_rows_pair.cuh -- whole rows of 256..4096 points in one HBM round trip:
// a warp-specialised persistent kernel with paired (FP32x2) consumers.
//
// Included by bfft_kernels.cu after bfft_fused.cuh (it uses the bulk-copy and
// mbarrier helpers of bfft_pass_tma.cuh and the pair arithmetic, pair
// twiddle tables and pair Stockham passes of bfft_pair.cuh).
//
// A tile is K = 2 NP rows.  Its rows land by bulk copies in a [row][element]
// stage (one copy when the tile's rows are adjacent and the stage unpadded,
// else one per row); consumer thread (t, p) then takes element t + m TF
// (m < 16) of rows 2p and 2p + 1 as one pair, so every butterfly and twiddle
// instruction serves two rows (the twiddles of a Stockham pass depend only on
// the element index, hence are the same for both rows of a pair).  The stage
// then serves as the pair exchange area and, after the last pass, as the
// [row][element] staging of the outputs for the bulk copies out.
//
// Warps: the consumer warps (threads 0 .. NC-1) compute and meet only at
// named barrier 1; lane 0 of the next warp (the loader) starts the loads;
// lane 0 of the last warp (the storer) issues the stores.  Three stages per
// CTA chained by mbarriers:
//   full[s]   loader    -> consumers: the tile landed;
//   staged[s] consumers -> storer: the outputs are staged;
//   empty[s]  storer    -> loader: the stores have read the stage.
// Tiles go to CTAs round-robin (tile = blockIdx.x + q gridDim.x), so every
// role knows the q-th tile without communication.  Each wait is bounded
// (kWaitLimitNs); an expired wait sets bit 0 of bfft_device_status, raises
// the CTA's abort flag, and every role then leaves after the copies it
// started have landed.
#pragma once

namespace bfft {

template <int LOG2L>
struct RowsPairGeo {
    static constexpr int L = 1 << LOG2L;
    static constexpr int TF = L / 16;  // threads sharing a row pair
    // 4096-point rows: a pair is 8192 points = 256 threads of 32 points each
    static constexpr int CONSUMERS = L > 2048 ? 256 : 128;
    static constexpr int NP = CONSUMERS / TF;  // row pairs per tile
    static constexpr int K = 2 * NP;           // rows per tile
    // Row stride of the landing / output staging, in elements.  Lane (t, p) of
    // a warp reads element t + m TF of row 2p: with NP >= 4 the NP rows of a
    // warp would meet on the same banks, so pad them apart (16-byte multiples,
    // so every row start stays a legal bulk-copy address).
    static constexpr int RS = NP >= 8 ? L + 2 : NP >= 4 ? L + 4 : L;
    static constexpr int SB = ((K * RS * 8) + 127) / 128 * 128;
    static constexpr int STAGES = 3;
    static constexpr int THREADS = CONSUMERS + 64;  // + the loader and the storer warps
    static constexpr int MINB = CONSUMERS > 128 ? 1 : 2;
    static constexpr int CTRL = 128;
    static constexpr size_t SMEM = 128 + (size_t)STAGES * SB + CTRL + (size_t)tw_total(LOG2L) * sizeof(CPair);
    static_assert(LOG2L >= 8 && LOG2L <= 12 && NP >= 1, "row pair geometry");
    static_assert(L * NP * 16 <= SB, "the pair exchange area fits in a stage");
    static_assert((RS * 8) % 16 == 0, "16-byte aligned row starts");
    static_assert(SMEM * MINB <= 227 * 1024, "stages");
};

template <int LOG2L>
__global__ void __launch_bounds__(RowsPairGeo<LOG2L>::THREADS, RowsPairGeo<LOG2L>::MINB)
    k_rows_pair(const float2* __restrict__ in, float2* __restrict__ out, PassArgs a, int in_contig,
                int out_contig) {
    using G = RowsPairGeo<LOG2L>;
    constexpr int ST = G::STAGES;
    constexpr int NC = G::CONSUMERS;
    static_assert(8 * 3 * ST + sizeof(int) <= G::CTRL, "control block");
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = align_smem<128>(smem_raw);
    unsigned char* ctrl = base + ST * G::SB;
    uint64_t* full = reinterpret_cast<uint64_t*>(ctrl);
    uint64_t* staged = full + ST;
    uint64_t* empty = staged + ST;
    volatile int* s_abort = reinterpret_cast<volatile int*>(empty + ST);
    CPair* tw = reinterpret_cast<CPair*>(ctrl + G::CTRL);
    auto stage = [&](int s) { return reinterpret_cast<float2*>(base + s * G::SB); };

    const int tid = threadIdx.x;
    const int64_t ntiles = (a.nsub + G::K - 1) / G::K;
    const int64_t imask = (int64_t(1) << a.inner_log2) - 1;
    const uint32_t row_bytes = static_cast<uint32_t>(G::L * sizeof(float2));
    auto rows_of = [&](int64_t tl) -> int {
        const int64_t left = a.nsub - tl * G::K;
        return static_cast<int>(left < G::K ? left : G::K);
    };
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
    fill_pair_twiddles<LOG2L>(tw);
    __syncthreads();  // the last CTA-wide barrier: the warps part ways here

    if (tid == NC) {
        // ================================================ loader
        griddep_wait();  // every read and write of the flow's buffers follows this
        int64_t q = 0;
        bool failed = false;
        for (int64_t tl = blockIdx.x; tl < ntiles; tl += gridDim.x, ++q) {
            const int s = (int)(q % ST);
            if (q >= ST && !mbar_wait_bounded(&empty[s], (uint32_t)(((q - ST) / ST) & 1))) {
                failed = true;
                break;
            }
            if (*s_abort) {
                failed = true;
                break;
            }
            const int rows = rows_of(tl);
            const int64_t f0 = tl * G::K;
            float2* dst = stage(s);
            mbar_arrive_expect_tx(&full[s], row_bytes * (uint32_t)rows);
            if (in_contig) {
                bulk_load(dst, row_in(f0), row_bytes * (uint32_t)rows, &full[s]);
            } else {
#pragma unroll 1
                for (int r = 0; r < rows; ++r) bulk_load(dst + r * G::RS, row_in(f0 + r), row_bytes, &full[s]);
            }
        }
        griddep_launch_dependents();  // this CTA's last loads are issued
        if (failed) *s_abort = 1;  // consumers waiting for an item never issued give up at their bound
        // the loads this CTA started land before it leaves (bounded)
        for (int64_t r = q - ST > 0 ? q - ST : 0; r < q; ++r)
            mbar_wait_bounded(&full[r % ST], (uint32_t)((r / ST) & 1));
        return;
    }
    if (tid == NC + 32) {
        // ================================================ storer
        griddep_wait();
        int64_t q = 0;
        for (int64_t tl = blockIdx.x; tl < ntiles; tl += gridDim.x, ++q) {
            const int s = (int)(q % ST);
            if (!mbar_wait_bounded(&staged[s], (uint32_t)((q / ST) & 1)) || *s_abort) {
                *s_abort = 1;
                break;
            }
            const int rows = rows_of(tl);
            const int64_t f0 = tl * G::K;
            const float2* buf = stage(s);
            if (out_contig) {
                bulk_store(row_out(f0), buf, row_bytes * (uint32_t)rows);
            } else {
#pragma unroll 1
                for (int r = 0; r < rows; ++r) bulk_store(row_out(f0 + r), buf + r * G::RS, row_bytes);
            }
            bulk_commit();
            bulk_wait_read<0>();  // the stage may be refilled
            mbar_arrive(&empty[s]);
        }
        bulk_wait<0>();
        return;
    }
    if (tid >= NC) return;

    // ==================================================== consumers (a row pair per TF threads)
    constexpr int NP = G::NP;
    const int p = tid % NP, t = tid / NP;  // rows 2p, 2p + 1 of the tile, elements t + m TF
    const u64 zero = 0;
    const u64 sre = f2splat(a.scale), sim = f2splat(a.conj_out ? -a.scale : a.scale);
    const bool scaled = a.scale != 1.0f || a.conj_out;
    int64_t q = 0;
    for (int64_t tl = blockIdx.x; tl < ntiles; tl += gridDim.x, ++q) {
        const int s = (int)(q % ST);
        const bool ok = mbar_wait_bounded(&full[s], (uint32_t)((q / ST) & 1));
        // one decision for all consumers (the flag may change between their reads)
        if (group_sync_or<NC>(!ok || *s_abort)) {
            *s_abort = 1;
            break;
        }
        float2* buf = stage(s);
        const float2* ra = buf + (2 * p) * G::RS;
        const float2* rb = ra + G::RS;
        CPair v[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            const float2 x = ra[t + m * G::TF], y = rb[t + m * G::TF];
            v[m] = CPair{f2pack(x.x, y.x), f2pack(x.y, y.y)};
            if (a.conj_in) v[m].im = f2sub(zero, v[m].im);
        }
        group_sync<NC>();  // the tile is now the exchange area
        pair_passes<LOG2L, 0, G::TF, NP, NC>(v, t, reinterpret_cast<ulonglong2*>(buf) + p, tw);
        // pair_passes ends with every exchange read done (a barrier after the last one)
        float2* wa = buf + (2 * p) * G::RS;
        float2* wb = wa + G::RS;
#pragma unroll
        for (int m = 0; m < 16; ++m) {
            CPair y = v[m];
            if (scaled) y = CPair{f2mul(y.re, sre), f2mul(y.im, sim)};
            wa[t + m * G::TF] = cp_first(y);
            wb[t + m * G::TF] = cp_second(y);
        }
        fence_proxy_async_smem();
        group_sync<NC>();
        if (tid == 0) mbar_arrive(&staged[s]);
    }
}

// ---- host side ----

template <int LOG2L>
static cudaError_t launch_rows_pair_t(const float2* in, float2* out, const PassArgs& a, int in_contig,
                                      int out_contig, cudaStream_t s) {
    using G = RowsPairGeo<LOG2L>;
    auto kern = k_rows_pair<LOG2L>;
    constexpr size_t kSmemCap = 227 * 1024;
    static std::atomic<int> blocks_per_sm[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    int sms = 0, nb = 0;
    e = device_sm_count(dev, &sms);
    if (e == cudaSuccess) e = cached_occupancy(blocks_per_sm[dev], kern, G::THREADS, G::SMEM, kSmemCap, &nb);
    if (e != cudaSuccess) return e;
    const int64_t ntiles = (a.nsub + G::K - 1) / G::K;
    int64_t grid = (int64_t)nb * sms;
    if (grid > ntiles) grid = ntiles;
    if (grid < 1) grid = 1;
    // a single copy per tile needs the unpadded stage
    const int ic = in_contig && G::RS == G::L ? 1 : 0, oc = out_contig && G::RS == G::L ? 1 : 0;
    return launch_maybe_pdl(kern, (unsigned)grid, G::THREADS, G::SMEM, s, a.pdl, in, out, a, ic, oc);
}

// Whole rows of 256, 1024, 2048 or 4096 points with no W_N twiddle, every row
// start 16-byte aligned; cudaErrorNotSupported for any other shape (the caller
// then runs the single-row-mapping pass).  512-point rows (radix 16, 16, 2)
// measured faster on the single-row-mapping pass (B200, B N = 2^24: 61.3
// against 66.3 us) and stay there.
static cudaError_t launch_rows_pair(int log2l, const float2* in, float2* out, const PassArgs& a, cudaStream_t s) {
    if (log2l < 8 || log2l > 12 || log2l == 9 || a.tw_mode != 0) return cudaErrorNotSupported;
    const int64_t L = int64_t(1) << log2l;
    const int64_t inner = int64_t(1) << a.inner_log2;
    if (((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) || a.in_stride != 1 ||
        a.out_stride != 1 || a.in_elem_bitrev || a.out_elem_bitrev)
        return cudaErrorNotSupported;
    if ((a.in_outer & 1) || (inner > 1 && (a.in_inner & 1)) || (a.out_outer & 1) || (inner > 1 && (a.out_inner & 1)))
        return cudaErrorNotSupported;
    int k = 0;
    switch (log2l) {
        case 8: k = RowsPairGeo<8>::K; break;
        case 10: k = RowsPairGeo<10>::K; break;
        case 11: k = RowsPairGeo<11>::K; break;
        default: k = RowsPairGeo<12>::K; break;
    }
    // a tile's rows are adjacent in memory: one copy per tile
    auto contiguous = [&](int64_t outer, int64_t inner_stride, int base_bits) {
        if (inner == 1) return outer == L;
        return !base_bits && inner_stride == L && outer == inner * L && inner % k == 0;
    };
    const int ic = contiguous(a.in_outer, a.in_inner, a.in_base_bits) ? 1 : 0;
    const int oc = contiguous(a.out_outer, a.out_inner, a.out_base_bits) ? 1 : 0;
    switch (log2l) {
        case 8: return launch_rows_pair_t<8>(in, out, a, ic, oc, s);
        case 10: return launch_rows_pair_t<10>(in, out, a, ic, oc, s);
        case 11: return launch_rows_pair_t<11>(in, out, a, ic, oc, s);
        default: return launch_rows_pair_t<12>(in, out, a, ic, oc, s);
    }
}

}  // namespace bfft
