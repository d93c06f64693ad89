// bfft_tc.cuh -- 16-point DFTs of contiguous rows on the tensor cores
// (tcgen05.mma, kind::tf32), 3xTF32 split precision.
//
// The B200 form of the reference's dense-dot core (src/xpu/kernels.py:487-532,
// local_matrix_kernel: a tile of rows times the tile's DFT matrix with FP32
// dot products).  A row of 16 complex64 is 32 floats in interleaved order, so
// a tile of 128 rows is the K-major matrix A[128 x 32] as it lies in memory,
// and its DFT is D = A B^T with the real 32 x 32 matrix
//     B[2i][2j] = cos t,  B[2i][2j+1] = sin t,  B[2i+1][2j] = -sin t,
//     B[2i+1][2j+1] = cos t,   t = 2 pi i j / 16
// (X_i = sum_j x_j (cos t - i sin t)).  TF32 keeps 11 significant bits, so
// FP32 accuracy needs the split A = Ah + Al, B = Bh + Bl (Ah: A with its low
// 13 mantissa bits cleared, Al = A - Ah exactly) and D = Al Bh + Ah Bl + Ah Bh,
// three products of four K = 8 MMAs each accumulated in tensor memory.
//
// One tile per CTA at a time: a TMA load of the 128 x 128-byte tile
// (SWIZZLE_128B, the canonical K-major layout of the MMA), the split by all
// threads into Ah / Al (same offsets, so the swizzle is kept), one thread
// issues the 12 MMAs and commits them to an mbarrier, every warp reads its 32
// rows of D from tensor memory (tcgen05.ld 32x32b.x32) into the staging
// buffer, and a TMA store writes the tile.  Five CTAs share an SM.  Waits are
// bounded (kWaitLimitNs); tensor memory is freed on every exit path.
#pragma once

namespace bfft {

struct TcGeo {
    static constexpr int M = 128, N = 32, K = 32;  // rows per tile, real outputs, real inputs
    static constexpr int THREADS = 128;
    static constexpr int TILE = M * K * 4;         // bytes of a 128 x 32 fp32 tile
    static constexpr int BMAT = N * K * 4;         // bytes of the 32 x 32 matrix
    static constexpr int TMEM_COLS = 32;
    // tile (landing, then Ah, then output staging), Al, Bh, Bl -- each 1024-byte
    // aligned (swizzle atoms) -- and the control words; five CTAs share an SM
    static constexpr size_t SMEM = 1024 + 2 * TILE + 2 * BMAT + 64;
};

__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
    // K-major, 128-byte swizzle: rows of 128 bytes, 8-row atoms 1024 bytes apart
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3fff);          // start address
    d |= (uint64_t)1 << 16;                               // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)((1024 >> 4) & 0x3fff) << 32;          // stride byte offset: 8 rows x 128 bytes
    d |= (uint64_t)1 << 46;                               // descriptor version (sm100)
    d |= (uint64_t)2 << 61;                               // layout: SWIZZLE_128B
    return d;
}

// kind::tf32, D in fp32, A and B K-major, M = 128, N = 32
constexpr uint32_t kTcInstrDesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(TcGeo::N >> 3) << 17) |
                                  ((uint32_t)(TcGeo::M >> 4) << 24);

__device__ __forceinline__ void tc_mma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kTcInstrDesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int c0, int c1, const void* src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(c0), "r"(c1), "r"(smem_u32(src))
                 : "memory");
}

// byte offset of (row r, 16-byte chunk c) in a 128-byte-swizzled tile
__device__ __forceinline__ int sw128(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// Nearest TF32 value (10 fraction bits; ties away from zero) of a finite float:
// the split x = tf32(x) + tf32(x - tf32(x)) + e has |e| <= 2^-22 |x|.
__host__ __device__ __forceinline__ float tf32_nearest(float x) {
#ifdef __CUDA_ARCH__
    return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xffffe000u);
#else
    uint32_t u;
    memcpy(&u, &x, 4);
    u = (u + 0x1000u) & 0xffffe000u;
    float r;
    memcpy(&r, &u, 4);
    return r;
#endif
}

__global__ void __launch_bounds__(TcGeo::THREADS)
    k_tc_dft16_rows(const __grid_constant__ CUtensorMap tin, const __grid_constant__ CUtensorMap tout,
                    int64_t rows, float scale, int conj_in, int conj_out) {
    using G = TcGeo;
    extern __shared__ unsigned char smem_raw[];
    unsigned char* base = align_smem<1024>(smem_raw);
    unsigned char* buf = base;  // TMA landing tile, then Ah in place, then the output staging
    unsigned char* al = base + G::TILE;
    unsigned char* bh = base + 2 * G::TILE;
    unsigned char* bl = bh + G::BMAT;
    uint64_t* bars = reinterpret_cast<uint64_t*>(bl + G::BMAT);  // [0] tile landed, [1] MMAs done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t ntiles = (rows + G::M - 1) / G::M;

    if (warp == 0) {  // tensor memory for D: 128 lanes x 32 fp32 columns
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(G::TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // the DFT-16 matrix, split into TF32 high and low parts, in the swizzled K-major layout
    for (int e = tid; e < G::N * G::K; e += G::THREADS) {
        const int n = e / G::K, k = e % G::K;
        const int i = n >> 1, j = k >> 1;
        double sn, cs;
        sincospi(2.0 * (double)((i * j) & 15) / 16.0, &sn, &cs);
        const double v = (n & 1) ? ((k & 1) ? cs : -sn) : ((k & 1) ? sn : cs);
        const float fh = tf32_nearest((float)v);
        const float fl = tf32_nearest((float)(v - (double)fh));
        const int off = sw128(n, k >> 2) + (k & 3) * 4;
        *reinterpret_cast<float*>(bh + off) = fh;
        *reinterpret_cast<float*>(bl + off) = fl;
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int it = 0;
    for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++it) {
        const uint32_t par = (uint32_t)(it & 1);
        if (tid == 0) {
            bulk_wait_read<0>();  // the previous tile's store has read the buffer
            mbar_arrive_expect_tx(&bars[0], (uint32_t)G::TILE);
            tma_load_2d(buf, &tin, 0, (int)(tile * G::M), &bars[0]);
        }
        if (__syncthreads_or(!mbar_wait_bounded(&bars[0], par))) break;
        // split into TF32 high (in place) and low parts; same byte offsets, so the swizzle is kept
#pragma unroll
        for (int q = 0; q < G::TILE / 16 / G::THREADS; ++q) {
            const int off = (tid + q * G::THREADS) * 16;
            float4 x = *reinterpret_cast<const float4*>(buf + off);
            if (conj_in) {  // odd floats are imaginary parts
                x.y = -x.y;
                x.w = -x.w;
            }
            const float4 h = make_float4(tf32_nearest(x.x), tf32_nearest(x.y), tf32_nearest(x.z), tf32_nearest(x.w));
            const float4 l = make_float4(tf32_nearest(x.x - h.x), tf32_nearest(x.y - h.y), tf32_nearest(x.z - h.z),
                                         tf32_nearest(x.w - h.w));
            *reinterpret_cast<float4*>(buf + off) = h;
            *reinterpret_cast<float4*>(al + off) = l;
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t a_hi = smem_u32(buf), a_lo = smem_u32(al), b_hi = smem_u32(bh), b_lo = smem_u32(bl);
            // small products first: Al Bh, Ah Bl, then Ah Bh; K = 32 as four K = 8 (32-byte) steps
            const uint32_t as[3] = {a_lo, a_hi, a_hi}, bs[3] = {b_hi, b_lo, b_hi};
#pragma unroll
            for (int p = 0; p < 3; ++p)
#pragma unroll
                for (int ks = 0; ks < G::K / 8; ++ks)
                    tc_mma_tf32(tmem, umma_desc_sw128(as[p] + ks * 32), umma_desc_sw128(bs[p] + ks * 32),
                                (p | ks) ? 1u : 0u);
            tc_commit(&bars[1]);
        }
        const bool bad = __syncthreads_or(!mbar_wait_bounded(&bars[1], par));
        tc_fence_after();
        if (bad) break;
        // D rows of this warp: tensor-memory lanes 32 w .. 32 w + 31, columns 0..31
        uint32_t d[32];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
            "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
            : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3]), "=r"(d[4]), "=r"(d[5]), "=r"(d[6]), "=r"(d[7]),
              "=r"(d[8]), "=r"(d[9]), "=r"(d[10]), "=r"(d[11]), "=r"(d[12]), "=r"(d[13]), "=r"(d[14]), "=r"(d[15]),
              "=r"(d[16]), "=r"(d[17]), "=r"(d[18]), "=r"(d[19]), "=r"(d[20]), "=r"(d[21]), "=r"(d[22]), "=r"(d[23]),
              "=r"(d[24]), "=r"(d[25]), "=r"(d[26]), "=r"(d[27]), "=r"(d[28]), "=r"(d[29]), "=r"(d[30]), "=r"(d[31])
            : "r"(tmem + ((uint32_t)(warp * 32) << 16)));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const int r = warp * 32 + lane;  // this thread's row of the tile
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            float4 o = make_float4(__uint_as_float(d[4 * c]), __uint_as_float(d[4 * c + 1]),
                                   __uint_as_float(d[4 * c + 2]), __uint_as_float(d[4 * c + 3]));
            if (conj_out) {
                o.y = -o.y;
                o.w = -o.w;
            }
            o.x *= scale;
            o.y *= scale;
            o.z *= scale;
            o.w *= scale;
            *reinterpret_cast<float4*>(buf + sw128(r, c)) = o;
        }
        fence_proxy_async_smem();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tma_store_2d(&tout, 0, (int)(tile * G::M), buf);
            bulk_commit();
        }
    }
    // a wait that ran out has set status bit 0 (mbar_wait_bounded)
    if (tid == 0) bulk_wait<0>();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(G::TMEM_COLS) : "memory");
    }
}

// 2-D map of the rows as fp32 [rows][32 floats], 128-byte swizzled boxes of 128 rows
static bool encode_rows16_map(CUtensorMap* m, const void* ptr, uint64_t rows) {
    EncodeTiledFn enc = tensor_map_encoder();
    if (!enc) return false;
    cuuint64_t dims[2] = {32, rows};
    cuuint64_t strides[1] = {128};
    cuuint32_t box[2] = {32, (cuuint32_t)TcGeo::M};
    cuuint32_t estr[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_tc_dft16_rows(const float2* in, float2* out, int64_t rows, float scale, int conj_in, int conj_out,
                                 cudaStream_t s) {
    if (rows < 1 || rows > (int64_t)0x7fffffff) return cudaErrorInvalidValue;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) return cudaErrorNotSupported;
    static std::atomic<int> blocks_per_sm[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    CUtensorMap tin, tout;
    if (!encode_rows16_map(&tin, in, (uint64_t)rows) || !encode_rows16_map(&tout, out, (uint64_t)rows))
        return cudaErrorNotSupported;
    int sms = 0, nb = 0;
    e = device_sm_count(dev, &sms);
    // CTAs per SM from the SM's shared memory (the occupancy query answered 1
    // for this kernel on B200 while five fit: the grid then covered one CTA
    // per SM); the whole carveout goes to shared memory
    if (e == cudaSuccess)
        e = cached_value(g_occ_mu, blocks_per_sm[dev], &nb, [&](int* v) {
            int per_sm = 0, reserved = 0;
            cudaError_t r = cudaFuncSetAttribute(k_tc_dft16_rows, cudaFuncAttributePreferredSharedMemoryCarveout,
                                                 (int)cudaSharedmemCarveoutMaxShared);
            if (r == cudaSuccess)
                r = cudaFuncSetAttribute(k_tc_dft16_rows, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)TcGeo::SMEM);
            if (r == cudaSuccess)
                r = cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
            if (r == cudaSuccess) r = cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, dev);
            if (r != cudaSuccess) return r;
            int k = per_sm / (int)(TcGeo::SMEM + (size_t)reserved);
            *v = k < 1 ? 1 : (k > 8 ? 8 : k);
            return cudaSuccess;
        });
    if (e != cudaSuccess) return e;
    const int64_t ntiles = (rows + TcGeo::M - 1) / TcGeo::M;
    int64_t grid = (int64_t)nb * sms;
    if (grid > ntiles) grid = ntiles;
    if (grid < 1) grid = 1;
    k_tc_dft16_rows<<<(unsigned)grid, TcGeo::THREADS, TcGeo::SMEM, s>>>(tin, tout, rows, scale, conj_in, conj_out);
    return cudaGetLastError();
}

}  // namespace bfft
