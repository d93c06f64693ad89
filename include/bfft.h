/*
 * bfft.h -- C ABI of the B200 FFT library (libbfft.so).
 *
 * The drop-in boundary for the reference's plan/operator API
 * (src/xpu/entry.py:292 plan_fft, :501 execute_fft_plan, src/xpu/runner.py
 * runner functions).  The reference has no C ABI of its own
 * (docs/reference/api.md:40): its Python layer calls Triton kernels directly.
 * Here the Python host layer (kunlunxin-fft_b200/bfft) resolves a plan on the
 * host exactly like the reference and then calls these entry points with
 * plain device pointers, sizes and a CUDA stream; an FFI from any other host
 * language would bind the same symbols.
 *
 * Conventions
 *   - Data is interleaved complex64 (float re, float im), batch-major (B, N),
 *     contiguous; R2C input / C2R output are float32 (B, N).
 *   - All pointers are device pointers on the plan's device; `stream` is a
 *     cudaStream_t (NULL = legacy default stream).  Nothing synchronises the
 *     host: calls enqueue work on `stream` and return.
 *   - Every entry point returns a bfft_status; 0 is success.  On failure
 *     bfft_last_error() returns a thread-local message.  Shape / value errors
 *     are detected before any launch.
 *   - Input and output must not overlap.
 */
#ifndef BFFT_H
#define BFFT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BFFT_API_VERSION 1

#if defined(__GNUC__)
#define BFFT_EXPORT __attribute__((visibility("default")))
#else
#define BFFT_EXPORT
#endif

typedef enum bfft_status {
    BFFT_OK = 0,
    BFFT_ERR_VALUE = 1,       /* bad enum / parameter (-> ValueError)            */
    BFFT_ERR_SHAPE = 2,       /* N / batch / shape contract (-> ValueError)      */
    BFFT_ERR_UNSUPPORTED = 3, /* no lowering for this combination (-> ValueError)*/
    BFFT_ERR_CUDA = 4,        /* CUDA runtime failure (-> RuntimeError)          */
    BFFT_ERR_NCCL = 5,        /* NCCL failure in a distributed plan              */
    BFFT_ERR_ALLOC = 6,       /* device allocation failed (-> MemoryError)       */
    BFFT_ERR_WORKSPACE = 7    /* workspace missing or too small (-> ValueError)  */
} bfft_status;

/* Decomposition direction (the reference's `direction`, entry.py:68). */
enum { BFFT_DIT = 0, BFFT_DIF = 1 };
/* transform_type (config.py:34). */
enum { BFFT_C2C = 0, BFFT_R2C = 1, BFFT_C2R = 2 };
/* transform_direction (config.py:35). */
enum { BFFT_FORWARD = 0, BFFT_INVERSE = 1 };
/* norm (config.py:36, entry.py:81-102). */
enum { BFFT_NORM_NONE = 0, BFFT_NORM_FORWARD = 1, BFFT_NORM_BACKWARD = 2, BFFT_NORM_ORTHO = 3 };
/* Batch variant of the M4 stage flow (runner.py:781-841). */
enum { BFFT_SPREAD = 0, BFFT_FOLDED = 1 };
/* Real-transform flow (entry.py:555-616): compat = packed C2C, dedicated =
 * half-length core + stitch / pre-twiddle / unpack epilogues. */
enum { BFFT_REAL_COMPAT = 0, BFFT_REAL_DEDICATED = 1 };

/* Runner identities: the reference's `plan.executed` names
 * (entry.py:175-225, runner.py, adapter_hybrid.py:224). */
typedef enum bfft_runner {
    BFFT_RUN_FFT_DIT = 0,              /* runner.py:118  M0 radix-2 DIT           */
    BFFT_RUN_FFT_DIF = 1,              /* runner.py:166  M0 radix-2 DIF           */
    BFFT_RUN_FFT_DIT_BATCH = 2,        /* runner.py:781  M4 batched DIT           */
    BFFT_RUN_FFT_DIF_BATCH = 3,        /* runner.py:844  M4 batched DIF           */
    BFFT_RUN_FFT_DIT_RADIX4 = 4,       /* runner.py:1399 M5 radix-4 DIT           */
    BFFT_RUN_FFT_DIF_RADIX4 = 5,       /* runner.py:1472 M5 radix-4 DIF           */
    BFFT_RUN_FFT_DIT_RADIX4_BATCH = 6, /* runner.py:1112                          */
    BFFT_RUN_FFT_DIF_RADIX4_BATCH = 7, /* runner.py:1193                          */
    BFFT_RUN_FFT_DIT_FUSED = 8,        /* runner.py:209  M1 fused local tile      */
    BFFT_RUN_FFT_DIT_MATRIX = 9,       /* runner.py:379  M2 local group + tail    */
    BFFT_RUN_FFT_DIF_MATRIX = 10,      /* runner.py:445                           */
    BFFT_RUN_FFT_DIT_MATRIX_BATCH = 11,/* runner.py:956  batch local-fused core   */
    BFFT_RUN_FFT_DIF_MATRIX_BATCH = 12,/* runner.py:1038                          */
    BFFT_RUN_FFT_DIT_GROUPED = 13,     /* runner.py:603  M3 grouped tail          */
    BFFT_RUN_FFT_DIF_GROUPED = 14,     /* runner.py:685                           */
    BFFT_RUN_RUN_HYBRID = 15           /* adapter_hybrid.py:224 4-step (N = T*R)  */
} bfft_runner;

/* Everything a plan needs; mirrors the fields of the reference's
 * ExecutionPlan (entry.py:105-125) that affect execution. */
typedef struct bfft_plan_desc {
    int32_t runner;              /* bfft_runner                                   */
    int32_t direction;           /* BFFT_DIT / BFFT_DIF                           */
    int64_t n;                   /* transform length (full length for R2C / C2R)  */
    int64_t batch;               /* number of transforms (>= 1)                   */
    int32_t transform_type;      /* BFFT_C2C / BFFT_R2C / BFFT_C2R                */
    int32_t transform_direction; /* BFFT_FORWARD / BFFT_INVERSE                   */
    int32_t norm;                /* BFFT_NORM_*                                   */
    int32_t real_flow;           /* BFFT_REAL_COMPAT / BFFT_REAL_DEDICATED        */
    int32_t block;               /* reference BLOCK; threads of stage kernels     */
    int32_t tile;                /* local group / hybrid tile (0 = default)       */
    int32_t rows;                /* M2 rows (tile-blocks per program)             */
    int32_t glog, maxp, cells;   /* M3 grouping knobs (matrices.py:373-405)       */
    int32_t variant;             /* BFFT_SPREAD / BFFT_FOLDED                     */
    int32_t device;              /* CUDA device ordinal                           */
} bfft_plan_desc;

typedef struct bfft_plan_s* bfft_plan_t;

/* API version (BFFT_API_VERSION of the built library). */
BFFT_EXPORT int bfft_api_version(void);

/* Thread-local message of the last failed call on this thread ("" if none). */
BFFT_EXPORT const char* bfft_last_error(void);

/* Create a plan: validates the descriptor (before any launch), allocates the
 * plan-owned twiddle tables on desc->device and returns the handle.
 * Replaces plan_fft's execution-side state (entry.py:292-426, the per-plan
 * caches of runner.py:298 / :507 and adapter_hybrid.py:62-86). */
BFFT_EXPORT bfft_status bfft_plan_create(const bfft_plan_desc* desc, bfft_plan_t* plan);

/* Bytes of caller-provided device workspace bfft_execute needs (may be 0). */
BFFT_EXPORT bfft_status bfft_plan_workspace_size(bfft_plan_t plan, size_t* bytes);

/* Number of kernel launches one bfft_execute of this plan enqueues. */
BFFT_EXPORT bfft_status bfft_plan_launches(bfft_plan_t plan, int* launches);

/* Execute the plan: in (B, N_in) -> out (B, N_out) with N_in / N_out the
 * transform-type shapes of entry.py:459-498.  Replaces execute_fft_plan
 * (entry.py:501-628): inverse conjugation, the norm epilogue and the real
 * pack / stitch / pre-twiddle / unpack all run inside this call. */
BFFT_EXPORT bfft_status bfft_execute(bfft_plan_t plan, const void* in, void* out, void* workspace,
                         size_t workspace_bytes, void* stream);

/* Release a plan and its twiddle tables. */
BFFT_EXPORT bfft_status bfft_plan_destroy(bfft_plan_t plan);

/* Y[b, i] = X[b, bitrev(i)] over (batch, n) complex64
 * (runner.py:1542-1552 bit_reverse_permute, kernels.py:81-97). */
BFFT_EXPORT bfft_status bfft_bit_reverse_permute(const void* x, void* y, int64_t n, int64_t batch,
                                     int32_t device, void* stream);

/* Dedicated real-transform epilogues as stand-alone calls
 * (runner.py:1687-1767, kernels.py:1127-1258).  z / u: (batch, n/2)
 * complex64; x: (batch, n/2+1) complex64; out: (batch, n) float32. */
BFFT_EXPORT bfft_status bfft_r2c_stitch(const void* z, void* x, int64_t n, int64_t batch, float scale,
                            int32_t device, void* stream);
BFFT_EXPORT bfft_status bfft_c2r_pre(const void* xh, void* z, int64_t n, int64_t batch, int32_t device,
                         void* stream);
BFFT_EXPORT bfft_status bfft_c2r_unpack(const void* u, void* out, int64_t n, int64_t batch, float scale,
                            int32_t device, void* stream);

/* Twiddle table of the reference (runner.py:93-97 twiddle_tables):
 * w[idx] = exp(-2 pi i idx / n) for idx < count, complex64, computed in
 * float64 and rounded once. */
BFFT_EXPORT bfft_status bfft_twiddle_table(void* w, int64_t n, int64_t count, int32_t device, void* stream);

/* Device index maps used by the kernels, written for i < 2^bits into the
 * uint32 device array `out`: kind 0 bit reversal (kernels.py:27-38),
 * 1 DIT radix-4 digit reversal (:41-57), 2 DIF digit reversal (:60-78). */
BFFT_EXPORT bfft_status bfft_index_map(int32_t kind, int32_t bits, void* out, int32_t device, void* stream);

/* 16-point DFT of every contiguous row of x ((rows, 16) complex64) on the
 * tensor cores: the dense-dot form of the reference's local_matrix_kernel
 * (src/xpu/kernels.py:487-532) with the DFT as a real 32 x 32 matrix, as
 * tcgen05.mma kind::tf32 products with the 3xTF32 split (x = hi + lo in TF32,
 * D = lo*Bhi + hi*Blo + hi*Bhi accumulated in FP32).  transform_direction
 * BFFT_INVERSE conjugates input and output; every output is multiplied by
 * scale.  Pointers 16-byte aligned, in != out, 1 <= rows < 2^31.
 * Experimental: no plan selects it (the FP32 row kernels are faster and more
 * accurate at this size). */
BFFT_EXPORT bfft_status bfft_tc_dft16_rows(const void* in, void* out, int64_t rows, int32_t transform_direction,
                                           float scale, int32_t device, void* stream);

/* 4-step C2C without any device allocation -- no counterpart in the reference.
 *
 * For callers that cannot allocate device memory while they run: code inside
 * another framework's fixed memory pool, loops where cudaMalloc / cudaFree
 * would synchronise the device, or an FFI host with no allocator for the CUDA
 * context.  Same transform as a run_hybrid plan through bfft_execute (x is
 * (batch, n) complex64, n = (n / tile) * tile with both factors <= 4096,
 * transform_direction / norm as in bfft_plan_desc) and the same kernels, but
 * the scratch buffer of the two passes is a fixed device array inside this
 * library.
 *   - Limit: n <= BFFT_NOALLOC_MAX_ELEMS (2^22), and for the two-pass shapes
 *     (1 < tile < n) batch * n <= BFFT_NOALLOC_MAX_ELEMS (32 MiB of complex64);
 *     larger requests return BFFT_ERR_SHAPE.  The one-pass shapes (tile 1 or
 *     n) use no scratch and take any batch.  Every GPU that loads the library
 *     holds that array (and a 32 KiB twiddle table) until the process exits.
 *   - No cudaMalloc / cudaFree or other allocating call is made.  The first
 *     call on a device sets up that device (looks up the arrays' device
 *     addresses, fills the library's unit twiddle tables and synchronises the
 *     legacy default stream once); make that first call before any stream
 *     capture.
 *   - All calls share the array and it keeps the last call's contents; calls
 *     whose executions overlap on the GPU race -- serialise them on one
 *     stream. */
#define BFFT_NOALLOC_MAX_ELEMS (1LL << 22)
BFFT_EXPORT bfft_status bfft_hybrid_c2c_noalloc(const void* in, void* out, int64_t n, int64_t batch,
                                                int64_t tile, int32_t transform_direction, int32_t norm,
                                                int32_t device, void* stream);

/* ------------------------------------------------------------------------
 * Multi-GPU paths.  The reference runs on one device only; these entry points
 * have no counterpart there and carry its single-device transforms across
 * ranks.  The host owns the process group and issues the exchanges (NCCL
 * all-to-all over NVLink); every call below touches this rank's device
 * memory only.
 *
 * Batch sharding (config 5a): rows [first, first + count) of a (batch, n)
 * job belong to `rank`; the first batch % nranks ranks take one extra row.
 * Each rank then runs an ordinary plan (bfft_plan_create) on its rows. */
BFFT_EXPORT bfft_status bfft_dist_batch_shard(int64_t batch, int32_t nranks, int32_t rank, int64_t* first,
                                              int64_t* count);

/* Distributed 4-step C2C of one transform of N = n1 * n2 points (config 5b),
 * the reference's hybrid 4-step (src/xpu/adapter_hybrid.py:224-270, N = T*R)
 * with the transposes that cross ranks done as all-to-alls.  Rank r holds the
 * contiguous slab x[r N/P, (r+1) N/P) on input and X[r N/P, (r+1) N/P) on
 * output (natural order), P = nranks (a power of two dividing n1 and n2).
 * One execution is
 *     phase 0 -> all-to-all -> phase 1 -> all-to-all -> phase 2 -> all-to-all -> phase 3
 * where each all-to-all exchanges equal chunks of N/P^2 complex64 (chunk s of
 * the send buffer goes to rank s; chunk p of the receive buffer comes from
 * rank p) and phase k+1 reads the receive buffer of the exchange before it.
 * With nranks = 1 the exchanges are identities (phase k+1 reads phase k's
 * output).  Every phase writes N/P complex64 to `out`; phases 1, 2 and 4 need
 * bfft_dist_workspace_size bytes of workspace.  Row FFT tiles 0 = default.
 * Transposed-output mode: phase 4 takes the place of phase 2, the third
 * all-to-all and phase 3,
 *     phase 0 -> all-to-all -> phase 1 -> all-to-all -> phase 4
 * and leaves rank r with the (n1/P) x n2 block out[k1'][k2] =
 * X[k2 n1 + r n1/P + k1'] (whole columns of the n1 x n2 output view) instead
 * of the natural-order slab. */
typedef struct bfft_dist_plan_s* bfft_dist_plan_t;
BFFT_EXPORT bfft_status bfft_dist_plan_create(int64_t n1, int64_t n2, int32_t nranks, int32_t rank,
                                              int32_t transform_direction, int32_t norm, int32_t row_tile1,
                                              int32_t row_tile2, int32_t device, bfft_dist_plan_t* plan);
BFFT_EXPORT bfft_status bfft_dist_workspace_size(bfft_dist_plan_t plan, size_t* bytes);
BFFT_EXPORT bfft_status bfft_dist_phase(bfft_dist_plan_t plan, int32_t phase, const void* in, void* out,
                                        void* workspace, size_t workspace_bytes, void* stream);
/* Peer-to-peer mode of the same transform: every exchange is fused into the
 * transpose before it.  Each rank owns two exchange buffers (2 N/P complex64,
 * allocated by bfft_dist_p2p_prepare); once every rank's buffers are mapped
 * into every process (bfft_dist_p2p_attach with the nranks CUDA IPC handles
 * of prepare, in rank order -- or bfft_dist_p2p_attach_pointers with device
 * pointers when all ranks live in one process), phase k writes its result
 * over NVLink straight into the destination ranks' buffers, in the layout
 * their next phase reads:
 *     barrier -> phase 0 -> barrier -> phase 1 -> barrier -> phase 2 -> barrier -> phase 3
 * where a barrier means every rank's previous phase has completed (the host
 * orders it, e.g. a stream-ordered all-reduce of one word).  Phase 0 reads
 * `in` (the rank's slab), phase 3 writes `out` (the rank's output slab);
 * phases 1 and 2 need bfft_dist_workspace_size bytes of workspace.  The
 * transposed-output order is barrier -> phase 0 -> barrier -> phase 1 ->
 * barrier -> phase 4, phase 4 writing the block described above to `out`.  No
 * device-side waits, no multicast: plain stores to peer memory. */
BFFT_EXPORT bfft_status bfft_dist_p2p_prepare(bfft_dist_plan_t plan, void* exchange_base, void* ipc_handle,
                                              size_t* handle_bytes);
BFFT_EXPORT bfft_status bfft_dist_p2p_attach(bfft_dist_plan_t plan, const void* handles);
BFFT_EXPORT bfft_status bfft_dist_p2p_attach_pointers(bfft_dist_plan_t plan, void* const* exchange_bases);
BFFT_EXPORT bfft_status bfft_dist_p2p_phase(bfft_dist_plan_t plan, int32_t phase, const void* in, void* out,
                                            void* workspace, size_t workspace_bytes, void* stream);
/* Kernel launches one bfft_dist_phase call of `phase` enqueues. */
BFFT_EXPORT bfft_status bfft_dist_plan_launches(bfft_dist_plan_t plan, int32_t phase, int* launches);
BFFT_EXPORT bfft_status bfft_dist_plan_destroy(bfft_dist_plan_t plan);

/* Host-to-host execution -- no counterpart in the reference (its operator API
 * takes device tensors).  A stream plan runs `chunks` back-to-back executions
 * of the plan described by `chunk_desc` (batch = rows per chunk) over host
 * arrays of chunks * batch rows, overlapping the copy in of chunk k+1, the
 * transform of chunk k and the copy out of chunk k-1 on three internal
 * streams with two device buffers per direction (allocated at creation).
 * bfft_stream_execute orders itself after the work already enqueued on
 * `stream` and makes `stream` wait for its completion; host buffers should be
 * page-locked for the copies to overlap.  Shapes per row as in bfft_execute. */
typedef struct bfft_stream_plan_s* bfft_stream_plan_t;
BFFT_EXPORT bfft_status bfft_stream_plan_create(const bfft_plan_desc* chunk_desc, int64_t chunks,
                                                bfft_stream_plan_t* plan);
BFFT_EXPORT bfft_status bfft_stream_plan_info(bfft_stream_plan_t plan, size_t* in_bytes_per_chunk,
                                              size_t* out_bytes_per_chunk, int* launches_per_chunk);
BFFT_EXPORT bfft_status bfft_stream_execute(bfft_stream_plan_t plan, const void* host_in, void* host_out,
                                            void* stream);
BFFT_EXPORT bfft_status bfft_stream_plan_destroy(bfft_stream_plan_t plan);

/* Status bits the kernels set on `device` when a bounded wait expired
 * (bit 0: a TMA pass gave up waiting for a tile copy and returned early, so
 * its output is incomplete).  Synchronises the device; clear != 0 resets the
 * word.  Always 0 in a healthy run -- the tests check it. */
BFFT_EXPORT bfft_status bfft_device_status(int32_t device, uint32_t* status, int32_t clear);

/* Failure-detection probe (no reference counterpart: the reference has no
 * device-side waits).  Runs one kernel on `stream` whose two bounded waits --
 * on an mbarrier nothing arrives on, then on a dependency counter nothing
 * increments -- each give up after their limit (about 1 s) and set status
 * bits 0 and 1; synchronises the stream and returns BFFT_OK.  Read and clear
 * the bits with bfft_device_status.  Takes about 2 s. */
BFFT_EXPORT bfft_status bfft_probe_bounded_waits(int32_t device, void* stream);

/* Total kernels this library has enqueued in this process (all devices). */
BFFT_EXPORT uint64_t bfft_launch_counter(void);

#ifdef __cplusplus
}
#endif

#endif /* BFFT_H */
