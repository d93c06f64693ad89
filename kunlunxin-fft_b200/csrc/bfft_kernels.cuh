// bfft_kernels.cuh -- kernel declarations and launch-parameter structs.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "bfft_device.cuh"

namespace bfft {

// Global unit twiddle tables: level Lp = 2^l (1 <= l <= kTwUnitBits) holds
// exp(-2 pi i e / Lp) for e < Lp at offset Lp, i.e. W_Lp^e = tw[Lp + e].
cudaError_t ensure_unit_twiddles(int device, cudaStream_t stream);
const float2* unit_twiddles(int device);

// Two-level table for W_N^e, e < N (plan-owned device memory).
cudaError_t fill_two_level(float2* lo, float2* hi, int lo_bits, int log2n, cudaStream_t s);
// Three-level table (3 x 2^bits entries, TwoLevel::l3) for W_N^e, e < N.
cudaError_t fill_three_level(float2* t, int bits, int log2n, cudaStream_t s);

// ---------------------------------------------------------------- stage kernels
struct StageArgs {
    int64_t n;        // transform length N
    int64_t batch;    // rows
    int64_t half;     // butterfly half-span (radix-2) or quarter-span n (radix-4)
    int64_t M;        // twiddle stride (exponent = j * M)
    int log2n;
    int in_perm;      // 0 none, 1 bit-reversed read (DIT stage 0), 2 DIT digit-reversed read
    int out_perm;     // 0 none, 1 bit-reversed store, 2 DIF digit-reversed store
    int conj_in;      // conjugate inputs (inverse via the conjugate trick)
    int conj_out;     // conjugate outputs
    float scale;      // applied to outputs (1 = none)
    int folded;       // 1: flat 1-D grid over batch * pairs (M4 "folded"), 0: spread
    TwoLevel tw;
};

cudaError_t launch_radix2_stage(bool dif, const float2* x, float2* y, const StageArgs& a,
                                int block, cudaStream_t s);
cudaError_t launch_radix4_stage(bool dif, const float2* x, float2* y, const StageArgs& a,
                                int block, cudaStream_t s);
cudaError_t launch_bitrev(const float2* x, float2* y, int64_t n, int64_t batch, int block,
                          cudaStream_t s, int conj = 0, float scale = 1.0f);

// Packed-compat real-transform helpers (src/xpu/entry.py:588-616, :671-696).
cudaError_t launch_real_to_complex(const float* x, float2* y, int64_t total, cudaStream_t s);
cudaError_t launch_crop(const float2* y, float2* out, int64_t n, int64_t batch, float scale,
                        cudaStream_t s);
cudaError_t launch_hermitian_conj(const float2* xh, float2* full, int64_t n, int64_t batch,
                                  cudaStream_t s);
cudaError_t launch_real_part(const float2* y, float* out, int64_t total, float scale,
                             cudaStream_t s);
cudaError_t launch_twiddle_table(float2* w, int64_t n, int64_t count, cudaStream_t s);
cudaError_t launch_index_map(int kind, int bits, uint32_t* out, cudaStream_t s);

// ---------------------------------------------------------------- cluster FFT
// Whole transforms of N = 2^13 .. 2^16 points in one HBM round trip on a
// thread-block cluster (4-step with the transpose in distributed shared
// memory).  `tw` is the plan's W_N table.
struct ClusterArgs {
    int64_t batch;
    TwoLevel tw;
    float scale;
    int conj_in, conj_out;
};
bool cluster_supported(int log2n);
cudaError_t launch_cluster_fft(int log2n, const float2* in, float2* out, const ClusterArgs& a, cudaStream_t s);

// ---------------------------------------------------------------- fused single pass
// Whole transforms of N = 2^13 .. 2^16 in one HBM round trip without
// clusters: the 4-step's two phases as tiles of one persistent kernel, the
// intermediate in an L2-resident ring of scratch slots (workspace).
struct FusedArgs {
    int64_t batch;
    TwoLevel tw;              // the plan's W_N
    float scale;
    int conj_in, conj_out;
    int tw_smem_entries, tw_smem_levels;  // set by the launcher
    uint32_t* counters;       // [0] ticket, [1, 1+S) a_done, [1+S, 1+2S) b_done; zeroed before each launch
    float2* scratch;          // S slots of N complex64
    int slots;                // S (set by the launcher)
    int lag;                  // D rounds (set by the launcher)
    int pdl;
};
bool fused_supported(int log2n);
// Workspace of one launch: the scratch ring and its counters.
size_t fused_workspace_bytes(int64_t n, int64_t batch);
cudaError_t launch_fused_fft(int log2n, const float2* in, float2* out, void* workspace, const FusedArgs& a,
                             cudaStream_t s);

// Status word the kernels set when a bounded wait expires (bit 0: an
// mbarrier wait of the TMA pass); read synchronously, optionally cleared.
cudaError_t read_device_status(unsigned* status, bool clear);
// One kernel whose two bounded waits (mbarrier, dependency counter) expire.
cudaError_t run_wait_probe(cudaStream_t s);

// SM count of `dev`, cached after the first query (thread-safe).
// 16-point DFT of each contiguous row of `rows` x 16 complex64 on the tensor
// cores (3xTF32 tcgen05.mma); conj_in / conj_out give the inverse.
cudaError_t launch_tc_dft16_rows(const float2* in, float2* out, int64_t rows, float scale, int conj_in, int conj_out,
                                 cudaStream_t s);
cudaError_t device_sm_count(int dev, int* sms);

// Library-wide error message (bfft_last_error) and launch counter.
void set_last_error(const char* msg);
void count_launches(int k);

// The run_hybrid flow (the same steps a BFFT_RUN_RUN_HYBRID plan builds) from
// `in` to `out` through `scratch` (batch * n complex64; unused when tile is 1
// or n): conj conjugates the input and the output, scale the output.  Counts
// its launches.
cudaError_t run_hybrid_flow(const float2* in, float2* out, float2* scratch, int64_t n, int64_t batch,
                            int64_t tile, const TwoLevel& tw, int conj, float scale, cudaStream_t s);

// Real-transform epilogues (standalone forms of the reference runner API).
cudaError_t launch_r2c_stitch(const float2* z, float2* x, int64_t n, int64_t batch, float scale,
                              TwoLevel twn, cudaStream_t s);
cudaError_t launch_c2r_pre(const float2* xh, float2* z, int64_t n, int64_t batch, TwoLevel twn,
                           cudaStream_t s);
cudaError_t launch_c2r_unpack(const float2* u, float* out, int64_t n, int64_t batch, float scale,
                              cudaStream_t s);
// y = scale * (conj?) x, elementwise over count complex values.
cudaError_t launch_scale(const float2* x, float2* y, int64_t count, float scale, int conj,
                         cudaStream_t s);

// ---------------------------------------------------------------- Stockham pass
// One CTA-resident pass: nsub independent sub-FFTs of length L = 2^log2l.
// Sub-FFT f = o * inner + c reads element m from
//     in[o*in_outer + C_in(c)*in_inner + P_in(m)*in_stride]
// and writes output k to
//     out[o*out_outer + C_out(c)*out_inner + P_out(k)*out_stride]
// where C_*(c) is c or bitrev(c, *_base_bits) and P_*(m) is m or
// bitrev(m, log2l).  Optional twiddles: pre (input m times W_N^{m*c*tw_mul})
// or post (output k times W_N^{k*c*tw_mul}) with the plan's two-level W_N.
struct PassArgs {
    int64_t nsub;
    int64_t inner;       // a power of two
    int inner_log2;
    int64_t in_outer, in_inner, in_stride;
    int64_t out_outer, out_inner, out_stride;
    int in_base_bits, out_base_bits;
    int in_elem_bitrev, out_elem_bitrev;
    int tw_mode;  // 0 none, 1 pre, 2 post
    int64_t tw_mul;
    TwoLevel tw;
    float scale;
    int conj_in, conj_out;
    const float2* unit_tw;  // unit twiddle levels (ensure_unit_twiddles)
    int tw_smem_entries;    // set by launch_pass: shared-memory entries of the staged W_N tables
    int tw_smem_levels;     // set by launch_pass: 0 global two-level, 2 / 3 staged two- / three-level
    // 1: the previous kernel on the stream is a pass of the same flow -- a TMA
    // pass is then launched as its programmatic dependent (it may start while
    // that kernel drains and waits for it before touching its output)
    int pdl;
};

constexpr int kMaxPassLog2 = 12;  // largest CTA-resident sub-FFT: 4096 points

// layout: 0 rows (element index fastest across threads), 1 columns (sub-FFT
// index fastest).  lmap: 1 = the tile is contiguous and is copied
// cooperatively (rows only).  smap: 0 store from registers, 1 staged store
// with the element index fastest, 2 staged store with the sub-FFT index
// fastest (rows only).
cudaError_t launch_pass(int log2l, int layout, int lmap, int smap, const float2* in, float2* out,
                        const PassArgs& a, cudaStream_t s);

}  // namespace bfft
