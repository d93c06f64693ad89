// ref_driver.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Thin extern "C" driver around the reference's own native CPU FFT
// (include/butterfly/fft.hpp, bit_reverse.hpp, twiddle.hpp).  The reference
// headers are NOT copied into this repository: oracle/Makefile compiles this
// file with -I pointing at the read-only reference tree and writes the result
// to oracle/_ref/libbutterfly_ref.so (git-ignored).  It is used to pin the
// oracle restatement and as the timed CPU baseline of bench.py.
#include <algorithm>
#include <complex>
#include <cstdint>
#include <thread>
#include <vector>

#include "butterfly/bit_reverse.hpp"
#include "butterfly/fft.hpp"
#include "butterfly/twiddle.hpp"

extern "C" {

// butterfly::bit_reverse (include/butterfly/bit_reverse.hpp:15-22).
uint32_t ref_bit_reverse(uint32_t x, int bits) { return butterfly::bit_reverse(x, bits); }

// Rows of a (batch, n) interleaved complex<double> array through
// butterfly::fft_dit (dif=0) or butterfly::fft_dif (dif=1)
// (include/butterfly/fft.hpp:70-97).  Rows are split over `threads`
// std::threads (threads <= 1 runs on the calling thread).  Returns 0 on
// success, 1 on a non-power-of-two length.
int ref_fft_c128(const double* x, double* y, int64_t n, int64_t batch, int dif, int threads) {
    if (!butterfly::is_power_of_two(static_cast<std::size_t>(n))) return 1;
    auto run_rows = [&](int64_t r0, int64_t r1) {
        std::vector<std::complex<double>> row(static_cast<std::size_t>(n));
        for (int64_t r = r0; r < r1; ++r) {
            const double* src = x + 2 * n * r;
            for (int64_t i = 0; i < n; ++i) row[i] = {src[2 * i], src[2 * i + 1]};
            auto out = dif ? butterfly::fft_dif(row) : butterfly::fft_dit(row);
            double* dst = y + 2 * n * r;
            for (int64_t i = 0; i < n; ++i) {
                dst[2 * i] = out[i].real();
                dst[2 * i + 1] = out[i].imag();
            }
        }
    };
    int t = std::max(1, threads);
    if (t == 1 || batch == 1) {
        run_rows(0, batch);
        return 0;
    }
    std::vector<std::thread> pool;
    int64_t per = (batch + t - 1) / t;
    for (int k = 0; k < t; ++k) {
        int64_t r0 = k * per, r1 = std::min<int64_t>(batch, r0 + per);
        if (r0 >= r1) break;
        pool.emplace_back(run_rows, r0, r1);
    }
    for (auto& th : pool) th.join();
    return 0;
}

}  // extern "C"
