// oracle/ref_shim.cpp -- C-ABI shim around the reference's own CPU oracle.
//
// TEST INFRASTRUCTURE ONLY (the checker and the CPU-baseline timer).  It is
// compiled together with the reference's Sources/CPURef/selective_scan_cpu.cpp
// straight from the reference tree by oracle/build_oracle.py, into
// oracle/_ref/libref_scan.so.  No reference source is copied into this repo.
//
//   ref_selective_scan_cpu   forwards to mamba::cpu::selective_scan_cpu
//                            (Sources/CPURef/selective_scan_cpu.hpp:31-36).
//   ref_scan_batched_mt      runs that same function over a batch of
//                            sequences in [B, L, D] / [B, L, N] layout, with
//                            the channel range split across host threads.
//                            The per-channel recurrences are independent and
//                            B, C are shared by all channels, so each slice is
//                            gathered into a contiguous [L, Dslice] buffer,
//                            scanned by the reference code, and scattered
//                            back.  Results equal the single-threaded call.
#include "selective_scan_cpu.hpp"

#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

extern "C" {

int ref_selective_scan_cpu(const float *x, const float *delta, const float *B,
                           const float *C, const float *A, const float *Dskip,
                           float *y, float *state_out, int L, int D, int N)
{
    mamba::cpu::selective_scan_cpu(x, delta, B, C, A, Dskip, y, state_out, L, D, N);
    return 0;
}

// x, delta, y: [batch, L, D]; B, C: [batch, L, N]; A: [D, N]; Dskip: [D];
// state_out: [batch, D, N] or NULL.
int ref_scan_batched_mt(const float *x, const float *delta, const float *B,
                        const float *C, const float *A, const float *Dskip,
                        float *y, float *state_out, int batch, int L, int D,
                        int N, int nthreads)
{
    if (nthreads < 1) nthreads = 1;
    // Work items: (batch row, channel slice).
    const int slices_per_row = nthreads;
    const int items = batch * slices_per_row;
    auto worker = [&](int tid) {
        for (int it = tid; it < items; it += nthreads) {
            const int b = it / slices_per_row, s = it % slices_per_row;
            const int d0 = (int)((int64_t)D * s / slices_per_row);
            const int d1 = (int)((int64_t)D * (s + 1) / slices_per_row);
            const int Ds = d1 - d0;
            if (Ds <= 0) continue;
            std::vector<float> xs((size_t)L * Ds), ds((size_t)L * Ds), ys((size_t)L * Ds);
            std::vector<float> hs((size_t)Ds * N);
            const size_t row = (size_t)b * L * D;
            for (int t = 0; t < L; ++t) {
                std::memcpy(&xs[(size_t)t * Ds], x + row + (size_t)t * D + d0, sizeof(float) * Ds);
                std::memcpy(&ds[(size_t)t * Ds], delta + row + (size_t)t * D + d0, sizeof(float) * Ds);
            }
            mamba::cpu::selective_scan_cpu(xs.data(), ds.data(),
                                           B + (size_t)b * L * N, C + (size_t)b * L * N,
                                           A + (size_t)d0 * N, Dskip + d0,
                                           ys.data(), hs.data(), L, Ds, N);
            for (int t = 0; t < L; ++t)
                std::memcpy(y + row + (size_t)t * D + d0, &ys[(size_t)t * Ds], sizeof(float) * Ds);
            if (state_out)
                std::memcpy(state_out + ((size_t)b * D + d0) * N, hs.data(), sizeof(float) * Ds * N);
        }
    };
    std::vector<std::thread> pool;
    for (int i = 1; i < nthreads; ++i) pool.emplace_back(worker, i);
    worker(0);
    for (auto &th : pool) th.join();
    return 0;
}

}  // extern "C"
