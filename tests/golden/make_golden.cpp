// tests/golden/make_golden.cpp -- writes the golden scan vectors.
//
// Built by tests/golden/make_golden.py against the reference's own
// Sources/CPURef/selective_scan_cpu.cpp (compiled from the reference tree,
// never copied).  Every output array below is produced by the reference's
// mamba::cpu::selective_scan_cpu; the inputs reproduce the reference test
// suite's cases, drawing from the same generator in the same order so that
// its known answer (last_y = -0.453731 for Tests/test_selective_scan.cpp)
// is reproduced.
//
// File format (little endian), one file per case, <outdir>/<name>.bin:
//   char[8] magic "MGOLD01\0"; int32 L, D, N, flags;
//   float32 x[L*D], delta[L*D], B[L*N], C[L*N], A[D*N], Dskip[D],
//           y[L*D], state[D*N]
#include "selective_scan_cpu.hpp"

#include <cmath>
#include <cstdint>
#include <cstdio>
#include <random>
#include <string>
#include <vector>

using mamba::cpu::selective_scan_cpu;

struct Case {
    std::string name;
    int L, D, N;
    std::vector<float> x, delta, B, C, A, Dskip, y, state;
    Case(std::string n, int l, int d, int s)
        : name(std::move(n)), L(l), D(d), N(s), x((size_t)l * d), delta((size_t)l * d),
          B((size_t)l * s), C((size_t)l * s), A((size_t)d * s), Dskip(d),
          y((size_t)l * d), state((size_t)d * s) {}
    void run() {
        selective_scan_cpu(x.data(), delta.data(), B.data(), C.data(), A.data(),
                           Dskip.data(), y.data(), state.data(), L, D, N);
    }
    bool write(const std::string &dir) const {
        std::string path = dir + "/" + name + ".bin";
        FILE *f = std::fopen(path.c_str(), "wb");
        if (!f) return false;
        const char magic[8] = {'M', 'G', 'O', 'L', 'D', '0', '1', 0};
        int32_t hdr[4] = {L, D, N, 0};
        std::fwrite(magic, 1, 8, f);
        std::fwrite(hdr, 4, 4, f);
        for (const auto *v : {&x, &delta, &B, &C, &A, &Dskip, &y, &state})
            std::fwrite(v->data(), sizeof(float), v->size(), f);
        std::fclose(f);
        return true;
    }
};

int main(int argc, char **argv) {
    const std::string dir = argc > 1 ? argv[1] : ".";
    std::vector<Case> cases;

    {   // Tests/test_selective_scan.cpp:12-24 inputs: mt19937(42), U(-1,1),
        // fill order x, delta*0.1, B, C, A=-|u|, Dskip*0.1.
        Case c("ref_test_selective_scan", 128, 64, 16);
        std::mt19937 rng(42);
        std::uniform_real_distribution<float> u(-1.f, 1.f);
        for (auto &v : c.x) v = u(rng);
        for (auto &v : c.delta) v = u(rng) * 0.1f;
        for (auto &v : c.B) v = u(rng);
        for (auto &v : c.C) v = u(rng);
        for (auto &v : c.A) v = -std::abs(u(rng));
        for (auto &v : c.Dskip) v = u(rng) * 0.1f;
        c.run();
        std::printf("ref_test_selective_scan last_y=%.6f\n", c.y.back());
        cases.push_back(std::move(c));
    }
    {   // Tests/test_numerical.cpp:16-36 impulse case.
        Case c("ref_test_impulse", 64, 4, 2);
        for (auto &v : c.x) v = 0.f;
        for (auto &v : c.delta) v = 0.1f;
        for (auto &v : c.B) v = 1.f;
        for (auto &v : c.C) v = 1.f;
        for (auto &v : c.A) v = -0.5f;
        for (auto &v : c.Dskip) v = 0.f;
        c.x[0] = 1.f;
        c.run();
        cases.push_back(std::move(c));
    }
    {   // Tests/test_numerical.cpp:38-51 zero-input case.
        Case c("ref_test_zero_input", 32, 8, 4);
        for (auto &v : c.x) v = 0.f;
        for (auto &v : c.delta) v = 0.1f;
        for (auto &v : c.B) v = 0.5f;
        for (auto &v : c.C) v = 0.5f;
        for (auto &v : c.A) v = -1.f;
        for (auto &v : c.Dskip) v = 0.1f;
        c.run();
        cases.push_back(std::move(c));
    }
    {   // Benchmarks/bench_scan.cpp:22-33 distribution: mt19937(123), U(-.5,.5),
        // delta*0.05, A=-|u|, Dskip*0.1; D reduced from 512 to 64, L = 256.
        Case c("ref_bench_dist", 256, 64, 16);
        std::mt19937 rng(123);
        std::uniform_real_distribution<float> u(-0.5f, 0.5f);
        for (auto &v : c.x) v = u(rng);
        for (auto &v : c.delta) v = u(rng) * 0.05f;
        for (auto &v : c.B) v = u(rng);
        for (auto &v : c.C) v = u(rng);
        for (auto &v : c.A) v = -std::abs(u(rng));
        for (auto &v : c.Dskip) v = u(rng) * 0.1f;
        c.run();
        cases.push_back(std::move(c));
    }
    {   // Single-sequence slice of the standalone-scan workload distributions:
        // x, B, C ~ N(0,1); delta_raw ~ N(-4.6, 0.5); A[d,n] = -(n+1); D = 1.
        Case c("scan_workload_slice", 256, 128, 16);
        std::mt19937 rng(2024);
        std::normal_distribution<float> g(0.f, 1.f);
        std::normal_distribution<float> gd(-4.6f, 0.5f);
        for (auto &v : c.x) v = g(rng);
        for (auto &v : c.delta) v = gd(rng);
        for (auto &v : c.B) v = g(rng);
        for (auto &v : c.C) v = g(rng);
        for (int d = 0; d < c.D; ++d)
            for (int n = 0; n < c.N; ++n) c.A[(size_t)d * c.N + n] = -(float)(n + 1);
        for (auto &v : c.Dskip) v = 1.f;
        c.run();
        cases.push_back(std::move(c));
    }
    {   // Edge values: A on both sides of the |A| <= 1e-6 branch (including 0
        // and a positive A), delta_raw above 20 (softplus identity branch) and
        // strongly negative; odd sizes L = 37, D = 13, N = 5.
        Case c("edge_branches", 37, 13, 5);
        std::mt19937 rng(7);
        std::uniform_real_distribution<float> u(-1.f, 1.f);
        for (auto &v : c.x) v = u(rng);
        for (auto &v : c.B) v = u(rng);
        for (auto &v : c.C) v = u(rng);
        for (auto &v : c.Dskip) v = u(rng);
        const float avals[8] = {0.f, 1e-6f, -1e-6f, 1.0001e-6f, -2e-6f, -3.f, 0.25f, -1e-7f};
        for (size_t i = 0; i < c.A.size(); ++i) c.A[i] = avals[i % 8];
        const float dvals[6] = {25.f, 20.f, 20.5f, -30.f, -4.6f, 0.f};
        for (size_t i = 0; i < c.delta.size(); ++i)
            c.delta[i] = (i % 3 == 0) ? dvals[(i / 3) % 6] : u(rng) * 0.1f;
        c.run();
        cases.push_back(std::move(c));
    }
    for (const auto &c : cases)
        if (!c.write(dir)) {
            std::fprintf(stderr, "cannot write %s\n", c.name.c_str());
            return 1;
        }
    std::printf("wrote %zu golden cases to %s\n", cases.size(), dir.c_str());
    return 0;
}
