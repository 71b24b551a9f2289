// rotation.cpp -- the USQ rotation matrix: a seeded uniform [-1, 1) square matrix,
// Householder-QR factorised, Q kept (row-major f32).  This is the method of
// src/quantization/usq/rotator.rs:15-39; the random stream (splitmix64) and the QR
// arithmetic (f64) are this library's own, so Q differs from the Rust build's bits.
// The matrix is part of the index and is saved with it.
#include <cmath>
#include <cstdint>
#include <vector>

namespace hanns {

void rotation_matrix(uint64_t seed, int D, float* out) {
    std::vector<double> A((size_t)D * D), Q((size_t)D * D, 0.0), v(D);
    uint64_t s = seed;
    auto next = [&]() {
        s += 0x9E3779B97F4A7C15ull;
        uint64_t z = s;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    for (size_t i = 0; i < A.size(); ++i)
        A[i] = (double)(next() >> 40) * (1.0 / 16777216.0) * 2.0 - 1.0;
    for (int i = 0; i < D; ++i) Q[(size_t)i * D + i] = 1.0;
    // Column-major work copy for cache-friendly reflections.
    std::vector<double> C((size_t)D * D);
    for (int r = 0; r < D; ++r)
        for (int c = 0; c < D; ++c) C[(size_t)c * D + r] = A[(size_t)r * D + c];
    for (int k = 0; k < D - 1; ++k) {
        double* ck = &C[(size_t)k * D];
        double nrm = 0;
        for (int i = k; i < D; ++i) nrm += ck[i] * ck[i];
        nrm = std::sqrt(nrm);
        if (nrm == 0) continue;
        const double alpha = ck[k] > 0 ? -nrm : nrm;
        for (int i = 0; i < D; ++i) v[i] = i < k ? 0.0 : ck[i];
        v[k] -= alpha;
        double vn = 0;
        for (int i = k; i < D; ++i) vn += v[i] * v[i];
        if (vn == 0) continue;
#pragma omp parallel for schedule(static)
        for (int j = k; j < D; ++j) {
            double* cj = &C[(size_t)j * D];
            double dot = 0;
            for (int i = k; i < D; ++i) dot += v[i] * cj[i];
            const double f = 2.0 * dot / vn;
            for (int i = k; i < D; ++i) cj[i] -= f * v[i];
        }
#pragma omp parallel for schedule(static)
        for (int r = 0; r < D; ++r) {
            double* qr = &Q[(size_t)r * D];
            double dot = 0;
            for (int i = k; i < D; ++i) dot += qr[i] * v[i];
            const double f = 2.0 * dot / vn;
            for (int i = k; i < D; ++i) qr[i] -= f * v[i];
        }
    }
    for (size_t i = 0; i < Q.size(); ++i) out[i] = (float)Q[i];
}

}  // namespace hanns
