// cpu_fast.cpp -- TEST/BENCH INFRASTRUCTURE ONLY (the timed CPU baseline).
//
// A portable fp32 restatement of the reference's fast CPU int4 GEMV path,
// cpu_gemv_neon (hetero-gemv/src/cpu_gemv.h:88-103): per 32-weight chunk the
// nibbles are unpacked and dotted with fp32 x, then folded into the row sum as
//   acc += S[g] * dot + B[g] * xs[chunk]
// with xs the per-32 partial sums of x.  The reference's version is ARM NEON and
// cannot build on x86; this one is plain C++ that the compiler vectorises
// (built with -O3 -march=x86-64-v3).  Rows are split over std::thread workers.
// It is only ever run as the CPU baseline next to the GPU numbers.

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

inline float h2f(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 0x1F, man = h & 0x3FF;
    uint32_t u;
    if (exp == 0) {
        if (man == 0) { u = sign; }
        else {  // subnormal: renormalise
            int e = -1;
            uint32_t mm = man;
            do { mm <<= 1; ++e; } while (!(mm & 0x400));
            u = sign | ((uint32_t)(127 - 15 - e) << 23) | ((mm & 0x3FF) << 13);
        }
    } else if (exp == 31) {
        u = sign | 0x7F800000u | (man << 13);
    } else {
        u = sign | ((exp + 112) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

void rows_f32(const uint8_t* W, const uint16_t* SB, const float* xf, const float* xs,
              float* y, uint32_t K, uint32_t G, uint32_t m0, uint32_t m1) {
    const uint32_t chunks = K / 32, cpg = G / 32, groups = K / G;
    for (uint32_t m = m0; m < m1; ++m) {
        const uint8_t* wp = W + (size_t)m * (K / 2);
        const uint16_t* sb = SB + (size_t)m * groups * 2;
        float accf = 0.0f;
        for (uint32_t j = 0; j < chunks; ++j) {
            const uint8_t* p = wp + j * 16;
            const float* x = xf + j * 32;
            float q[32];
            for (int i = 0; i < 16; ++i) {
                q[2 * i] = (float)(p[i] & 0xF);
                q[2 * i + 1] = (float)(p[i] >> 4);
            }
            float d = 0.0f;
            for (int i = 0; i < 32; ++i) d += q[i] * x[i];
            uint32_t g = j / cpg;
            accf += h2f(sb[2 * g]) * d + h2f(sb[2 * g + 1]) * xs[j];
        }
        y[m] = accf;
    }
}

}  // namespace

extern "C" {

// y[M] fp32 from W (packed nibbles), SB (interleaved fp16 scale,bias), x fp16.
// xs is computed here once per call (the per-token prepass); nthreads <= 0 uses
// every hardware thread.  Returns the thread count used.
int cpu_fast_gemv_int4_sb(const uint32_t* W, const uint16_t* SB, const uint16_t* x,
                          float* y, uint32_t M, uint32_t K, uint32_t G, int nthreads) {
    std::vector<float> xf(K), xs(K / 32, 0.0f);
    for (uint32_t k = 0; k < K; ++k) xf[k] = h2f(x[k]);
    for (uint32_t j = 0; j < K / 32; ++j)
        for (uint32_t t = 0; t < 32; ++t) xs[j] += xf[j * 32 + t];
    unsigned n = nthreads > 0 ? (unsigned)nthreads
                              : std::max(1u, std::thread::hardware_concurrency());
    std::vector<std::thread> th;
    uint32_t chunk = (M + n - 1) / n;
    unsigned used = 0;
    for (unsigned i = 0; i < n; ++i) {
        uint32_t a = i * chunk, b = std::min(M, a + chunk);
        if (a >= b) break;
        th.emplace_back(rows_f32, (const uint8_t*)W, SB, xf.data(), xs.data(), y, K, G, a, b);
        ++used;
    }
    for (auto& t : th) t.join();
    return (int)used;
}

}  // extern "C"
