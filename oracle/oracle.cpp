// oracle.cpp -- TEST INFRASTRUCTURE ONLY.
//
// CPU restatement of the reference's own CPU references for the decode hot path
// (int4 group-affine GEMV, VQ codebook GEMV, fused MoE block).  It exists to
// check the CUDA kernels: only tests/, __graft_entry__.smoke() and the
// cpu_baseline leg of bench.py load it.  libcuda-graft.so never links it and no
// product code path calls it.
//
// Every reference routine accumulates in fp64 and evaluates the sum in the
// "straightforward order" (one weight at a time, k ascending); the functions
// below do the same so that their results are independent of how the GPU
// kernels factor the arithmetic.  Parity is pinned by tests/golden/, whose
// vectors were produced by the reference's own functions compiled from the
// reference sources (oracle/ref_build.sh -> oracle/_ref/libref.so).
//
// Half/bfloat16 -> double conversions are written out bit by bit (every fp16
// and bf16 value is exactly representable in double), so the oracle does not
// depend on the host compiler's __fp16/_Float16 support.

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

// IEEE binary16 -> double, exact (normals, subnormals, inf, nan).
double h2d_slow(uint16_t h) {
    const uint32_t sign = h >> 15, exp = (h >> 10) & 0x1F, man = h & 0x3FF;
    double v;
    if (exp == 0)       v = std::ldexp((double)man, -24);                 // subnormal / zero
    else if (exp == 31) v = man ? NAN : INFINITY;
    else                v = std::ldexp((double)(man | 0x400), (int)exp - 25);
    return sign ? -v : v;
}

struct HalfTable {
    double v[65536];
    HalfTable() { for (uint32_t i = 0; i < 65536; ++i) v[i] = h2d_slow((uint16_t)i); }
};
const HalfTable g_half;

inline double h2d(uint16_t h) { return g_half.v[h]; }

// bfloat16 -> double: the top 16 bits of an IEEE float (moe-fused/src/main.mm:43).
inline double bf2d(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return (double)f;
}

inline double scale_to_d(uint16_t v, bool bf16) { return bf16 ? bf2d(v) : h2d(v); }

// Row-block parallel loop, as the reference's cpuRef/parRows/par helpers do
// (int4-gemv/src/main.mm:81-92, vq-gemv/src/main.mm:81-90, moe-fused/src/main.mm:63-72).
template <class F>
void par_rows(uint32_t M, int nthreads, F f) {
    unsigned n = nthreads > 0 ? (unsigned)nthreads
                              : std::max(1u, std::thread::hardware_concurrency());
    if (n == 1 || M < 2) { f(0u, M); return; }
    std::vector<std::thread> th;
    uint32_t chunk = (M + n - 1) / n;
    for (unsigned i = 0; i < n; ++i) {
        uint32_t a = i * chunk, b = std::min(M, a + chunk);
        if (a >= b) break;
        th.emplace_back(f, a, b);
    }
    for (auto& t : th) t.join();
}

inline uint32_t nib(const uint32_t* row, uint32_t k) {
    return (row[k >> 3] >> (4 * (k & 7))) & 0xFu;
}

}  // namespace

extern "C" {

// int4 GEMV with separate scale and bias arrays.
// Follows cpuRefRows, int4-gemv/src/main.mm:64-79:
//   y[m] = sum_k (S[m,k/G] * q[m,k] + B[m,k/G]) * x[k], fp64, k ascending.
// W is [M][K/8] uint32 (nibble j of word w is k = 8w+j), S/B fp16 [M][K/G], x fp16 [K].
void oracle_gemv_int4_sep(const uint32_t* W, const uint16_t* S, const uint16_t* B,
                          const uint16_t* x, double* y, uint32_t M, uint32_t K,
                          uint32_t G, int nthreads) {
    const uint32_t wpr = K / 8, gpr = K / G;
    par_rows(M, nthreads, [=](uint32_t m0, uint32_t m1) {
        for (uint32_t m = m0; m < m1; ++m) {
            const uint32_t* wr = W + (size_t)m * wpr;
            const uint16_t* sr = S + (size_t)m * gpr;
            const uint16_t* br = B + (size_t)m * gpr;
            double acc = 0.0;
            for (uint32_t k = 0; k < K; ++k) {
                uint32_t g = k / G;
                acc += (h2d(sr[g]) * (double)nib(wr, k) + h2d(br[g])) * h2d(x[k]);
            }
            y[m] = acc;
        }
    });
}

// int4 GEMV with interleaved (scale, bias) half2 pairs, SB [M][K/G][2].
// Follows int4RefRows, vq-gemv/src/main.mm:66-80 (same as refRows,
// hetero-gemv/src/main.mm:52-66).
void oracle_gemv_int4_sb(const uint32_t* W, const uint16_t* SB, const uint16_t* x,
                         double* y, uint32_t M, uint32_t K, uint32_t G, int nthreads) {
    const uint32_t wpr = K / 8, gpr = K / G;
    par_rows(M, nthreads, [=](uint32_t m0, uint32_t m1) {
        for (uint32_t m = m0; m < m1; ++m) {
            const uint32_t* wr = W + (size_t)m * wpr;
            const uint16_t* sb = SB + (size_t)m * gpr * 2;
            double acc = 0.0;
            for (uint32_t k = 0; k < K; ++k) {
                uint32_t g = k / G;
                acc += (h2d(sb[2 * g]) * (double)nib(wr, k) + h2d(sb[2 * g + 1])) * h2d(x[k]);
            }
            y[m] = acc;
        }
    });
}

// Per-32 partial sums of x, in fp32 and in the order of the reference kernel
// xsum32 (int4-gemv/src/kernels.metal:54-65): eight half4 loads, each folded as
// ((x0+x1)+x2)+x3 and then added to the running sum.
void oracle_xsum32(const uint16_t* x, float* xs, uint32_t K) {
    for (uint32_t j = 0; j < K / 32; ++j) {
        float s = 0.0f;
        for (uint32_t i = 0; i < 8; ++i) {
            const uint16_t* v = x + j * 32 + i * 4;
            float t = (float)h2d(v[0]) + (float)h2d(v[1]);
            t = t + (float)h2d(v[2]);
            t = t + (float)h2d(v[3]);
            s += t;
        }
        xs[j] = s;
    }
}

// VQ d=2 GEMV.  Follows vqRefRows, vq-gemv/src/main.mm:51-65:
//   y[m] = sum_i S[m, 2i/SG] * (C[IDX[m,i]][0]*x[2i] + C[IDX[m,i]][1]*x[2i+1])
// IDX [M][K/2] uint8, C [256][2] fp16, x fp16 [K].  S holds one fp16 scale per
// SG weights: SG = 32 is the reference layout ([M][K/32]); SG = K is one scale
// per row ([M]), the BASELINE configuration's layout.
void oracle_gemv_vq(const uint8_t* IDX, const uint16_t* C, const uint16_t* S,
                    uint32_t SG, const uint16_t* x, double* y, uint32_t M, uint32_t K,
                    int nthreads) {
    const uint32_t spr = K / SG;
    par_rows(M, nthreads, [=](uint32_t m0, uint32_t m1) {
        for (uint32_t m = m0; m < m1; ++m) {
            const uint8_t* ir = IDX + (size_t)m * (K / 2);
            const uint16_t* sr = S + (size_t)m * spr;
            double acc = 0.0;
            for (uint32_t i = 0; i < K / 2; ++i) {
                uint32_t c = ir[i];
                double s = h2d(sr[(2 * i) / SG]);
                acc += s * (h2d(C[2 * c]) * h2d(x[2 * i]) + h2d(C[2 * c + 1]) * h2d(x[2 * i + 1]));
            }
            y[m] = acc;
        }
    });
}

// Codebook decode check: out[m][2i+t] = C[IDX[m,i]][t] as raw fp16 bits.
void oracle_vq_decode(const uint8_t* IDX, const uint16_t* C, uint16_t* out, uint64_t n_idx) {
    for (uint64_t i = 0; i < n_idx; ++i) {
        out[2 * i] = C[2 * IDX[i]];
        out[2 * i + 1] = C[2 * IDX[i] + 1];
    }
}

// ---------------------------------------------------------------------------
// Fused MoE block.
//
// Layout of one expert blob (moe-fused/src/main.mm:23-25): projections gate, up,
// down at off_gate/off_up/off_down; inside each, W (uint32 [rows][K/8]) at sub_w,
// S and B ([rows][K/group]) at sub_s/sub_b and the per-row output bias BI
// ([rows]) at sub_bi.  scale_bf16 selects bf16 S/B/BI (the reference's gpt-oss
// format) or fp16 S/B (the BASELINE configuration); has_bias_out says whether
// BI exists.  router_f16 selects fp16 R and x (BASELINE) or fp32 (reference).
typedef struct {
    uint32_t hidden, inter, n_experts, top_k, group;
    uint32_t scale_bf16, has_bias_out, router_f16;
    uint32_t expert_lo, expert_hi;   // experts in [lo,hi) contribute to y (EP partial)
    uint64_t blob, off_gate, off_up, off_down, sub_w, sub_s, sub_b, sub_bi;
} OracleMoECfg;

// One projection of one expert, fp64.  Follows refProj, moe-fused/src/main.mm:46-62.
static void moe_proj(const OracleMoECfg* c, const uint8_t* blob, uint64_t proj,
                     const double* x, double* y, uint32_t M, uint32_t K, int nthreads) {
    const uint32_t* W = (const uint32_t*)(blob + proj + c->sub_w);
    const uint16_t* S = (const uint16_t*)(blob + proj + c->sub_s);
    const uint16_t* B = (const uint16_t*)(blob + proj + c->sub_b);
    const uint16_t* BI = (const uint16_t*)(blob + proj + c->sub_bi);
    const bool bf = c->scale_bf16 != 0, bias = c->has_bias_out != 0;
    const uint32_t wpr = K / 8, G = c->group, gpr = K / G;
    par_rows(M, nthreads, [=](uint32_t m0, uint32_t m1) {
        for (uint32_t m = m0; m < m1; ++m) {
            const uint32_t* wr = W + (size_t)m * wpr;
            double a = 0.0;
            for (uint32_t k = 0; k < K; ++k) {
                uint32_t g = k / G;
                a += (scale_to_d(S[(size_t)m * gpr + g], bf) * (double)nib(wr, k)
                      + scale_to_d(B[(size_t)m * gpr + g], bf)) * x[k];
            }
            y[m] = a + (bias ? scale_to_d(BI[m], bf) : 0.0);
        }
    });
}

// gpt-oss SwiGLU (moe-fused/src/main.mm:327-330, moe-pipeline/src/kernels.metal:85-98):
//   h = min(g,7) * sigmoid(1.702*min(g,7)) * (clamp(u,-7,7) + 1)
static inline double swiglu(double g, double u) {
    double gg = std::min(g, 7.0), ll = std::max(-7.0, std::min(u, 7.0));
    return (gg / (1.0 + std::exp(-1.702 * gg))) * (ll + 1.0);
}

// Whole block, fp64.  Follows moe-fused/src/main.mm:302-334:
//   logits[e] = R[e] . x; top_k by repeated strict-'>' argmax (lowest index wins
//   ties); softmax over the selected logits with max subtraction; for each
//   selected expert h = SwiGLU(gate(x), up(x)), y += w_j * down(h).
// Outputs: idx[top_k], wgt[top_k], logits[n_experts], h[top_k][inter] (may be
// null), y[hidden].  Only experts in [expert_lo, expert_hi) add into y.
int oracle_moe_block(const OracleMoECfg* c, const uint8_t* pool, const void* R,
                     const void* x, uint32_t* idx, double* wgt, double* logits,
                     double* h_out, double* y, int nthreads) {
    const uint32_t H = c->hidden, I = c->inter, E = c->n_experts, T = c->top_k;
    if (T == 0 || T > E || T > 32) return -1;
    std::vector<double> xd(H);
    for (uint32_t i = 0; i < H; ++i)
        xd[i] = c->router_f16 ? h2d(((const uint16_t*)x)[i]) : (double)((const float*)x)[i];
    for (uint32_t e = 0; e < E; ++e) {
        double s = 0.0;
        for (uint32_t k = 0; k < H; ++k) {
            double r = c->router_f16 ? h2d(((const uint16_t*)R)[(size_t)e * H + k])
                                     : (double)((const float*)R)[(size_t)e * H + k];
            s += r * xd[k];
        }
        logits[e] = s;
    }
    std::vector<double> lg(logits, logits + E), sel(T);
    for (uint32_t j = 0; j < T; ++j) {
        uint32_t bi = 0;
        double bv = -1e300;
        for (uint32_t e = 0; e < E; ++e)
            if (lg[e] > bv) { bv = lg[e]; bi = e; }
        idx[j] = bi; sel[j] = bv; lg[bi] = -1e300;
    }
    double mx = *std::max_element(sel.begin(), sel.end()), sm = 0.0;
    for (uint32_t j = 0; j < T; ++j) { wgt[j] = std::exp(sel[j] - mx); sm += wgt[j]; }
    for (uint32_t j = 0; j < T; ++j) wgt[j] /= sm;

    std::fill(y, y + H, 0.0);
    std::vector<double> g(I), u(I), hh(I), yy(H);
    for (uint32_t j = 0; j < T; ++j) {
        const uint8_t* bb = pool + (size_t)idx[j] * c->blob;
        moe_proj(c, bb, c->off_gate, xd.data(), g.data(), I, H, nthreads);
        moe_proj(c, bb, c->off_up, xd.data(), u.data(), I, H, nthreads);
        for (uint32_t i = 0; i < I; ++i) hh[i] = swiglu(g[i], u[i]);
        if (h_out) std::copy(hh.begin(), hh.end(), h_out + (size_t)j * I);
        if (idx[j] < c->expert_lo || idx[j] >= c->expert_hi) continue;
        moe_proj(c, bb, c->off_down, hh.data(), yy.data(), H, I, nthreads);
        for (uint32_t i = 0; i < H; ++i) y[i] += wgt[j] * yy[i];
    }
    return 0;
}

// One projection in gpt-oss's on-disk form (bf16 S, B and per-row output bias
// BI) against fp32 x: gemv_int4_bf16, moe-pipeline/src/kernels.metal:53-83,
// restated like refProj (moe-fused/src/main.mm:46-62) in fp64.
void oracle_gemv_int4_bf16(const uint32_t* W, const uint16_t* S, const uint16_t* B,
                           const uint16_t* BI, const float* x, double* y, uint32_t M,
                           uint32_t K, uint32_t G, int nthreads) {
    const uint32_t wpr = K / 8, gpr = K / G;
    par_rows(M, nthreads, [=](uint32_t m0, uint32_t m1) {
        for (uint32_t m = m0; m < m1; ++m) {
            const uint32_t* wr = W + (size_t)m * wpr;
            double a = 0.0;
            for (uint32_t k = 0; k < K; ++k) {
                uint32_t g = k / G;
                a += (bf2d(S[(size_t)m * gpr + g]) * (double)nib(wr, k)
                      + bf2d(B[(size_t)m * gpr + g])) * (double)x[k];
            }
            y[m] = a + bf2d(BI[m]);
        }
    });
}

// One expert as moe-pipeline's encode_expert computes it
// (moe-pipeline/src/main.mm:201-239): gate and up of fp32 x, gpt-oss SwiGLU,
// down of h; fp64 throughout.
int oracle_expert_forward(const OracleMoECfg* c, const uint8_t* blob, const float* x,
                          double* y, int nthreads) {
    const uint32_t H = c->hidden, I = c->inter;
    std::vector<double> xd(H), g(I), u(I), h(I);
    for (uint32_t k = 0; k < H; ++k) xd[k] = (double)x[k];
    moe_proj(c, blob, c->off_gate, xd.data(), g.data(), I, H, nthreads);
    moe_proj(c, blob, c->off_up, xd.data(), u.data(), I, H, nthreads);
    for (uint32_t i = 0; i < I; ++i) h[i] = swiglu(g[i], u[i]);
    moe_proj(c, blob, c->off_down, h.data(), y, H, I, nthreads);
    return 0;
}

}  // extern "C"
