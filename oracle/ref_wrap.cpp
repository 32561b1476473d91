// ref_wrap.cpp -- TEST INFRASTRUCTURE ONLY.
//
// Runs the reference's own CPU reference routines on this machine, so that the
// oracle restatement (oracle.cpp) can be checked against the real thing and the
// golden vectors under tests/golden/ come from the reference itself.
//
// ref_build.sh pulls the needed line ranges verbatim out of the reference
// sources at build time into oracle/_ref/*.inc (git-ignored, never committed)
// and compiles this file against them into oracle/_ref/libref.so.  The included
// ranges are plain C++ (the surrounding Objective-C++ harness is left behind);
// the only adaptation is `-D__fp16=_Float16`, because GCC on x86 spells the
// IEEE half type _Float16.
//
//   int4_ref.inc  : int4-gemv/src/main.mm:26, :56-92   (GemvParams, h2f, cpuRefRows, cpuRef)
//   vq_ref.inc    : vq-gemv/src/main.mm:25-26, :31-33, :48-90 (params, vqRefRows, int4RefRows, parRows)
//   moe_proj.inc  : moe-fused/src/main.mm:43-72        (bf2f, refProj, par)
//   moe_block.inc : moe-fused/src/main.mm:303-333      (router, top-k, softmax, SwiGLU, combine)

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <thread>
#include <vector>

namespace ref_int4 {
#include "int4_ref.inc"
}

namespace ref_vq {
#include "vq_ref.inc"
}

namespace ref_moe {
// moe-fused/src/main.mm:23-25 fixes the gpt-oss-120b blob layout as constants;
// here they are variables with the same names so that small synthetic blobs can
// be run through the same refProj and block code.
size_t BLOB, OFF_GATE, OFF_UP, OFF_DOWN, SUB_W, SUB_S, SUB_B, SUB_BI;
#include "moe_proj.inc"

static void block(const uint8_t* poolp, const float* R, const float* X, uint32_t HID,
                  uint32_t INTER, uint32_t NEXP, uint32_t TOPK, uint32_t* out_idx,
                  double* out_w, double* out_logits, double* out_y) {
#include "moe_block.inc"
    for (uint32_t j = 0; j < TOPK; ++j) { out_idx[j] = ridx[j]; out_w[j] = rw[j]; }
    for (uint32_t e = 0; e < NEXP; ++e) out_logits[e] = logits[e];
    for (uint32_t i = 0; i < HID; ++i) out_y[i] = yref[i];
}
}  // namespace ref_moe

extern "C" {

// cpuRef (int4-gemv/src/main.mm:81-92): separate S/B, fp64, fp32 out.
void ref_int4_cpuRef(const uint32_t* W, const uint16_t* S, const uint16_t* B,
                     const uint16_t* x, float* y, uint32_t M, uint32_t K, uint32_t G) {
    ref_int4::GemvParams P{M, K, G, K / 8, K / G, G / 32};
    ref_int4::cpuRef(W, S, B, x, y, P);
}

// cpuRefRows on a row range, single thread (the timed CPU reference arm
// spreads row ranges over its own threads).
void ref_int4_cpuRefRows(const uint32_t* W, const uint16_t* S, const uint16_t* B,
                         const uint16_t* x, float* y, uint32_t M, uint32_t K, uint32_t G,
                         uint32_t m0, uint32_t m1) {
    ref_int4::GemvParams P{M, K, G, K / 8, K / G, G / 32};
    ref_int4::cpuRefRows(W, S, B, x, y, P, m0, m1);
}

// int4RefRows over parRows (vq-gemv/src/main.mm:66-90): interleaved SB.
void ref_int4_sb(const uint32_t* W, const uint16_t* SB, const uint16_t* x, float* y,
                 uint32_t M, uint32_t K, uint32_t G) {
    ref_vq::Int4Params P{M, K, G, K / 8, K / G, G / 32};
    ref_vq::parRows(M, [&](uint32_t a, uint32_t b) { ref_vq::int4RefRows(W, SB, x, y, P, a, b); });
}

// vqRefRows over parRows (vq-gemv/src/main.mm:51-65, :81-90): per-32 scales.
void ref_vq_gemv(const uint8_t* IDX, const uint16_t* C, const uint16_t* S, const uint16_t* x,
            float* y, uint32_t M, uint32_t K) {
    ref_vq::VQParams P{M, K, K / 32, 256};
    ref_vq::parRows(M, [&](uint32_t a, uint32_t b) { ref_vq::vqRefRows(IDX, C, S, x, y, P, a, b); });
}

// The fp64 MoE block reference (moe-fused/src/main.mm:303-333) on a pool laid
// out as the given blob/offsets (bf16 S/B/BI, fp32 router and x, group 64).
void ref_moe_block(const uint8_t* pool, const float* R, const float* X, uint32_t hidden,
                   uint32_t inter, uint32_t n_experts, uint32_t top_k, uint64_t blob,
                   uint64_t off_gate, uint64_t off_up, uint64_t off_down, uint64_t sub_w,
                   uint64_t sub_s, uint64_t sub_b, uint64_t sub_bi, uint32_t* idx,
                   double* wgt, double* logits, double* y) {
    ref_moe::BLOB = blob; ref_moe::OFF_GATE = off_gate; ref_moe::OFF_UP = off_up;
    ref_moe::OFF_DOWN = off_down; ref_moe::SUB_W = sub_w; ref_moe::SUB_S = sub_s;
    ref_moe::SUB_B = sub_b; ref_moe::SUB_BI = sub_bi;
    ref_moe::block(pool, R, X, hidden, inter, n_experts, top_k, idx, wgt, logits, y);
}

}  // extern "C"
