// q4_rows.cuh -- the register-direct int4 group-affine row-dot engine: loads
// go straight to registers.  Used where the tensor-pipe tile engine
// (q4_mma.cuh) does not apply: group sizes other than 32/64/128, rows too long
// for its shared memory, MoE shapes it does not take; and by the VQ GEMV.
//
// The reference computes, per 32-weight chunk c of a row (int4-gemv/src/kernels.metal:20-30),
//     y += S[g] * sum_{k in c} q_k x_k  +  B[g] * xs[c],   xs[c] = sum_{k in c} x_k
// so the bias costs one multiply per chunk.  Here sum q_k x_k is accumulated in
// fp32 from exact fp16 products of (1024+q) or (1024+16q) with x (see
// dev::dot8_q4) and the constant part is removed once per chunk with
//     off[c] = 1024 * sum_{k in c, k even} x_k + 64 * sum_{k in c, k odd} x_k,
// which the CTA computes once into shared memory together with xs[c].
//
// Work split: one warp owns R rows at a time; lane l takes chunks l, l+32,
// l+64, ... of every row (each warp-wide 16-byte load covers 512 contiguous
// bytes of a row), U chunks per step with all R*U weight loads issued before
// any is consumed.  The activation chunk is read from shared memory once per
// step and reused for all R rows.
#pragma once
#include "graft_common.cuh"

namespace graft {
namespace dev {
namespace simple {

// Scale/bias storage of a weight matrix.
enum ScaleLayout : int {
    kSBHalf2 = 0,  // interleaved fp16 (scale, bias) pairs [rows][groups][2] (v4..v6)
    kSepF16 = 1,   // separate fp16 S[rows][groups], B[rows][groups]          (v0..v3, BASELINE MoE)
    kSepBF16 = 2   // separate bf16 S, B                                       (gpt-oss MoE blobs)
};

// Per-chunk facts kept in shared memory next to the activations.
struct ChunkMeta {
    float off;   // 1024*sum(even x) + 64*sum(odd x)
    float xsum;  // sum of the chunk's 32 activations, for the bias term
};

// Stages K fp16 activations into shared memory (swizzled, see xslot) and
// builds the per-chunk metadata.  `xs_in`, if given, supplies the bias-term
// sums (the reference's xsum32 output); otherwise they are computed here.
// Must be called by all threads of the CTA; ends with a barrier.
__device__ __forceinline__ void stage_act_f16(const uint4* __restrict__ x, int K,
                                              const float* __restrict__ xs_in,
                                              uint4* __restrict__ xsm,
                                              ChunkMeta* __restrict__ meta) {
    const int n16 = K >> 3;
    for (int i = threadIdx.x; i < n16; i += blockDim.x) xsm[xslot(i >> 2, i & 3)] = ld_ro(x + i);
    __syncthreads();
    const int chunks = K >> 5;
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
        float e = 0.f, o = 0.f;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            uint4 v = xsm[xslot(c, p)];
            uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float2 f = __half22float2(*reinterpret_cast<__half2*>(&w4[i]));
                e += f.x;
                o += f.y;
            }
        }
        ChunkMeta m;
        m.off = fmaf(1024.f, e, 64.f * o);
        m.xsum = xs_in ? xs_in[c] : e + o;
        meta[c] = m;
    }
    __syncthreads();
}

// Same, for activations that arrive as fp32 (they are rounded to fp16 first,
// as the reference's router pass does for the MoE input, moe-fused/src/kernels.metal:137).
__device__ __forceinline__ void stage_act_f32(const float* __restrict__ x, int K,
                                              uint4* __restrict__ xsm,
                                              ChunkMeta* __restrict__ meta,
                                              const float* __restrict__ xs_in = nullptr) {
    const int n16 = K >> 3;
    for (int i = threadIdx.x; i < n16; i += blockDim.x) {
        const float4* p = reinterpret_cast<const float4*>(x) + 2 * i;
        float4 a = p[0], b = p[1];
        __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
        __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
        uint4 v;
        v.x = *reinterpret_cast<uint32_t*>(&h0);
        v.y = *reinterpret_cast<uint32_t*>(&h1);
        v.z = *reinterpret_cast<uint32_t*>(&h2);
        v.w = *reinterpret_cast<uint32_t*>(&h3);
        xsm[xslot(i >> 2, i & 3)] = v;
    }
    __syncthreads();
    const int chunks = K >> 5;
    for (int c = threadIdx.x; c < chunks; c += blockDim.x) {
        float e = 0.f, o = 0.f;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
            uint4 v = xsm[xslot(c, p)];
            uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float2 f = __half22float2(*reinterpret_cast<__half2*>(&w4[i]));
                e += f.x;
                o += f.y;
            }
        }
        meta[c] = ChunkMeta{fmaf(1024.f, e, 64.f * o), xs_in ? xs_in[c] : e + o};
    }
    __syncthreads();
}

// One row's weight source: packed codes, and scale/bias rows.  For kSBHalf2 `s`
// points at the row's interleaved pairs and `b` is unused.
struct RowSrc {
    const uint8_t* w;
    const uint8_t* s;
    const uint8_t* b;
};

template <int LAYOUT>
__device__ __forceinline__ void load_sb(const RowSrc& r, int g, uint32_t& s, uint32_t& b) {
    if (LAYOUT == kSBHalf2) {
        s = ld_stream32(r.s + 4 * (size_t)g);
        b = 0;
    } else {
        s = ld_stream16(r.s + 2 * (size_t)g);
        b = ld_stream16(r.b + 2 * (size_t)g);
    }
}

template <int LAYOUT>
__device__ __forceinline__ float2 decode_sb(uint32_t s, uint32_t b) {
    if (LAYOUT == kSBHalf2) return __half22float2(*reinterpret_cast<__half2*>(&s));
    if (LAYOUT == kSepF16) return make_float2(h2f((uint16_t)s), h2f((uint16_t)b));
    return make_float2(bf2f((uint16_t)s), bf2f((uint16_t)b));
}

// acc[r] += sum over the row of w[r,k] * x[k], for this lane's chunks.  The
// caller reduces acc over the warp.  `cpg_shift` >= 0 means groups are
// 2^cpg_shift chunks long; otherwise `cpg` (chunks per group) divides.
template <int R, int U, int LAYOUT>
__device__ __forceinline__ void rows_dot(const RowSrc (&rows)[R], const uint4* __restrict__ xsm,
                                         const ChunkMeta* __restrict__ meta, int chunks,
                                         int cpg_shift, int cpg, int lane, float (&acc)[R]) {
    const int steps = (chunks + 31) >> 5;
    for (int t0 = 0; t0 < steps; t0 += U) {
        uint4 wv[U][R];
        uint32_t sv[U][R], bv[U][R];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = lane + 32 * (t0 + u);
            const bool ok = c < chunks;
            const int g = cpg_shift >= 0 ? (c >> cpg_shift) : (c / cpg);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (ok) {
                    wv[u][r] = ld_stream(rows[r].w + 16 * (size_t)c);
                    load_sb<LAYOUT>(rows[r], g, sv[u][r], bv[u][r]);
                } else {
                    wv[u][r] = make_uint4(0, 0, 0, 0);
                    sv[u][r] = bv[u][r] = 0;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = lane + 32 * (t0 + u);
            if (c < chunks) {
                const uint4 x0 = xsm[xslot(c, 0)], x1 = xsm[xslot(c, 1)];
                const uint4 x2 = xsm[xslot(c, 2)], x3 = xsm[xslot(c, 3)];
                const ChunkMeta mt = meta[c];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    float ae = 0.f, ao = 0.f;
                    dot8_q4(wv[u][r].x, x0, ae, ao);
                    dot8_q4(wv[u][r].y, x1, ae, ao);
                    dot8_q4(wv[u][r].z, x2, ae, ao);
                    dot8_q4(wv[u][r].w, x3, ae, ao);
                    const float d = fmaf(ao, 0.0625f, ae) - mt.off;
                    const float2 sb = decode_sb<LAYOUT>(sv[u][r], bv[u][r]);
                    acc[r] = fmaf(sb.x, d, fmaf(sb.y, mt.xsum, acc[r]));
                }
            }
        }
    }
}

// As rows_dot, but row r has its own staged activations (xsm[r], meta[r]) and
// rows with active[r] == false issue no loads and contribute nothing.  Used by
// the MoE down pass, where the R rows are the same output row of R different
// experts, each dotted with that expert's own hidden vector h.
template <int R, int U, int LAYOUT>
__device__ __forceinline__ void rows_dot_px(const RowSrc (&rows)[R], const bool (&active)[R],
                                            const uint4* const (&xsm)[R],
                                            const ChunkMeta* const (&meta)[R], int chunks,
                                            int cpg_shift, int cpg, int lane, float (&acc)[R]) {
    const int steps = (chunks + 31) >> 5;
    for (int t0 = 0; t0 < steps; t0 += U) {
        uint4 wv[U][R];
        uint32_t sv[U][R], bv[U][R];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = lane + 32 * (t0 + u);
            const int g = cpg_shift >= 0 ? (c >> cpg_shift) : (c / cpg);
#pragma unroll
            for (int r = 0; r < R; ++r) {
                if (active[r] && c < chunks) {
                    wv[u][r] = ld_stream(rows[r].w + 16 * (size_t)c);
                    load_sb<LAYOUT>(rows[r], g, sv[u][r], bv[u][r]);
                } else {
                    wv[u][r] = make_uint4(0, 0, 0, 0);
                    sv[u][r] = bv[u][r] = 0;
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int c = lane + 32 * (t0 + u);
            if (c < chunks) {
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if (!active[r]) continue;
                    const uint4* xr = xsm[r];
                    const ChunkMeta mt = meta[r][c];
                    float ae = 0.f, ao = 0.f;
                    dot8_q4(wv[u][r].x, xr[xslot(c, 0)], ae, ao);
                    dot8_q4(wv[u][r].y, xr[xslot(c, 1)], ae, ao);
                    dot8_q4(wv[u][r].z, xr[xslot(c, 2)], ae, ao);
                    dot8_q4(wv[u][r].w, xr[xslot(c, 3)], ae, ao);
                    const float d = fmaf(ao, 0.0625f, ae) - mt.off;
                    const float2 sb = decode_sb<LAYOUT>(sv[u][r], bv[u][r]);
                    acc[r] = fmaf(sb.x, d, fmaf(sb.y, mt.xsum, acc[r]));
                }
            }
        }
    }
}

}  // namespace simple
}  // namespace dev
}  // namespace graft
