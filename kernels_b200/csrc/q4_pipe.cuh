// q4_pipe.cuh -- the pipelined int4 group-affine row-dot engine (sm_100a),
// shared by the int4 GEMV and the MoE projections.
//
// Work unit: R weight rows x one K-part (a range of 32-weight chunks).  Every
// warp owns a ring of DEPTH shared-memory slots, one unit per slot:
//   * the R row segments of packed codes arrive by TMA 1-D bulk copy
//     (cp.async.bulk, issued by lane 0, counted in bytes on the slot mbarrier);
//   * each lane fetches the (scale, bias) words of its own chunks with cp.async
//     and signals the same mbarrier when they land (cp.async.mbarrier.arrive).
// Loads run DEPTH units ahead of the arithmetic without holding registers.
//
// A warp always works on the same K-part, so lane l always handles the same
// chunks c0+l, c0+l+32, ... (at most TMAX of them): their activations and the
// per-chunk constants stay in registers for the whole kernel.
//
// Arithmetic per chunk and row (int4-gemv/src/kernels.metal:20-30):
//     y += S * sum_k q_k x_k + B * xs_chunk
// with sum q_k x_k from dot8q (exact fp16 products, fp32 sums) minus `off`.
#pragma once
#include "async_copy.cuh"
#include "graft_common.cuh"

namespace graft {
namespace dev {

// 8 codes of `w` against the swapped activation pairs of one word:
//   ae += sum_{j even} (1024 + q_j) x_j,   ao += sum_{j odd} (1024 + 16 q_j) x_j
// Activations are held as (x4,x0) (x5,x1) (x6,x2) (x7,x3), the mirror of the
// code pairs (q0,q4) (q1,q5) (q2,q6) (q3,q7) the decode produces, so that no
// mixed-precision FMA takes both operands from high half-words (that would
// cost a register permute per FMA).
__device__ __forceinline__ void dot8q(uint32_t w, uint4 xs, float& ae, float& ao) {
    asm("{\n\t"
        ".reg .b32 t0, t1, t2, t3, w8;\n\t"
        ".reg .f16 q0, q1, q2, q3, q4, q5, q6, q7;\n\t"
        ".reg .f16 x0, x1, x2, x3, x4, x5, x6, x7;\n\t"
        "lop3.b32 t0, %2, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 t1, %2, 0x00F000F0, 0x64006400, 0xEA;\n\t"
        "shr.u32 w8, %2, 8;\n\t"
        "lop3.b32 t2, w8, 0x000F000F, 0x64006400, 0xEA;\n\t"
        "lop3.b32 t3, w8, 0x00F000F0, 0x64006400, 0xEA;\n\t"
        "mov.b32 {q0, q4}, t0;\n\t"
        "mov.b32 {q1, q5}, t1;\n\t"
        "mov.b32 {q2, q6}, t2;\n\t"
        "mov.b32 {q3, q7}, t3;\n\t"
        "mov.b32 {x4, x0}, %3;\n\t"
        "mov.b32 {x5, x1}, %4;\n\t"
        "mov.b32 {x6, x2}, %5;\n\t"
        "mov.b32 {x7, x3}, %6;\n\t"
        "fma.rn.f32.f16 %0, q0, x0, %0;\n\t"
        "fma.rn.f32.f16 %1, q1, x1, %1;\n\t"
        "fma.rn.f32.f16 %0, q4, x4, %0;\n\t"
        "fma.rn.f32.f16 %1, q5, x5, %1;\n\t"
        "fma.rn.f32.f16 %0, q2, x2, %0;\n\t"
        "fma.rn.f32.f16 %1, q3, x3, %1;\n\t"
        "fma.rn.f32.f16 %0, q6, x6, %0;\n\t"
        "fma.rn.f32.f16 %1, q7, x7, %1;\n\t"
        "}\n"
        : "+f"(ae), "+f"(ao)
        : "r"(w), "r"(xs.x), "r"(xs.y), "r"(xs.z), "r"(xs.w));
}

// Swapped-pair form of 8 activations given as {x0x1, x2x3, x4x5, x6x7}.
__device__ __forceinline__ uint4 swap_pairs(uint4 v) {
    uint4 s;
    s.x = __byte_perm(v.z, v.x, 0x5410);  // (x4 lo, x0 hi)
    s.y = __byte_perm(v.z, v.x, 0x7632);  // (x5, x1)
    s.z = __byte_perm(v.w, v.y, 0x5410);  // (x6, x2)
    s.w = __byte_perm(v.w, v.y, 0x7632);  // (x7, x3)
    return s;
}

// One lane's activations for up to TMAX chunks, with the chunk constants.
template <int TMAX>
struct LaneX {
    uint4 x[TMAX][4];
    float off[TMAX];   // 1024*sum(x at even k) + 64*sum(x at odd k)
    float xsum[TMAX];  // sum of the chunk's 32 activations (bias term)

    // Loads chunks c0+lane+32t (< c1) of x (fp16, 16-byte aligned); xs_in, if
    // given, supplies the bias-term sums (the reference's xsum32 output).
    __device__ __forceinline__ void load(const uint4* __restrict__ xg, int c0, int c1, int lane,
                                         const float* __restrict__ xs_in) {
#pragma unroll
        for (int t = 0; t < TMAX; ++t) {
            const int c = c0 + lane + 32 * t;
            float e = 0.f, o = 0.f;
            if (c < c1) {
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    x[t][p] = swap_pairs(ld_ro(xg + 4 * (size_t)c + p));
                    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&x[t][p].x));
                    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&x[t][p].y));
                    const float2 cc = __half22float2(*reinterpret_cast<const __half2*>(&x[t][p].z));
                    const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&x[t][p].w));
                    e += (a.x + a.y) + (cc.x + cc.y);
                    o += (b.x + b.y) + (d.x + d.y);
                }
            } else {
#pragma unroll
                for (int p = 0; p < 4; ++p) x[t][p] = make_uint4(0, 0, 0, 0);
            }
            off[t] = fmaf(1024.f, e, 64.f * o);
            xsum[t] = (xs_in && c < c1) ? xs_in[c] : e + o;
        }
    }

    // Same, from activations staged in shared memory as swapped pairs.
    __device__ __forceinline__ void load_smem(const uint4* __restrict__ xs, int c0, int c1,
                                              int lane) {
#pragma unroll
        for (int t = 0; t < TMAX; ++t) {
            const int c = c0 + lane + 32 * t;
            float e = 0.f, o = 0.f;
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                x[t][p] = c < c1 ? xs[4 * c + p] : make_uint4(0, 0, 0, 0);
                const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&x[t][p].x));
                const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&x[t][p].y));
                const float2 cc = __half22float2(*reinterpret_cast<const __half2*>(&x[t][p].z));
                const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&x[t][p].w));
                e += (a.x + a.y) + (cc.x + cc.y);
                o += (b.x + b.y) + (d.x + d.y);
            }
            off[t] = fmaf(1024.f, e, 64.f * o);
            xsum[t] = e + o;
        }
    }
};

// Shared-memory slot: W [R][TMAX*32 chunks][16 B] (as the bulk copies land),
// then the scale/bias words.  With SB_BULK (interleaved pairs whose row
// segments are 16-byte aligned) they land as [R][TMAX*32 groups][4 B] by bulk
// copy; otherwise each lane copies its own as [TMAX][R][NW][32 lanes][4 B].
template <int LAYOUT, int TMAX, int R>
struct Slot {
    static constexpr int NW = LAYOUT == kSBHalf2 ? 1 : 2;
    static constexpr int W_ROW = TMAX * 32 * 16;
    static constexpr int W_BYTES = R * W_ROW;
    static constexpr int SB_ROW = TMAX * 32 * 4;   // bulk layout: words per row
    static constexpr int SB_BYTES = TMAX * R * NW * 32 * 4;
    static constexpr int BYTES = W_BYTES + SB_BYTES;
};

// Arrivals per slot phase: lane 0's expect-tx arrive plus one cp.async
// completion arrive from each of the 32 lanes.
constexpr uint32_t kSlotArrivals = 33;

__device__ __forceinline__ int group_of(int c, int cpg_shift, int cpg) {
    return cpg_shift >= 0 ? (c >> cpg_shift) : (c / cpg);
}

template <int LAYOUT>
__device__ __forceinline__ float2 sb_pair(uint32_t sw, uint32_t bw, uint32_t sh_s,
                                          uint32_t sh_b) {
    if (LAYOUT == kSBHalf2) return __half22float2(*reinterpret_cast<__half2*>(&sw));
    const uint16_t s = (uint16_t)(sw >> sh_s), b = (uint16_t)(bw >> sh_b);
    if (LAYOUT == kSepF16) return make_float2(h2f(s), h2f(b));
    return make_float2(bf2f(s), bf2f(b));
}

// Per-lane constants of a warp's K-range: which chunk slots are live and the
// group of each (relative to the range's first group for bulk-copied scales).
template <int TMAX>
struct LaneK {
    int gl[TMAX];     // group index (absolute, or relative to g0 in bulk mode)
    bool live[TMAX];  // chunk c0 + lane + 32t < c1
    __device__ __forceinline__ void init(int c0, int c1, int lane, int cpg_shift, int cpg,
                                         bool relative) {
        const int g0 = relative ? group_of(c0, cpg_shift, cpg) : 0;
#pragma unroll
        for (int t = 0; t < TMAX; ++t) {
            const int c = c0 + lane + 32 * t;
            live[t] = c < c1;
            gl[t] = group_of(live[t] ? c : c0, cpg_shift, cpg) - g0;
        }
    }
};

// acc[r] += this lane's share of row r over the unit's chunks.  For separate
// scale layouts, s/b are row 0's scale and bias arrays (rows s_rs apart).
template <int LAYOUT, int TMAX, int R, bool SB_BULK>
__device__ __forceinline__ void compute_unit(const uint8_t* slot, const LaneX<TMAX>& lx,
                                             const LaneK<TMAX>& lk, int lane,
                                             const uint8_t* s, const uint8_t* b, size_t s_rs,
                                             float (&acc)[R]) {
    using SL = Slot<LAYOUT, TMAX, R>;
    const uint4* wsm = reinterpret_cast<const uint4*>(slot);
    const uint32_t* sbw = reinterpret_cast<const uint32_t*>(slot + SL::W_BYTES);
#pragma unroll
    for (int t = 0; t < TMAX; ++t) {
        if (!lk.live[t]) continue;
        const int cl = lane + 32 * t;
        // word-major over the R rows: consecutive dot8q calls feed different
        // accumulators, so the FMA chains of the rows interleave
        uint4 wv[R];
        float ae[R], ao[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            wv[r] = wsm[r * (SL::W_ROW / 16) + cl];
            ae[r] = 0.f;
            ao[r] = 0.f;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) dot8q(wv[r].x, lx.x[t][0], ae[r], ao[r]);
#pragma unroll
        for (int r = 0; r < R; ++r) dot8q(wv[r].y, lx.x[t][1], ae[r], ao[r]);
#pragma unroll
        for (int r = 0; r < R; ++r) dot8q(wv[r].z, lx.x[t][2], ae[r], ao[r]);
#pragma unroll
        for (int r = 0; r < R; ++r) dot8q(wv[r].w, lx.x[t][3], ae[r], ao[r]);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float d = fmaf(ao[r], 0.0625f, ae[r]) - lx.off[t];
            float2 sb;
            if (SB_BULK) {
                sb = sb_pair<LAYOUT>(sbw[r * (SL::SB_ROW / 4) + lk.gl[t]], 0u, 0u, 0u);
            } else if (LAYOUT == kSBHalf2) {
                sb = sb_pair<LAYOUT>(sbw[((t * R + r) * SL::NW) * 32 + lane], 0u, 0u, 0u);
            } else {
                // which half of its 4-byte word each 2-byte value sits in
                const uint32_t sh = (uint32_t)(((uintptr_t)(s + r * s_rs + 2 * (size_t)lk.gl[t]) & 2) * 8);
                const uint32_t shb = (uint32_t)(((uintptr_t)(b + r * s_rs + 2 * (size_t)lk.gl[t]) & 2) * 8);
                const int wi = ((t * R + r) * SL::NW) * 32 + lane;
                sb = sb_pair<LAYOUT>(sbw[wi], sbw[wi + 32], sh, shb);
            }
            acc[r] = fmaf(sb.x, d, fmaf(sb.y, lx.xsum[t], acc[r]));
        }
    }
}

// Per-lane issue state of a warp's unit stream: lanes 0..R-1 each bulk-copy
// one row's codes, lanes R..2R-1 one row's scale/bias segment (bulk mode);
// every lane advances its source by a constant stride per unit.
template <int LAYOUT, int TMAX, int R, bool SB_BULK>
struct Issuer {
    using SL = Slot<LAYOUT, TMAX, R>;
    const uint8_t* src;     // this lane's next source (null: copies nothing in bulk)
    size_t step;            // source advance per unit
    uint32_t dst_off;       // offset inside a slot
    uint32_t bytes;         // copy size
    uint32_t unit_tx;       // bytes per full unit (lane 0 posts it)
    int row;                // which row of the unit this lane serves
    // separate-layout / unaligned scale words, copied per lane
    const uint8_t* s_row;   // row 0 scale array of the next unit
    const uint8_t* b_row;
    size_t s_step, s_rs;

    __device__ __forceinline__ void init(const uint8_t* w0, size_t w_rs, const uint8_t* s0,
                                         const uint8_t* b0, size_t s_rs_, size_t rows_per_step,
                                         int c0, int c1, int cpg_shift, int cpg, int lane) {
        const uint32_t rowb = (uint32_t)(c1 - c0) * 16;
        const int g0 = group_of(c0, cpg_shift, cpg);
        const int ng = group_of(c1 - 1, cpg_shift, cpg) - g0 + 1;
        unit_tx = (rowb + (SB_BULK ? (uint32_t)ng * 4 : 0u)) * R;
        src = nullptr; step = 0; dst_off = 0; bytes = 0; row = R;
        if (lane < R) {
            row = lane;
            src = w0 + lane * w_rs;
            step = rows_per_step * w_rs;
            dst_off = lane * SL::W_ROW;
            bytes = rowb;
        } else if (SB_BULK && lane < 2 * R) {
            row = lane - R;
            src = s0 + row * s_rs_ + 4 * (size_t)g0;
            step = rows_per_step * s_rs_;
            dst_off = SL::W_BYTES + row * SL::SB_ROW;
            bytes = (uint32_t)ng * 4;
        }
        s_row = s0; b_row = b0; s_rs = s_rs_; s_step = rows_per_step * s_rs_;
    }

    // Issues the next unit (nrows real rows) into slot `slot` on barrier `bar`.
    __device__ __forceinline__ void issue(uint32_t slot, uint32_t bar, int nrows, int lane,
                                          const LaneK<TMAX>& lk, const uint8_t* s_end,
                                          const uint8_t* b_end) {
        if (lane == 0)
            mbar_arrive_expect_tx(bar, nrows == R ? unit_tx : unit_tx / R * (uint32_t)nrows);
        if (row < nrows && src) {
            fence_proxy_async_smem();
            bulk_g2s(slot + dst_off, src, bytes, bar);
        }
        src += step;
        if (!SB_BULK) {
            const uint32_t sbase = slot + SL::W_BYTES;
#pragma unroll
            for (int t = 0; t < TMAX; ++t) {
                if (!lk.live[t]) continue;
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if (r >= nrows) continue;
                    const uint32_t d = sbase + (uint32_t)(((t * R + r) * SL::NW) * 128 + lane * 4);
                    if (LAYOUT == kSBHalf2) {
                        cp_async4(d, s_row + r * s_rs + 4 * (size_t)lk.gl[t]);
                    } else {
                        const uint8_t* ps = s_row + r * s_rs + 2 * (size_t)lk.gl[t];
                        const uint8_t* pb = b_row + r * s_rs + 2 * (size_t)lk.gl[t];
                        // the 4-byte word holding the 2-byte value; for the last
                        // value of an array that word may end past the array, so
                        // that value is stored directly
                        const uint8_t* ws = (const uint8_t*)((uintptr_t)ps & ~(uintptr_t)3);
                        const uint8_t* wb = (const uint8_t*)((uintptr_t)pb & ~(uintptr_t)3);
                        if (ws + 4 <= s_end) cp_async4(d, ws);
                        else asm volatile("st.shared.u32 [%0], %1;" ::"r"(d),
                                          "r"((uint32_t)*(const uint16_t*)ps << (((uintptr_t)ps & 2) * 8)));
                        if (wb + 4 <= b_end) cp_async4(d + 128, wb);
                        else asm volatile("st.shared.u32 [%0], %1;" ::"r"(d + 128),
                                          "r"((uint32_t)*(const uint16_t*)pb << (((uintptr_t)pb & 2) * 8)));
                    }
                }
            }
            s_row += s_step;
            if (b_row) b_row += s_step;
        }
        cp_async_mbar_arrive(bar);
    }
};

// Issues one unit whose R rows have arbitrary sources (w_row[r] = codes of
// chunk c0 of row r, s_row/b_row = that row's scale/bias arrays); used where
// the rows of a unit do not sit at one stride (MoE gate/up pairs, gathered
// experts).  Scales are copied per lane.  Called by all 32 lanes.
template <int LAYOUT, int TMAX, int R>
__device__ __forceinline__ void issue_rows(uint32_t slot, uint32_t bar,
                                           const uint8_t* const (&w_row)[R],
                                           const uint8_t* const (&s_row)[R],
                                           const uint8_t* const (&b_row)[R], int nc, int nrows,
                                           int lane, const LaneK<TMAX>& lk, const uint8_t* s_end,
                                           const uint8_t* b_end) {
    using SL = Slot<LAYOUT, TMAX, R>;
    const uint32_t rowb = (uint32_t)nc * 16;
    if (lane == 0) mbar_arrive_expect_tx(bar, rowb * (uint32_t)nrows);
#pragma unroll
    for (int r = 0; r < R; ++r) {
        if (lane == r && r < nrows) {
            fence_proxy_async_smem();
            bulk_g2s(slot + r * SL::W_ROW, w_row[r], rowb, bar);
        }
    }
    const uint32_t sbase = slot + SL::W_BYTES;
#pragma unroll
    for (int t = 0; t < TMAX; ++t) {
        if (!lk.live[t]) continue;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (r >= nrows) continue;
            const uint32_t d = sbase + (uint32_t)(((t * R + r) * SL::NW) * 128 + lane * 4);
            if (LAYOUT == kSBHalf2) {
                cp_async4(d, s_row[r] + 4 * (size_t)lk.gl[t]);
            } else {
                const uint8_t* ps = s_row[r] + 2 * (size_t)lk.gl[t];
                const uint8_t* pb = b_row[r] + 2 * (size_t)lk.gl[t];
                const uint8_t* ws = (const uint8_t*)((uintptr_t)ps & ~(uintptr_t)3);
                const uint8_t* wb = (const uint8_t*)((uintptr_t)pb & ~(uintptr_t)3);
                if (ws + 4 <= s_end) cp_async4(d, ws);
                else asm volatile("st.shared.u32 [%0], %1;" ::"r"(d),
                                  "r"((uint32_t)*(const uint16_t*)ps << (((uintptr_t)ps & 2) * 8)));
                if (wb + 4 <= b_end) cp_async4(d + 128, wb);
                else asm volatile("st.shared.u32 [%0], %1;" ::"r"(d + 128),
                                  "r"((uint32_t)*(const uint16_t*)pb << (((uintptr_t)pb & 2) * 8)));
            }
        }
    }
    cp_async_mbar_arrive(bar);
}

// acc[r] += row r's share for rows with arbitrary scale arrays s_row/b_row
// (separate layouts), lane-copied scales.
template <int LAYOUT, int TMAX, int R>
__device__ __forceinline__ void compute_rows(const uint8_t* slot, const LaneX<TMAX>& lx,
                                             const LaneK<TMAX>& lk, int lane,
                                             const uint8_t* const (&s_row)[R],
                                             const uint8_t* const (&b_row)[R], float (&acc)[R]) {
    using SL = Slot<LAYOUT, TMAX, R>;
    const uint4* wsm = reinterpret_cast<const uint4*>(slot);
    const uint32_t* sbw = reinterpret_cast<const uint32_t*>(slot + SL::W_BYTES);
#pragma unroll
    for (int t = 0; t < TMAX; ++t) {
        if (!lk.live[t]) continue;
        const int cl = lane + 32 * t;
        uint4 wv[R];
        float ae[R], ao[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            wv[r] = wsm[r * (SL::W_ROW / 16) + cl];
            ae[r] = 0.f;
            ao[r] = 0.f;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) dot8q(wv[r].x, lx.x[t][0], ae[r], ao[r]);
#pragma unroll
        for (int r = 0; r < R; ++r) dot8q(wv[r].y, lx.x[t][1], ae[r], ao[r]);
#pragma unroll
        for (int r = 0; r < R; ++r) dot8q(wv[r].z, lx.x[t][2], ae[r], ao[r]);
#pragma unroll
        for (int r = 0; r < R; ++r) dot8q(wv[r].w, lx.x[t][3], ae[r], ao[r]);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const float d = fmaf(ao[r], 0.0625f, ae[r]) - lx.off[t];
            const int wi = ((t * R + r) * SL::NW) * 32 + lane;
            float2 sb;
            if (LAYOUT == kSBHalf2) {
                sb = sb_pair<LAYOUT>(sbw[wi], 0u, 0u, 0u);
            } else {
                const uint32_t sh = (uint32_t)(((uintptr_t)(s_row[r] + 2 * (size_t)lk.gl[t]) & 2) * 8);
                const uint32_t shb = (uint32_t)(((uintptr_t)(b_row[r] + 2 * (size_t)lk.gl[t]) & 2) * 8);
                sb = sb_pair<LAYOUT>(sbw[wi], sbw[wi + 32], sh, shb);
            }
            acc[r] = fmaf(sb.x, d, fmaf(sb.y, lx.xsum[t], acc[r]));
        }
    }
}

// Stages `n` fp16 activations (16-byte aligned, n % 32 == 0) into shared memory
// as swapped pairs (the layout LaneX holds), for LaneX::load_smem.  All
// threads of the CTA call it; no barrier inside.
__device__ __forceinline__ void stage_swapped(const uint4* __restrict__ src, int n,
                                              uint4* __restrict__ dst) {
    for (int i = threadIdx.x; i < n / 8; i += blockDim.x) dst[i] = swap_pairs(ld_ro(src + i));
}

// Reduces v[0..R-1] over the 32 lanes; afterwards lane r (r < R) holds row r's
// total.  Butterfly reduce-scatter: R-1 + log2(32/R) shuffles instead of 5R.
template <int R>
__device__ __forceinline__ float reduce_rows(float (&v)[R], int lane) {
    if (R == 1) {
        return warp_sum(v[0]);
    } else if (R == 2) {
        const bool hi = lane & 16;
        float keep = hi ? v[1] : v[0], send = hi ? v[0] : v[1];
        keep += __shfl_xor_sync(0xffffffffu, send, 16);
#pragma unroll
        for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
        // lanes 0..15 hold row 0, 16..31 row 1; move row 1 to lane 1
        const float r1 = __shfl_sync(0xffffffffu, keep, 16);
        return lane == 1 ? r1 : keep;
    } else {  // R == 4
        const bool h16 = lane & 16, h8 = lane & 8;
        float k0 = h16 ? v[2] : v[0], k1 = h16 ? v[3] : v[1];
        const float s0 = h16 ? v[0] : v[2], s1 = h16 ? v[1] : v[3];
        k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
        k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
        float keep = h8 ? k1 : k0;
        const float send = h8 ? k0 : k1;
        keep += __shfl_xor_sync(0xffffffffu, send, 8);
#pragma unroll
        for (int o = 4; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
        // row = 2*(lane>>4) + ((lane>>3)&1): rows live at lanes 0, 8, 16, 24
        const float r = __shfl_sync(0xffffffffu, keep, (lane & 3) * 8);
        return lane < 4 ? r : keep;
    }
}

// Bounded wait for a slot phase.  Returns false (and records an error bit)
// if the phase does not complete within ~2^26 probes.
__device__ __forceinline__ bool wait_slot(uint32_t bar, uint32_t parity, unsigned* err) {
    for (uint32_t i = 0; i < (1u << 26); ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (err) atomicOr(err, 1u);
    return false;
}

}  // namespace dev
}  // namespace graft
