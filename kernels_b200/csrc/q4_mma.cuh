// q4_mma.cuh -- int4 group-affine row dots on the tensor pipe (sm_100a).
//
// Work unit: a tile of 16 weight rows x one K-part of 8 groups (G*8 weights).
// A warp owns a ring of shared-memory slots; lane 0 fills a slot with TMA
// tensor copies:
//   * codes: WPG 2-D boxes of 16 rows x 128 B from a tensor map over the code
//     matrix, 128-byte swizzled (16-byte chunk c of smem line l holds chunk
//     c ^ (l % 8)), so a slot is [WPG segments][16 rows][128 B];
//   * scales: one box of 16 rows x the part's groups when the scale rows are
//     16-byte strided, else one bulk copy of the 16 rows' whole scale rows
//     (contiguous in memory) read at an offset;
// so a unit costs 2-6 copies (the TMA unit, not the bytes, limits small
// copies).  Tile row r of MMA row g is sigma(g) (and sigma(g)+8 for row g+8):
// the permutation puts the eight rows one load instruction touches on
// distinct banks under the swizzle.
//
// Arithmetic (int4-gemv/src/kernels.metal:20-30 restated per group):
//     y_row += sum_G  s_G * (sum_{k in G} q_k x_k)  +  b_G * sum_{k in G} x_k
// The inner sums run on mma.sync m16n8k16 (f16 in, f32 accumulate):
//   * A = the tile's codes decoded in registers to fp16 1024+q (low nibble of
//     each byte) or 1024+16q (high nibble) -- one lop3 per pair, no converts;
//     1024+q times an fp16 x is exact in f32, so after subtracting
//     off_G = 1024*sum(x at low nibbles) + 64*sum(x at high nibbles) the sum is
//     that of the true codes;
//   * B = x, arranged so that column n of the 8 output columns receives the
//     products of group G0+n only (the lanes feeding the other columns supply
//     zeros): the accumulator tile holds 8 groups' partial dots at once and the
//     per-group scale is applied once every 8 groups, by all 32 lanes;
//   * the k-order inside an MMA is free as long as A and B agree: lane t of a
//     row takes its word(s) of every group, and the x fragments are staged in
//     the matching order {(x0,x4), (x2,x6), (x1,x5), (x3,x7)} per word.
// A group spans WPG = G/32 words per lane (G = 32, 64, 128).
#pragma once
#include "async_copy.cuh"
#include "graft_common.cuh"

namespace graft {
namespace dev {

constexpr int kTileRows = 16;
constexpr int kWindow = 8;            // groups per unit: the 8 accumulator columns
constexpr uint32_t kTileArrivals = 1;   // lane 0 posts each unit

__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 8 codes (nibble j = weight j of the word) as fp16 pairs:
//   e0 = (1024+q0, 1024+q4)      e1 = (1024+q2, 1024+q6)
//   o0 = (1024+16q1, 1024+16q5)  o1 = (1024+16q3, 1024+16q7)
__device__ __forceinline__ void decode_word(uint32_t w, uint32_t& e0, uint32_t& e1, uint32_t& o0,
                                            uint32_t& o1) {
    const uint32_t w8 = w >> 8;
    asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(e0) : "r"(w));
    asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(o0) : "r"(w));
    asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(e1) : "r"(w8));
    asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(o1) : "r"(w8));
}

// x fragment of one word, from its 8 fp16 values {x0x1, x2x3, x4x5, x6x7}:
// {(x0,x4), (x2,x6), (x1,x5), (x3,x7)} -- B of the even and of the odd MMA.
__device__ __forceinline__ uint4 frag_of(uint4 v) {
    uint4 f;
    f.x = __byte_perm(v.x, v.z, 0x5410);
    f.y = __byte_perm(v.y, v.w, 0x5410);
    f.z = __byte_perm(v.x, v.z, 0x7632);
    f.w = __byte_perm(v.y, v.w, 0x7632);
    return f;
}

// 1024*sum(x at even positions) + 64*sum(x at odd positions) and sum(x) of one
// word's fragment, in f32.
__device__ __forceinline__ void frag_sums(uint4 f, float& even, float& odd) {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&f.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&f.y));
    const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&f.z));
    const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&f.w));
    even = (a.x + a.y) + (b.x + b.y);
    odd = (c.x + c.y) + (d.x + d.y);
}

// A K-part is one window of 8 groups: 8*WPG chunks, 128*WPG bytes of codes
// per row.  A slot's codes are [WPG segments][16 rows][128 B] (1024-byte
// aligned for the swizzle); its scales sit in a separate region of NARR
// arrays x `scap` bytes (runtime).
template <int WPG>
struct PartGeom {
    static constexpr int CHUNKS = kWindow * WPG;
    static constexpr int SEGS = WPG;
    static constexpr int CODE_BYTES = SEGS * kTileRows * 128;
};

template <int LAYOUT>
struct ScaleGeom {
    static constexpr int ES = LAYOUT == kSBHalf2 ? 4 : 2;     // bytes per scale entry
    static constexpr int NARR = LAYOUT == kSBHalf2 ? 1 : 2;   // scale arrays per row
};

// MMA row g (g < 8) reads tile row sigma(g); row g+8 reads sigma(g)+8.
template <int WPG>
__device__ __forceinline__ int tile_row_of(int g) {
    return WPG == 4 ? (g >> 1) + 4 * (g & 1) : (g < 4 ? 2 * g : 2 * (g - 4) + 1);
}

// An L2 policy under which the lines a copy brings in are evicted first: for
// streams read once per call (weights, their scales), so that they do not push
// out what is read again (activations, outputs, small tables).
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Brings a tensor map's descriptor into the TMA unit's cache ahead of use.
__device__ __forceinline__ void prefetch_tmap(const void* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* map, int x, int y,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* map, int x, int y, int z,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
        : "memory");
}
// The same copies with an L2 cache policy (l2_evict_first()).
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const void* map, int x, int y,
                                                 uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst), "l"(map), "r"(x), "r"(y),
        "r"(bar), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d_hint(uint32_t dst, const void* map, int x, int y,
                                                 int z, uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst), "l"(map), "r"(x),
        "r"(y), "r"(z), "r"(bar), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void tma_load_4d_hint(uint32_t dst, const void* map, int x, int y,
                                                 int z, int w, uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst), "l"(map), "r"(x),
        "r"(y), "r"(z), "r"(w), "r"(bar), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void tma_load_5d_hint(uint32_t dst, const void* map, int x, int y,
                                                 int z, int w, int v, uint32_t bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(dst), "l"(map),
        "r"(x), "r"(y), "r"(z), "r"(w), "r"(v), "r"(bar), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* map, int x, int y, int z,
                                            int w, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(z),
        "r"(w), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tma_load_5d(uint32_t dst, const void* map, int x, int y, int z,
                                            int w, int v, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3, %4, %5, %6}], [%7];" ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(z),
        "r"(w), "r"(v), "r"(bar)
        : "memory");
}

// One 1-D bulk copy of bytes [p, p + n) of an array ending at `end`, as the
// 16-byte-aligned span around it, into shared `dst` (the span start lands at
// dst).  Where the span would pass the array end, the aligned part goes by
// bulk copy and the ragged end by 2-byte loads (done here, before the caller
// arrives on the barrier).  Returns the bulk bytes to expect.
struct SpanCopy {
    const uint8_t* src;
    uint32_t dst, bytes;
};
__device__ __forceinline__ SpanCopy span_copy(uint32_t dst, const uint8_t* p, uint32_t n,
                                              const uint8_t* end) {
    const uintptr_t s0 = (uintptr_t)p & ~(uintptr_t)15;
    const uintptr_t s1 = ((uintptr_t)p + n + 15) & ~(uintptr_t)15;
    SpanCopy c{(const uint8_t*)s0, dst, (uint32_t)(s1 - s0)};
    if (s1 > (uintptr_t)end) {
        const uintptr_t e16 = (uintptr_t)end & ~(uintptr_t)15;
        const uintptr_t b1 = e16 > s0 ? e16 : s0;
        c.bytes = (uint32_t)(b1 - s0);
        for (uintptr_t q = b1 > (uintptr_t)p ? b1 : (uintptr_t)p; q < (uintptr_t)p + n; q += 2) {
            const uint16_t v = *reinterpret_cast<const uint16_t*>(q);
            asm volatile("st.shared.u16 [%0], %1;" ::"r"(dst + (uint32_t)(q - s0)), "h"(v));
        }
    }
    return c;
}
__device__ __forceinline__ void bulk_copy(const SpanCopy& c, uint32_t bar) {
    if (c.bytes) bulk_g2s(c.dst, c.src, c.bytes, bar);
}
__device__ __forceinline__ void bulk_copy_hint(const SpanCopy& c, uint32_t bar, uint64_t pol) {
    if (c.bytes) bulk_g2s_hint(c.dst, c.src, c.bytes, bar, pol);
}

// Where a unit's scales sit: entry G of tile row R, array a, at
// sc + a*scap + so[a] + R*rs[a] + ES*G.
struct ScaleView {
    uint32_t so[2], rs[2];
};

template <int WPG>
__device__ __forceinline__ void load_words(const uint8_t* p, uint32_t (&w)[WPG]) {
    if (WPG == 1) {
        w[0] = *reinterpret_cast<const uint32_t*>(p);
    } else if (WPG == 2) {
        const uint2 v = *reinterpret_cast<const uint2*>(p);
        w[0] = v.x; w[WPG - 1] = v.y;
    } else {
        const uint4 v = *reinterpret_cast<const uint4*>(p);
        w[0] = v.x; w[1 % WPG] = v.y; w[2 % WPG] = v.z; w[3 % WPG] = v.w;
    }
}

template <int LAYOUT>
__device__ __forceinline__ float2 scale_pair(const uint8_t* s, const uint8_t* b) {
    if (LAYOUT == kSBHalf2) return __half22float2(*reinterpret_cast<const __half2*>(s));
    const uint16_t sv = *reinterpret_cast<const uint16_t*>(s);
    const uint16_t bv = *reinterpret_cast<const uint16_t*>(b);
    if (LAYOUT == kSepF16) return make_float2(h2f(sv), h2f(bv));
    return make_float2(bf2f(sv), bf2f(bv));
}

// x in shared memory: per window of 8 groups, the word fragments (32*WPG
// uint4) followed by WPG zero fragments; a lane reads its step-j fragment at
// a fixed offset from the window base -- the real one at step j == g, the
// zeros otherwise -- so no per-step select is needed.
template <int WPG>
struct XWin {
    static constexpr int WORDS = 32 * WPG;         // fragments of one window
    static constexpr int STRIDE = WORDS + WPG;     // uint4 per window incl. zeros
    __host__ __device__ static int uint4s(int K) { return (K / (256 * WPG) + 1) * STRIDE; }
};

// Shared-memory loads by 32-bit shared address (the tile engine keeps its
// addresses in 32 bits: one integer add per load, no 64-bit pointer math).
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(a));
    return v;
}
template <int WPG>
__device__ __forceinline__ void lds_words(uint32_t a, uint32_t (&w)[WPG]) {
    if (WPG == 1) {
        w[0] = lds32(a);
    } else if (WPG == 2) {
        const uint2 v = lds64(a);
        w[0] = v.x; w[WPG - 1] = v.y;
    } else {
        const uint4 v = lds128(a);
        w[0] = v.x; w[1 % WPG] = v.y; w[2 % WPG] = v.z; w[3 % WPG] = v.w;
    }
}

// Per-lane constants of the tile engine (fixed for a warp's lifetime).
template <int WPG>
struct LaneGeom {
    int R;         // tile row read for MMA row g (and R+8 for row g+8)
    int offs[8];   // byte offset of this lane's words of group j, tile row R
    int xoff[8];   // byte offset of this lane's x fragments for step j
    __device__ __forceinline__ void init(int lane) {
        const int g = lane >> 2, t = lane & 3;
        R = tile_row_of<WPG>(g);
        const int X = R & 7, lo = 4 * WPG * t;
#pragma unroll
        for (int j = 0; j < kWindow; ++j) {
            const int o = 16 * WPG * j + lo;   // byte in the row's 128*WPG
            offs[j] = (o >> 7) * (kTileRows * 128) + R * 128 + ((((o >> 4) & 7) ^ X) << 4) + (o & 15);
            xoff[j] = 16 * (g == j ? (4 * j + t) * WPG : XWin<WPG>::WORDS);
        }
    }
};

template <int LAYOUT, int WPG, bool FULL>
__device__ __forceinline__ void tile_dot_w(const uint8_t* slot, const uint8_t* sc,
                                           const uint4* xwin, const float2* gc, int ng, int lane,
                                           const LaneGeom<WPG>& lg, const ScaleView& sv,
                                           uint32_t scap, float (&acc)[2]) {
    using SG = ScaleGeom<LAYOUT>;
    const int t = lane & 3;
    const uint32_t sa = smem_u32(slot), xa = smem_u32(xwin);
    // two MMA chains: the even nibbles (1024+q) and the odd ones (1024+16q)
    float de[4] = {0.f, 0.f, 0.f, 0.f}, dd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < kWindow; ++j) {
        if (FULL || j < ng) {
            const uint32_t pa = sa + (uint32_t)lg.offs[j], px = xa + (uint32_t)lg.xoff[j];
            uint32_t wa[WPG], wb[WPG];
            lds_words<WPG>(pa, wa);
            lds_words<WPG>(pa + 8 * 128, wb);
#pragma unroll
            for (int i = 0; i < WPG; ++i) {
                const uint4 xv = lds128(px + 16 * i);
                uint32_t ae0, ae1, ao0, ao1, be0, be1, bo0, bo1;
                decode_word(wa[i], ae0, ae1, ao0, ao1);
                decode_word(wb[i], be0, be1, bo0, bo1);
                mma_16816(de, ae0, be0, ae1, be1, xv.x, xv.y);
                mma_16816(dd, ao0, bo0, ao1, bo1, xv.z, xv.w);
            }
        }
    }
    // column 2t+c of the accumulators is group 2t+c; [q]: tile row R + 8*(q>>1)
    const uint32_t s0 = smem_u32(sc) + sv.so[0] + lg.R * sv.rs[0] + SG::ES * 2 * t;
    const uint32_t b0 = smem_u32(sc) + scap + sv.so[1] + lg.R * sv.rs[1] + SG::ES * 2 * t;
    const uint4 kq = lds128(smem_u32(gc + 2 * t));   // (off, sum x) of groups 2t, 2t+1
    const float4 kk = make_float4(__uint_as_float(kq.x), __uint_as_float(kq.y),
                                  __uint_as_float(kq.z), __uint_as_float(kq.w));
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const int c = q & 1, r = q >> 1;
        if (FULL || 2 * t + c < ng) {
            const float off = c ? kk.z : kk.x, xsum = c ? kk.w : kk.y;
            const float d = fmaf(dd[q], 0.0625f, de[q]) - off;
            const uint32_t sp = s0 + r * 8 * sv.rs[0] + SG::ES * c;
            float2 sb;
            if (LAYOUT == kSBHalf2) {
                const uint32_t v = lds32(sp);
                sb = __half22float2(*reinterpret_cast<const __half2*>(&v));
            } else {
                const uint32_t bp = b0 + r * 8 * sv.rs[1] + SG::ES * c;
                const uint32_t sv16 = lds32(sp & ~3u) >> (8 * (sp & 2));
                const uint32_t bv16 = lds32(bp & ~3u) >> (8 * (bp & 2));
                sb = LAYOUT == kSepF16 ? make_float2(h2f((uint16_t)sv16), h2f((uint16_t)bv16))
                                       : make_float2(bf2f((uint16_t)sv16), bf2f((uint16_t)bv16));
            }
            acc[r] = fmaf(sb.x, d, fmaf(sb.y, xsum, acc[r]));
        }
    }
}

// acc[0] += tile row R, acc[1] += tile row R+8 (R = sigma(g)), over the groups
// 2t, 2t+1 of the unit (g = lane/4, t = lane%4).  slot: the unit's codes; sc:
// its scale regions; xwin: the part's x window; gc: (off, sum x) of the
// part's groups (16-byte aligned); ng (<= 8): groups in the part; sv: where
// the scales sit; scap: bytes per scale region.
template <int LAYOUT, int WPG>
__device__ __forceinline__ void tile_dot(const uint8_t* slot, const uint8_t* sc,
                                         const uint4* xwin, const float2* gc, int ng, int lane,
                                         const LaneGeom<WPG>& lg, const ScaleView& sv,
                                         uint32_t scap, float (&acc)[2]) {
    if (ng == kWindow)
        tile_dot_w<LAYOUT, WPG, true>(slot, sc, xwin, gc, ng, lane, lg, sv, scap, acc);
    else
        tile_dot_w<LAYOUT, WPG, false>(slot, sc, xwin, gc, ng, lane, lg, sv, scap, acc);
}

// Sum over the 4 lanes t of a row quad; every lane ends with the total.
__device__ __forceinline__ float quad_sum(float v) {
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    return v;
}

// Stages x (n fp16 values, 16-byte aligned) as word fragments in the XWin
// layout (zero fragments included), and the per-group constants (off, sum x)
// for groups of WPG*32; xs_in, if given, supplies the per-32 sums of x for
// the bias term.  One thread per 16-byte word of x (a round of blockDim words
// at a time); a group's 4*WPG words sit on consecutive lanes, whose sums meet
// by shuffles.  Split in two so that the loads can be issued ahead of a TMA
// burst (which would otherwise queue in front of them) and finished after it:
// XStage<WPG> st; st.load(...); ...; st.store(...).  All threads of the CTA
// call both; no barrier inside (the caller syncs).
template <int WPG>
struct XStage {
    static constexpr int kHold = 4;   // rounds of words a thread loads ahead
    static constexpr int GW = 4 * WPG;   // words per group
    uint4 v[kHold];
    // 8 fp16 values of x as one 16-byte word: x16 as given, or x32 rounded
    __device__ __forceinline__ static uint4 word(const uint4* __restrict__ x16,
                                                 const float* __restrict__ x32, int i) {
        if (!x32) return ld_ro(x16 + i);
        const float4 a = __ldg(reinterpret_cast<const float4*>(x32) + 2 * i);
        const float4 b = __ldg(reinterpret_cast<const float4*>(x32) + 2 * i + 1);
        __half2 h[4] = {__floats2half2_rn(a.x, a.y), __floats2half2_rn(a.z, a.w),
                        __floats2half2_rn(b.x, b.y), __floats2half2_rn(b.z, b.w)};
        return *reinterpret_cast<uint4*>(h);
    }
    // x16: fp16 activations, or x32 (if non-null): fp32 activations, rounded to fp16
    __device__ __forceinline__ void load(const uint4* __restrict__ x, int n,
                                         const float* __restrict__ x32 = nullptr) {
        const int words = n / 8;
#pragma unroll
        for (int r = 0; r < kHold; ++r) {
            const int wd = r * (int)blockDim.x + (int)threadIdx.x;
            if (wd < words) v[r] = word(x, x32, wd);
        }
    }
    // One round: word wd (if on) into its window slot; the group's sums.
    __device__ __forceinline__ static void one(uint4 raw, int wd, bool on,
                                               const float* __restrict__ xs_in, uint4* xf,
                                               float2* gc) {
        using XW = XWin<WPG>;
        float e = 0.f, o = 0.f;
        if (on) {
            const int w = wd / XW::WORDS;
            const uint4 f = frag_of(raw);
            xf[w * XW::STRIDE + (wd - w * XW::WORDS)] = f;
            frag_sums(f, e, o);
        }
#pragma unroll
        for (int m = 1; m < GW; m <<= 1) {
            e += __shfl_xor_sync(0xffffffffu, e, m);
            o += __shfl_xor_sync(0xffffffffu, o, m);
        }
        if (on && (wd & (GW - 1)) == 0) {
            const int G = wd / GW;
            float s = e + o;
            if (xs_in) {
                s = 0.f;
                for (int c = 0; c < WPG; ++c) s += xs_in[WPG * G + c];
            }
            gc[G] = make_float2(fmaf(1024.f, e, 64.f * o), s);
        }
    }
    __device__ __forceinline__ void store(const uint4* __restrict__ x, int n,
                                          const float* __restrict__ xs_in, uint4* xf,
                                          float2* gc, const float* __restrict__ x32 = nullptr) {
        using XW = XWin<WPG>;
        const int words = n / 8, nt = (int)blockDim.x;
#pragma unroll
        for (int r = 0; r < kHold; ++r) {
            const int wd = r * nt + (int)threadIdx.x;
            if (r * nt < words) one(v[r], wd, wd < words, xs_in, xf, gc);
        }
        for (int r = kHold; r * nt < words; ++r) {   // long rows: loaded here
            const int wd = r * nt + (int)threadIdx.x;
            one(wd < words ? word(x, x32, wd) : make_uint4(0, 0, 0, 0), wd, wd < words, xs_in,
                xf, gc);
        }
        const int nwin = n / (256 * WPG) + 1;
        for (int i = threadIdx.x; i < nwin * WPG; i += blockDim.x)
            xf[(i / WPG) * XW::STRIDE + XW::WORDS + i % WPG] = make_uint4(0, 0, 0, 0);
    }
};

template <int WPG>
__device__ __forceinline__ void stage_x(const uint4* __restrict__ x, int n,
                                        const float* __restrict__ xs_in, uint4* xf, float2* gc,
                                        const float* __restrict__ x32 = nullptr) {
    XStage<WPG> st;
    st.load(x, n, x32);
    st.store(x, n, xs_in, xf, gc, x32);
}

// Wait for a slot phase, bounded in time (2 s); false (and an error bit) if
// it never completes.
constexpr uint64_t kTileWaitNs = 2000000000ull;
__device__ __forceinline__ bool wait_tile(uint32_t bar, uint32_t parity, unsigned* err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - t0 > kTileWaitNs) {
            if (err) atomicOr(err, 1u);
            return false;
        }
    }
    return true;
}

}  // namespace dev
}  // namespace graft
