// Small-M affine-quantized matmul for sm_100a:  y[M,N] = x[M,K] . deq(W)[N,K]^T.
//
// Replaces SmallMQuantizedMatmul.apply (Sources/DFlashKit/SmallMQuantizedMatmul.swift:
// 210-224) and the stock quantizedMatmul it stands in for.  The work is bound by the
// packed weight stream (M <= 16 rows against N*K quantized weights), so everything is
// arranged to move those bytes from HBM exactly once at full bandwidth:
//
//  * Three kernels per call, chained with programmatic dependent launch (PDL).  A tiny
//    prep kernel writes x, permuted into MMA fragment order, and per-group x sums into
//    the workspace.  The main kernel starts streaming weights, scales and biases before
//    its grid dependency resolves (they are never written by the preceding kernels),
//    so consecutive calls overlap launch latency and pipeline fill with the previous
//    call's tail.  A fixup kernel sums the partials of row tiles cut between CTAs.
//  * Persistent grid, one CTA per SM.  The weight matrix is cut into row tiles of 256
//    output features; the (row tile, quantization group) pairs are split into equal
//    contiguous ranges, one per CTA (stream-K).  A CTA writes a row tile it covers
//    whole straight to y; for a tile cut between CTAs it publishes an fp32 partial and
//    moves on without waiting, and the fixup kernel adds the partials in a fixed order
//    (results are deterministic).
//  * One producer thread issues TMA tile loads (cp.async.bulk.tensor, no multicast)
//    into a 4-deep shared-memory ring: per stage a [256 rows x 128 B] weight box with
//    128-byte swizzle, the matching x columns and x group sums, and the scale/bias
//    columns.
//  * 16 consumer warps: 8 slices of 32 features x 2 groups that take alternate stages.
//    Each dequantises in registers and contracts on mma.sync m16n8k16 with the weights
//    as the 16-row A operand and x (<= 8 rows per n-tile) as the n=8 B operand, so a
//    weight is read and dequantised once for all M rows.
//
// Dequantisation uses the factored form  sum_k x (q s + b) = s (sum_k x q) + b (sum_k x)
// per group, on fp16 MMA operands.  A code becomes an exact fp16 value by OR-ing its
// nibble into the mantissa of a power of two, one LOP3 per two weights: a nibble in
// bits 0-3 of a 16-bit lane over 1024.0 (0x6400) reads 1024 + q; a nibble in bits 4-7
// over 64.0 (0x5400) reads 64 + q (the mantissa step there is 1/16), so both nibbles of
// a byte unpack without a shift and a packed word costs 4 LOP3 and one shift for 8
// weights.  The ALU pipe, which those LOP3s load, is what bounds the kernel.  The MMA
// yields sum_k x (q + offset_k); the prep kernel supplies per group the sum of x and
// z = sum_k offset_k x, so  y += (s f) tmp + b xs - s z  recovers the exact sum.  For
// 8-bit codes the high nibble over 1024.0 reads 1024 + 16 q_hi, so both MMAs use the
// same x and z = 2048 xs.  x enters fp16 scaled per (row, group) by a power of two
// f^-1 that keeps it below 2^15 (exact: bf16 values fit fp16's significand), so no
// input overflows.  Within a thread's slice of a group the k order is permuted
// identically for weights and x (a sum does not depend on k order), so weights are
// consumed exactly as MLX packs them.
#include "common.cuh"

namespace dflash {
namespace qmm {

constexpr int kRows = 256;            // output features per row tile
constexpr int kRowBytes = 128;        // weight bytes per row per stage (one swizzle span)
constexpr int kRowSlices = 8;         // 32-feature slices per tile (one per consumer warp)
constexpr int kKSplit = 2;            // consumer warp groups, alternating stages
constexpr int kConsumerWarps = kRowSlices * kKSplit;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;
constexpr int kStages = 4;
constexpr int kRedPitch = kRows + 4;  // floats per m row of the reduction buffer (bank spread)
constexpr int kMaxCtas = 160;         // upper bound on the persistent grid (B200: 148 SMs)
constexpr int kMaxTiles = 4096;       // N <= kMaxTiles * kRows
constexpr int kXsWidth = 16;          // x rows covered by the per-group table (M <= 16)
constexpr int kTabWidth = 64;         // floats per group row of the table: xs[16] f[16] z[16] pad
constexpr int kBarConsumers = 1;      // named barrier id used by the consumer warps
constexpr int kPrepThreads = 256;

template <int BITS_, int GROUP_, int NT_, bool STMA_>
struct Cfg {
    static constexpr int BITS = BITS_, GROUP = GROUP_, NT = NT_;
    static constexpr bool STMA = STMA_;                  // scales/biases through TMA
    static constexpr int GB = GROUP * BITS / 8;          // bytes per row per group
    static constexpr int GPS = kRowBytes / GB;           // groups per stage
    static constexpr int TB = GB / 4;                    // bytes per thread per row per group
    static constexpr int KPS = GPS * GROUP;              // k per stage
    static constexpr int XBOX = KPS / 64;                // x boxes (64 k each) per stage
    static constexpr int XROWS = 8 * NT;
    static constexpr int W_BYTES = kRows * kRowBytes;
    static constexpr int XBOX_BYTES = XROWS * 128;
    static constexpr int X_BYTES = XBOX * XBOX_BYTES;
    static constexpr int S_BYTES = kRows * 16;           // [256 rows x 8 groups] bf16
    static constexpr int TAB_ROW = 48;                   // floats loaded per group: xs, f, z
    static constexpr int XS_BYTES = GPS * TAB_ROW * 4;   // [GPS groups x 48] fp32
    static constexpr int XS_OFF = W_BYTES + X_BYTES + 2 * S_BYTES;
    static constexpr int STAGE_BYTES = XS_OFF + 2048;
    static constexpr uint32_t TX_BYTES = W_BYTES + X_BYTES + XS_BYTES + (STMA ? 2 * S_BYTES : 0);
    static constexpr int VPT = GROUP / 4;                // values per thread per row per group
    static constexpr int PV = VPT < 16 ? VPT : 16;       // values per piece
    static constexpr int PIECES = VPT / PV;
    static constexpr int PB = PV * BITS / 8;             // bytes per piece per row
    static constexpr int PW = PB / 4;                    // 32-bit words per piece per row
    static constexpr int PSTEPS = PV / 4;                // k16 MMA steps per piece
    static constexpr int PXCH = PV / 8;                  // 8-value x chunks per piece
    // Two warps share each 32-feature slice.  With at least two groups per stage they
    // split the stage's groups (even / odd) and every consumer warp takes every stage;
    // with one group per stage they take alternate stages.
    static constexpr bool SPLIT = GPS >= 2;
    static constexpr int EMPTY_ARRIVALS = SPLIT ? kConsumerWarps : kRowSlices;
    static constexpr int RED_FLOATS = NT * 8 * kRedPitch;
    static constexpr int SMEM_BYTES = kStages * STAGE_BYTES + RED_FLOATS * 4 + 256 + 1024;
    static_assert(GPS >= 1 && GPS <= 8 && (8 % GPS) == 0, "stage/group geometry");
    static_assert(XS_BYTES <= 2048, "x group-table stage slot");
    static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte swizzle alignment");
    static_assert(SMEM_BYTES <= 232448, "shared memory budget");
};

struct Params {
    dflash_bf16* y;
    const dflash_bf16* scales;
    const dflash_bf16* biases;
    float* partials;
    int M, N, K, GT, tiles, G;
    long long U;
    int y_vec;
};

// ------------------------------------------------------------------ workspace layout
//
//   [fp32 partial tiles, kMaxCtas x 2 x 16 x 256]
//   [x group table, GT x 64 fp32][x in fragment order, M x K fp16]
// Every region is rewritten by each call before it is read, so one workspace serves
// calls of any shape and needs no initialisation.
inline size_t partials_bytes() { return (size_t)kMaxCtas * 2 * 16 * kRows * 4; }
inline size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline size_t xs_offset() { return partials_bytes(); }
inline size_t xperm_offset(int K, int group) { return xs_offset() + round_up((size_t)(K / group) * kTabWidth * 4, 1024); }
inline size_t workspace_size(int M, int K, int group) {
    return xperm_offset(K, group) + round_up((size_t)M * K * 2, 1024);
}

// ------------------------------------------------------------------ PDL
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ------------------------------------------------------------------ prep kernel
//
// x [M, K] bf16 -> xperm [M, K] fp16, each run of 8 values reordered so that one
// 16-byte load gives a thread its four B-fragment registers: 4-bit codes pair k with
// k+4 ((0,4),(1,5),(2,6),(3,7)), 8-bit codes pair k with k+2 ((0,2),(1,3),(4,6),(5,7)).
// Per (row m, group G) the values are scaled by 2^-e, e >= 0 the smallest exponent that
// keeps them below 2^15 (e = 0 for any ordinary activation), and the table row G holds
//   xs[m] = sum_k x,  f[m] = 2^e,  z[m] = sum_k offset_k x
// with offset_k = 1024 for k even and 64 for k odd (4-bit), 2048 (8-bit); rows m >= M
// hold xs = z = 0, f = 1.
template <int BITS>
__global__ void __launch_bounds__(kPrepThreads) qmm_prep_kernel(const dflash_bf16* __restrict__ x,
                                                              uint16_t* __restrict__ xperm, float* __restrict__ tab,
                                                              int M, int K, int group) {
    pdl_launch_dependents();
    pdl_wait();  // the previous call may still be reading this workspace
    const int chunks_per_row = K / 8;
    const long long idx = (long long)blockIdx.x * kPrepThreads + threadIdx.x;
    const bool live = idx < (long long)kXsWidth * chunks_per_row;
    const int m = live ? (int)(idx / chunks_per_row) : kXsWidth;
    const int c = live ? (int)(idx % chunks_per_row) : 0;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = 0.f;
    if (live && m < M) {
        const uint4 r = *reinterpret_cast<const uint4*>(x + (size_t)m * K + (size_t)c * 8);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    float sum = 0.f, z = 0.f, amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        sum += v[i];
        amax = fmaxf(amax, fabsf(v[i]));
        if constexpr (BITS == 4) z = fmaf((i & 1) ? 64.f : 1024.f, v[i], z);
    }
    if constexpr (BITS == 8) z = 2048.f * sum;
    // reduce over the group's group/8 consecutive chunks (aligned lanes of one warp)
    const int lanes = group / 8;
    for (int off = 1; off < lanes; off <<= 1) {
        sum += __shfl_xor_sync(0xffffffffu, sum, off);
        z += __shfl_xor_sync(0xffffffffu, z, off);
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    }
    int e = 0;
    if (amax >= 32768.f && amax <= 3.0e38f) e = min(ilogbf(amax) - 14, 120);
    if (live && m < M) {
        const float sc = ldexpf(1.f, -e);
        uint16_t h[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            __half hv = __float2half_rn(v[i] * sc);
            h[i] = *reinterpret_cast<uint16_t*>(&hv);
        }
        uint4 o;
        if constexpr (BITS == 4) {
            o.x = h[0] | ((uint32_t)h[4] << 16);
            o.y = h[1] | ((uint32_t)h[5] << 16);
            o.z = h[2] | ((uint32_t)h[6] << 16);
            o.w = h[3] | ((uint32_t)h[7] << 16);
        } else {
            o.x = h[0] | ((uint32_t)h[2] << 16);
            o.y = h[1] | ((uint32_t)h[3] << 16);
            o.z = h[4] | ((uint32_t)h[6] << 16);
            o.w = h[5] | ((uint32_t)h[7] << 16);
        }
        *reinterpret_cast<uint4*>(xperm + (size_t)m * K + (size_t)c * 8) = o;
    }
    if (live && (c % lanes) == 0) {
        float* row = tab + (size_t)(c / lanes) * kTabWidth;
        row[m] = sum;
        row[16 + m] = ldexpf(1.f, e);
        row[32 + m] = z;
    }
}

// ------------------------------------------------------------------ main kernel helpers

__device__ __forceinline__ long long owner_of(long long u, const Params& p) {
    return ((u + 1) * p.G - 1) / p.U;
}
__device__ __forceinline__ long long range_begin(long long c, const Params& p) {
    return c * p.U / p.G;
}

constexpr uint32_t kLoNib = 0x000F000Fu;      // nibble in bits 0-3 of each 16-bit lane
constexpr uint32_t kHiNib = 0x00F000F0u;      // nibble in bits 4-7 of each 16-bit lane
constexpr uint32_t kMag1024 = 0x64006400u;    // fp16x2 (1024, 1024): + nibble in bits 0-3 (4-7: +16q)
constexpr uint32_t kMag64 = 0x54005400u;      // fp16x2 (64, 64): + nibble in bits 4-7
// (v & mask) | mag as one LOP3: the mask is an immediate, the magic a register (left
// to itself the compiler splits this into an AND and an OR with two immediates, which
// doubles the load on the ALU pipe that bounds this kernel).
template <uint32_t MASK>
__device__ __forceinline__ uint32_t unpack(uint32_t v, uint32_t mag) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(v), "n"(MASK), "r"(mag));
    return d;
}
// A constant the compiler cannot fold, so it stays in a register.
template <uint32_t V>
__device__ __forceinline__ uint32_t pinned() {
    uint32_t d;
    asm volatile("mov.b32 %0, %1;" : "=r"(d) : "n"(V));
    return d;
}
// bf16 bits -> fp32 as an integer multiply (FMA pipe) by a register holding 65536.
__device__ __forceinline__ float bf16_to_f32_fma(uint32_t b, uint32_t k65536) {
    uint32_t d;
    asm("mul.lo.u32 %0, %1, %2;" : "=r"(d) : "r"(b), "r"(k65536));
    return __uint_as_float(d);
}

// Registers pinned for the unpack and the scale conversion.
struct Pinned {
    uint32_t mag1024, mag64, k65536;
};
__device__ __forceinline__ Pinned make_pinned() {
    return Pinned{pinned<kMag1024>(), pinned<kMag64>(), pinned<65536u>()};
}

// Fragment row g of 16-row block i of a warp's 32-feature slice maps to feature row
//     rb + 16 i + 2 sigma(g) + h        (h = 0: fragment rows 0..7, h = 1: rows 8..15)
// sigma spreads the 128-byte swizzle keys (row & 7) of the rows a half-warp (LDS.64)
// or quarter-warp (LDS.128) reads, so the weight reads of a warp hit distinct banks.
__device__ __forceinline__ int sigma(int g) { return (g & 4) | ((g & 1) << 1) | ((g >> 1) & 1); }

// Per-thread offsets of the fragment layout, computed once per CTA.
template <class C>
struct LaneLayout {
    int row[2];                                   // feature row of (i = 0, h); i = 1 adds 16
    uint32_t wofs[2];                             // stage-relative byte offset of group 0, piece 0
    uint32_t xofs[C::NT][C::PIECES][C::PXCH];     // offset within the x region, group 0
};

template <class C>
__device__ __forceinline__ LaneLayout<C> lane_layout(int rb, int g, int tq) {
    LaneLayout<C> L;
    const uint32_t T = tq * C::TB;  // this thread's byte slice of a row's group
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int r = rb + 2 * sigma(g) + h;
        L.row[h] = r;
        L.wofs[h] = r * kRowBytes + ((((T >> 4) ^ (r & 7))) << 4) + (T & 15);
    }
#pragma unroll
    for (int j = 0; j < C::NT; ++j) {
        const int m = 8 * j + g;
#pragma unroll
        for (int pc = 0; pc < C::PIECES; ++pc)
#pragma unroll
            for (int c = 0; c < C::PXCH; ++c) {
                const int kt = tq * C::VPT + pc * C::PV + 8 * c;  // k within group 0 of the stage
                L.xofs[j][pc][c] = (kt >> 6) * C::XBOX_BYTES + m * 128 + ((((kt & 63) >> 3) ^ (m & 7)) << 4);
            }
    }
    return L;
}

// Compile-time parts of the weight address of (group gl, piece pc): XOR into the
// swizzled chunk bits, plus an in-chunk byte offset.
template <class C> __device__ __forceinline__ constexpr uint32_t w_xor(int gl, int pc) {
    return (uint32_t)(gl * C::GB + ((pc * C::PB) & ~15));
}
template <class C> __device__ __forceinline__ constexpr uint32_t w_add(int pc) {
    return (uint32_t)((pc * C::PB) & 15);
}
// x address of group gl: XOR of the chunk bits (groups of 32) and a whole-box offset.
template <class C> __device__ __forceinline__ constexpr uint32_t x_xor(int gl) {
    return (uint32_t)(((gl * C::GROUP) & 63) << 1);
}
template <class C> __device__ __forceinline__ constexpr uint32_t x_add(int gl) {
    return (uint32_t)(((gl * C::GROUP) >> 6) * C::XBOX_BYTES);
}

template <int PB>
__device__ __forceinline__ void lds_words(uint32_t* dst, uint32_t addr) {
    if constexpr (PB == 4) {
        dst[0] = lds32(addr);
    } else if constexpr (PB == 8) {
        const uint2 v = lds64(addr);
        dst[0] = v.x;
        dst[1] = v.y;
    } else {
        const uint4 v = lds128(addr);
        dst[0] = v.x;
        dst[1] = v.y;
        dst[2] = v.z;
        dst[3] = v.w;
    }
}

// D = A * B (+ D unless FIRST), m16n8k16 fp16 -> fp32.
template <bool FIRST>
__device__ __forceinline__ void mma_step(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    if constexpr (FIRST) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
            "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %10, %10, %10};"
            : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.f));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
            "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

// One quantization group (index gl within the stage) for one consumer warp:
// 32 feature rows x GROUP k, all M rows.  wb[h] = stage base + wofs[h]; xb = x region;
// sb[h] = scale-tile address of row[h] at this stage's group 0; xsb = this thread's
// x group-sum slot (group 0, n-tile 0) in the stage.
template <class C>
__device__ __forceinline__ void consume_group(const LaneLayout<C>& L, const Pinned& P, const uint32_t (&wb)[2],
                                              uint32_t xb, const uint32_t (&sb)[2], uint32_t xsb, int gl, int G,
                                              int tile_row0, const Params& p, float (&acc)[2][C::NT][4]) {
    float tmp[2][C::NT][4];
#pragma unroll
    for (int pc = 0; pc < C::PIECES; ++pc) {
        // B fragments, already in register order (prep kernel)
        uint32_t xf[C::NT][C::PXCH][4];
#pragma unroll
        for (int j = 0; j < C::NT; ++j)
#pragma unroll
            for (int c = 0; c < C::PXCH; ++c) {
                const uint4 r = lds128(xb + ((L.xofs[j][pc][c] ^ x_xor<C>(gl)) + x_add<C>(gl)));
                xf[j][c][0] = r.x;
                xf[j][c][1] = r.y;
                xf[j][c][2] = r.z;
                xf[j][c][3] = r.w;
            }
        // A operand source: packed words of the 4 feature rows (i, h).
        uint32_t wv[2][2][C::PW];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t a = (wb[h] ^ w_xor<C>(gl, pc)) + w_add<C>(pc);
            lds_words<C::PB>(wv[0][h], a);
            lds_words<C::PB>(wv[1][h], a + 16 * kRowBytes);
        }
#pragma unroll
        for (int s = 0; s < C::PSTEPS; ++s) {
            const bool first = (pc == 0 && s == 0);
            if constexpr (C::BITS == 4) {
                // word w of the piece: step 2w uses nibbles (0,4) and (1,5), step 2w+1
                // nibbles (2,6) and (3,7) of the word shifted right by 8.
                const int w = s >> 1, q = (s & 1) * 2;
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const uint32_t v0 = q ? (wv[i][0][w] >> 8) : wv[i][0][w];
                    const uint32_t v1 = q ? (wv[i][1][w] >> 8) : wv[i][1][w];
                    const uint32_t a0 = unpack<kLoNib>(v0, P.mag1024), a1 = unpack<kLoNib>(v1, P.mag1024);
                    const uint32_t a2 = unpack<kHiNib>(v0, P.mag64), a3 = unpack<kHiNib>(v1, P.mag64);
#pragma unroll
                    for (int j = 0; j < C::NT; ++j) {
                        const uint32_t b0 = xf[j][w][q], b1 = xf[j][w][q + 1];
                        if (first) mma_step<true>(tmp[i][j], a0, a1, a2, a3, b0, b1);
                        else mma_step<false>(tmp[i][j], a0, a1, a2, a3, b0, b1);
                    }
                }
            } else {
                // word s: bytes (0,2) in place and bytes (1,3) shifted right by 8; the low
                // nibbles read 1024 + q_lo, the high ones 1024 + 16 q_hi, both against x.
                const int w = s, c = s >> 1, q = (s & 1) * 2;
#pragma unroll
                for (int i = 0; i < 2; ++i) {
                    const uint32_t w0 = wv[i][0][w], w1 = wv[i][1][w];
                    const uint32_t t0 = w0 >> 8, t1 = w1 >> 8;
                    const uint32_t l0 = unpack<kLoNib>(w0, P.mag1024), l1 = unpack<kLoNib>(w1, P.mag1024);
                    const uint32_t l2 = unpack<kLoNib>(t0, P.mag1024), l3 = unpack<kLoNib>(t1, P.mag1024);
                    const uint32_t u0 = unpack<kHiNib>(w0, P.mag1024), u1 = unpack<kHiNib>(w1, P.mag1024);
                    const uint32_t u2 = unpack<kHiNib>(t0, P.mag1024), u3 = unpack<kHiNib>(t1, P.mag1024);
#pragma unroll
                    for (int j = 0; j < C::NT; ++j) {
                        const uint32_t b0 = xf[j][c][q], b1 = xf[j][c][q + 1];
                        if (first) mma_step<true>(tmp[i][j], l0, l1, l2, l3, b0, b1);
                        else mma_step<false>(tmp[i][j], l0, l1, l2, l3, b0, b1);
                        mma_step<false>(tmp[i][j], u0, u1, u2, u3, b0, b1);
                    }
                }
            }
        }
    }

    // group table for this thread's output columns m = 8j + 2tq, 8j + 2tq + 1
    float xs[C::NT][2], xf2[C::NT][2], zz[C::NT][2];
#pragma unroll
    for (int j = 0; j < C::NT; ++j) {
        const uint32_t a = xsb + (gl * C::TAB_ROW + 8 * j) * 4;
        const uint2 v0 = lds64(a), v1 = lds64(a + 16 * 4), v2 = lds64(a + 32 * 4);
        xs[j][0] = __uint_as_float(v0.x);
        xs[j][1] = __uint_as_float(v0.y);
        xf2[j][0] = __uint_as_float(v1.x);
        xf2[j][1] = __uint_as_float(v1.y);
        zz[j][0] = __uint_as_float(v2.x);
        zz[j][1] = __uint_as_float(v2.y);
    }
    // acc += s (f tmp - z) + b xs, per feature row.
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float s, b;
            if constexpr (C::STMA) {
                const uint32_t a = sb[h] + i * 16 * 16 + 2 * gl;
                s = bf16_to_f32_fma(lds16(a), P.k65536);
                b = bf16_to_f32_fma(lds16(a + C::S_BYTES), P.k65536);
            } else {
                const int n = tile_row0 + L.row[h] + 16 * i;
                if (n < p.N) {
                    const size_t idx = (size_t)n * p.GT + G;
                    s = bf16_bits_to_float(__ldg(p.scales + idx));
                    b = bf16_bits_to_float(__ldg(p.biases + idx));
                } else {
                    s = 0.f;
                    b = 0.f;
                }
            }
#pragma unroll
            for (int j = 0; j < C::NT; ++j)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const float t = fmaf(xf2[j][e], tmp[i][j][2 * h + e], -zz[j][e]);
                    acc[i][j][2 * h + e] = fmaf(s, t, fmaf(b, xs[j][e], acc[i][j][2 * h + e]));
                }
        }
}

// This warp's groups of one stage: all of them (PAR < 0) or those with gl % 2 == PAR.
// CHECK: the stage is the first or last of a segment and some of its groups fall
// outside [ga, gb).
template <class C, bool CHECK, int PAR>
__device__ __forceinline__ void consume_stage(const LaneLayout<C>& L, const Pinned& P, uint32_t st, int sc, int ga,
                                              int gb, int tq, int tile_row0, const Params& p,
                                              float (&acc)[2][C::NT][4]) {
    const uint32_t wb[2] = {st + L.wofs[0], st + L.wofs[1]};
    const uint32_t xb = st + C::W_BYTES;
    const uint32_t s0 = st + C::W_BYTES + C::X_BYTES + 2 * ((sc * C::GPS) & 7);
    const uint32_t sb[2] = {s0 + L.row[0] * 16, s0 + L.row[1] * 16};
    const uint32_t xsb = st + C::XS_OFF + 2 * tq * 4;
#pragma unroll
    for (int gl = 0; gl < C::GPS; ++gl) {
        if (PAR >= 0 && (gl & 1) != PAR) continue;
        const int G = sc * C::GPS + gl;
        if (CHECK && (G < ga || G >= gb)) continue;
        consume_group<C>(L, P, wb, xb, sb, xsb, gl, G, tile_row0, p, acc);
    }
}

// Writes the fp32 tile in `red` ([NT*8][kRedPitch]) to y as bf16.
template <class C>
__device__ __forceinline__ void write_tile(const float* red, int t, const Params& p, int ctid) {
    const int n0 = t * kRows;
    if (p.y_vec) {
        for (int idx = ctid; idx < C::NT * 8 * (kRows / 8); idx += kConsumerThreads) {
            const int m = idx / (kRows / 8), r0 = (idx % (kRows / 8)) * 8;
            if (m >= p.M || n0 + r0 >= p.N) continue;
            const float4 a = *reinterpret_cast<const float4*>(red + m * kRedPitch + r0);
            const float4 b = *reinterpret_cast<const float4*>(red + m * kRedPitch + r0 + 4);
            __nv_bfloat162 o0 = __floats2bfloat162_rn(a.x, a.y), o1 = __floats2bfloat162_rn(a.z, a.w);
            __nv_bfloat162 o2 = __floats2bfloat162_rn(b.x, b.y), o3 = __floats2bfloat162_rn(b.z, b.w);
            uint4 v;
            v.x = *reinterpret_cast<uint32_t*>(&o0);
            v.y = *reinterpret_cast<uint32_t*>(&o1);
            v.z = *reinterpret_cast<uint32_t*>(&o2);
            v.w = *reinterpret_cast<uint32_t*>(&o3);
            *reinterpret_cast<uint4*>(p.y + (size_t)m * p.N + n0 + r0) = v;
        }
    } else {
        for (int idx = ctid; idx < C::NT * 8 * kRows; idx += kConsumerThreads) {
            const int m = idx / kRows, r = idx % kRows;
            if (m >= p.M || n0 + r >= p.N) continue;
            __nv_bfloat16 o = __float2bfloat16_rn(red[m * kRedPitch + r]);
            p.y[(size_t)m * p.N + n0 + r] = *reinterpret_cast<uint16_t*>(&o);
        }
    }
}

template <class C>
__global__ void __launch_bounds__(kThreads, 1)
    qmm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x,
               const __grid_constant__ CUtensorMap tm_s, const __grid_constant__ CUtensorMap tm_b,
               const __grid_constant__ CUtensorMap tm_xs, const Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* red = reinterpret_cast<float*>(smem + kStages * C::STAGE_BYTES);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * C::STAGE_BYTES + C::RED_FLOATS * 4);
    uint64_t* empty = full + kStages;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kStages);


    pdl_launch_dependents();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], C::EMPTY_ARRIVALS);
        }
        *abort_flag = 0;

        fence_barrier_init();
    }
    __syncthreads();

    const long long c = blockIdx.x;
    const long long u0 = range_begin(c, p), u1 = range_begin(c + 1, p);
    const int first_tile = (int)(u0 / p.GT);

    if (warp == kConsumerWarps) {
        // ------------------------------------------------------------ producer
        if (lane != 0) return;
        prefetch_tensormap(&tm_w);
        prefetch_tensormap(&tm_x);
        prefetch_tensormap(&tm_xs);
        if constexpr (C::STMA) {
            prefetch_tensormap(&tm_s);
            prefetch_tensormap(&tm_b);
        }
        // Stage j covers groups [sc*GPS, sc*GPS+GPS) of row tile t.  The weight-side
        // loads (W, scales, biases) of the first ring fill go out before the grid
        // dependency resolves; x and its group sums only after it.
        int j = 0;
        bool ok = true, dep_resolved = false;
        int pend_sc[kStages];
        int n_pend = 0;
        auto issue_x = [&](int slot, int sc) {
            uint8_t* st = smem + slot * C::STAGE_BYTES;
#pragma unroll
            for (int b = 0; b < C::XBOX; ++b)
                tma_load_2d(st + C::W_BYTES + b * C::XBOX_BYTES, &tm_x, &full[slot], sc * C::KPS + 64 * b, 0);
            tma_load_2d(st + C::XS_OFF, &tm_xs, &full[slot], 0, sc * C::GPS);
        };
        for (long long u = u0; u < u1 && ok;) {
            const int t = (int)(u / p.GT);
            const int ga = (int)(u - (long long)t * p.GT);
            const int gb = (int)min((long long)p.GT, u1 - (long long)t * p.GT);
            for (int sc = ga / C::GPS; sc < (gb + C::GPS - 1) / C::GPS; ++sc, ++j) {
                const int slot = j % kStages;
                const uint32_t ph = (uint32_t)(j / kStages) & 1u;
                if (!dep_resolved && j == kStages) {
                    pdl_wait();
                    dep_resolved = true;
                    for (int i = 0; i < n_pend; ++i) issue_x(i, pend_sc[i]);
                }
                if (!mbar_wait_bounded(&empty[slot], ph ^ 1u, abort_flag, DFLASH_DEVERR_QMM_PIPELINE)) {
                    ok = false;
                    break;
                }
                uint8_t* st = smem + slot * C::STAGE_BYTES;
                mbar_arrive_expect_tx(&full[slot], C::TX_BYTES);
                tma_load_2d(st, &tm_w, &full[slot], sc * (kRowBytes / 4), t * kRows);
                if constexpr (C::STMA) {
                    const int gx = (sc * C::GPS) & ~7;
                    tma_load_2d(st + C::W_BYTES + C::X_BYTES, &tm_s, &full[slot], gx, t * kRows);
                    tma_load_2d(st + C::W_BYTES + C::X_BYTES + C::S_BYTES, &tm_b, &full[slot], gx, t * kRows);
                }
                if (dep_resolved) {
                    issue_x(slot, sc);
                } else {
                    pend_sc[n_pend++] = sc;
                }
            }
            u = (long long)t * p.GT + gb;
        }
        if (!dep_resolved) {
            pdl_wait();
            for (int i = 0; i < n_pend; ++i) issue_x(i, pend_sc[i]);
        }
        // Drain: do not leave the CTA while issued copies may still be landing.
        for (int i = max(0, j - kStages); i < j; ++i) {
            const int slot = i % kStages;
            const uint32_t ph = (uint32_t)(i / kStages) & 1u;
            const unsigned long long t0 = globaltimer_ns();
            while (!mbar_try_wait(&full[slot], ph) && globaltimer_ns() - t0 < kWaitLimitNs) {
            }
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    pdl_wait();  // y and the workspace may still be in use by the previous call
    const int rs = warp % kRowSlices, par = warp / kRowSlices;
    const int g = lane >> 2, tq = lane & 3;
    const int rb = rs * 32;
    const LaneLayout<C> L = lane_layout<C>(rb, g, tq);
    const Pinned P = make_pinned();
    const int ctid = threadIdx.x;  // 0 .. kConsumerThreads-1
    int j = 0;

    for (long long u = u0; u < u1;) {
        const int t = (int)(u / p.GT);
        const int ga = (int)(u - (long long)t * p.GT);
        const int gb = (int)min((long long)p.GT, u1 - (long long)t * p.GT);
        const int tile_row0 = t * kRows;

        float acc[2][C::NT][4];
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int jj = 0; jj < C::NT; ++jj)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[i][jj][e] = 0.f;

        for (int sc = ga / C::GPS; sc < (gb + C::GPS - 1) / C::GPS; ++sc, ++j) {
            if (!C::SPLIT && (j % kKSplit) != par) continue;
            const int slot = j % kStages;
            const uint32_t ph = (uint32_t)(j / kStages) & 1u;
            // mma.sync below is warp-collective: every lane must take the same branch
            const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(&full[slot], ph, abort_flag,
                                                                       DFLASH_DEVERR_QMM_PIPELINE));
            if (ok) {
                const uint32_t st = smem_u32(smem + slot * C::STAGE_BYTES);
                const bool whole = sc * C::GPS >= ga && sc * C::GPS + C::GPS <= gb;
                if constexpr (C::SPLIT) {
                    if (par == 0) {
                        if (whole) consume_stage<C, false, 0>(L, P, st, sc, ga, gb, tq, tile_row0, p, acc);
                        else consume_stage<C, true, 0>(L, P, st, sc, ga, gb, tq, tile_row0, p, acc);
                    } else {
                        if (whole) consume_stage<C, false, 1>(L, P, st, sc, ga, gb, tq, tile_row0, p, acc);
                        else consume_stage<C, true, 1>(L, P, st, sc, ga, gb, tq, tile_row0, p, acc);
                    }
                } else {
                    if (whole) consume_stage<C, false, -1>(L, P, st, sc, ga, gb, tq, tile_row0, p, acc);
                    else consume_stage<C, true, -1>(L, P, st, sc, ga, gb, tq, tile_row0, p, acc);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
        }

        // ---- reduce the two stage-parity halves into `red`
        named_bar_sync(kBarConsumers, kConsumerThreads);
        if (par == 1) {
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int jj = 0; jj < C::NT; ++jj)
#pragma unroll
                        for (int e = 0; e < 2; ++e)
                            red[(8 * jj + 2 * tq + e) * kRedPitch + L.row[h] + 16 * i] = acc[i][jj][2 * h + e];
        }
        named_bar_sync(kBarConsumers, kConsumerThreads);
        if (par == 0) {
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int jj = 0; jj < C::NT; ++jj)
#pragma unroll
                        for (int e = 0; e < 2; ++e)
                            red[(8 * jj + 2 * tq + e) * kRedPitch + L.row[h] + 16 * i] += acc[i][jj][2 * h + e];
        }
        named_bar_sync(kBarConsumers, kConsumerThreads);

        if (ga == 0 && gb == p.GT) {
            write_tile<C>(red, t, p, ctid);
        } else {
            // ---- a tile cut between CTAs: publish this CTA's share as an fp32 partial
            // in its slot (0: the tile is this CTA's first segment, 1: its last); the
            // fixup kernel adds the contributors' partials in CTA order.
            constexpr int TILE_FLOATS = C::NT * 8 * kRows;
            const int slot = (t == first_tile) ? 0 : 1;
            float* dst = p.partials + (size_t)(c * 2 + slot) * TILE_FLOATS;
            for (int idx = ctid; idx < TILE_FLOATS / 4; idx += kConsumerThreads) {
                const int m = idx / (kRows / 4), r4 = (idx % (kRows / 4)) * 4;
                __stcg(reinterpret_cast<float4*>(dst + m * kRows + r4),
                       *reinterpret_cast<const float4*>(red + m * kRedPitch + r4));
            }
        }
        named_bar_sync(kBarConsumers, kConsumerThreads);
        u = (long long)t * p.GT + gb;
    }
}

// ------------------------------------------------------------------ fixup kernel
//
// One block per row tile.  A tile covered whole by one CTA was written by the main
// kernel; for a tile cut between CTAs cf..cl the block sums their partials (slot 0 when
// the tile is the CTA's first segment, else 1) in CTA order and writes y.
template <int NT>
__global__ void __launch_bounds__(256) qmm_fixup_kernel(const Params p) {
    pdl_launch_dependents();
    pdl_wait();  // the main kernel's partials
    const int t = blockIdx.x;
    const long long cf = owner_of((long long)t * p.GT, p);
    const long long cl = owner_of((long long)(t + 1) * p.GT - 1, p);
    if (cf == cl) return;
    constexpr int TILE_FLOATS = NT * 8 * kRows;
    const int n0 = t * kRows;
    for (int idx = threadIdx.x; idx < TILE_FLOATS / 4; idx += blockDim.x) {
        const int m = idx / (kRows / 4), r4 = (idx % (kRows / 4)) * 4;
        if (m >= p.M) break;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        for (long long cc = cf; cc <= cl; ++cc) {
            const int sl = ((int)(range_begin(cc, p) / p.GT) == t) ? 0 : 1;
            const float4 q = __ldcg(reinterpret_cast<const float4*>(p.partials + (size_t)(cc * 2 + sl) * TILE_FLOATS +
                                                                    m * kRows + r4));
            v.x += q.x;
            v.y += q.y;
            v.z += q.z;
            v.w += q.w;
        }
        const float vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int n = n0 + r4 + e;
            if (n < p.N) {
                __nv_bfloat16 o = __float2bfloat16_rn(vv[e]);
                p.y[(size_t)m * p.N + n] = *reinterpret_cast<uint16_t*>(&o);
            }
        }
    }
}

// ------------------------------------------------------------------ host side

struct Shape {
    int M, N, K, group, bits;
};

inline int n_tiles(int N) { return (N + kRows - 1) / kRows; }

// Launch with programmatic stream serialization: the kernel may begin while the
// previous kernel in the stream is still running; griddepcontrol.wait in the kernel
// orders everything that depends on it.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <class C>
int launch(const Shape& s, const dflash_bf16* x, const uint32_t* w, const dflash_bf16* scales,
           const dflash_bf16* biases, dflash_bf16* y, void* ws, cudaStream_t stream) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    std::call_once(once, [] {
        attr_err = cudaFuncSetAttribute(qmm_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        C::SMEM_BYTES);
    });
    if (attr_err != cudaSuccess)
        return fail(DFLASH_ERR_CUDA, "cudaFuncSetAttribute(qmm): %s", cudaGetErrorString(attr_err));

    uint8_t* wsb = reinterpret_cast<uint8_t*>(ws);
    float* xs = reinterpret_cast<float*>(wsb + xs_offset());
    uint16_t* xperm = reinterpret_cast<uint16_t*>(wsb + xperm_offset(s.K, s.group));
    const int GT = s.K / s.group;

    CUtensorMap tm_w, tm_x, tm_s, tm_b, tm_xs;
    int st;
    const uint64_t words = (uint64_t)s.K * s.bits / 32;
    st = encode_tensor_map_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, words, (uint64_t)s.N, words * 4,
                              kRowBytes / 4, kRows, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = encode_tensor_map_2d(&tm_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xperm, (uint64_t)s.K, (uint64_t)s.M,
                              (uint64_t)s.K * 2, 64, C::XROWS, CU_TENSOR_MAP_SWIZZLE_128B);
    if (st) return st;
    st = encode_tensor_map_2d(&tm_xs, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, xs, kTabWidth, (uint64_t)GT, kTabWidth * 4,
                              C::TAB_ROW, C::GPS, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (st) return st;
    if constexpr (C::STMA) {
        st = encode_tensor_map_2d(&tm_s, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, scales, (uint64_t)GT, (uint64_t)s.N,
                                  (uint64_t)GT * 2, 8, kRows, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
        st = encode_tensor_map_2d(&tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, biases, (uint64_t)GT, (uint64_t)s.N,
                                  (uint64_t)GT * 2, 8, kRows, CU_TENSOR_MAP_SWIZZLE_NONE);
        if (st) return st;
    } else {
        tm_s = tm_w;
        tm_b = tm_w;
    }

    int dev = 0;
    DFLASH_CUDA_TRY(cudaGetDevice(&dev));
    Params p;
    p.y = y;
    p.scales = scales;
    p.biases = biases;
    p.partials = reinterpret_cast<float*>(wsb);
    p.M = s.M;
    p.N = s.N;
    p.K = s.K;
    p.GT = GT;
    p.tiles = n_tiles(s.N);
    p.U = (long long)p.tiles * p.GT;
    long long G = sm_count(dev);
    if (G > kMaxCtas) G = kMaxCtas;
    if (G > p.U) G = p.U;
    p.G = (int)G;
    p.y_vec = (s.N % 8 == 0) && aligned16(y);

    const long long prep_threads = (long long)kXsWidth * (s.K / 8);
    const int prep_blocks = (int)((prep_threads + kPrepThreads - 1) / kPrepThreads);
    if (s.bits == 4)
        DFLASH_CUDA_TRY(launch_pdl(qmm_prep_kernel<4>, dim3(prep_blocks), dim3(kPrepThreads), 0, stream, x, xperm, xs,
                                   s.M, s.K, s.group));
    else
        DFLASH_CUDA_TRY(launch_pdl(qmm_prep_kernel<8>, dim3(prep_blocks), dim3(kPrepThreads), 0, stream, x, xperm, xs,
                                   s.M, s.K, s.group));
    DFLASH_CUDA_TRY(launch_pdl(qmm_kernel<C>, dim3(p.G), dim3(kThreads), (size_t)C::SMEM_BYTES, stream, tm_w, tm_x,
                               tm_s, tm_b, tm_xs, p));
    DFLASH_CUDA_TRY(launch_pdl(qmm_fixup_kernel<C::NT>, dim3(p.tiles), dim3(256), 0, stream, p));
    return DFLASH_OK;
}

template <int BITS, int GROUP, int NT>
int dispatch_stma(const Shape& s, const dflash_bf16* x, const uint32_t* w, const dflash_bf16* sc,
                  const dflash_bf16* bi, dflash_bf16* y, void* ws, cudaStream_t st) {
    const bool stma = ((s.K / s.group) % 8 == 0) && aligned16(sc) && aligned16(bi);
    if (stma) return launch<Cfg<BITS, GROUP, NT, true>>(s, x, w, sc, bi, y, ws, st);
    return launch<Cfg<BITS, GROUP, NT, false>>(s, x, w, sc, bi, y, ws, st);
}

template <int BITS, int GROUP>
int dispatch_nt(const Shape& s, const dflash_bf16* x, const uint32_t* w, const dflash_bf16* sc,
                const dflash_bf16* bi, dflash_bf16* y, void* ws, cudaStream_t st) {
    if (s.M <= 8) return dispatch_stma<BITS, GROUP, 1>(s, x, w, sc, bi, y, ws, st);
    return dispatch_stma<BITS, GROUP, 2>(s, x, w, sc, bi, y, ws, st);
}

template <int BITS>
int dispatch_group(const Shape& s, const dflash_bf16* x, const uint32_t* w, const dflash_bf16* sc,
                   const dflash_bf16* bi, dflash_bf16* y, void* ws, cudaStream_t st) {
    switch (s.group) {
        case 32: return dispatch_nt<BITS, 32>(s, x, w, sc, bi, y, ws, st);
        case 64: return dispatch_nt<BITS, 64>(s, x, w, sc, bi, y, ws, st);
        case 128: return dispatch_nt<BITS, 128>(s, x, w, sc, bi, y, ws, st);
    }
    return fail(DFLASH_ERR_UNSUPPORTED, "group_size %d not in {32, 64, 128}", s.group);
}

int validate(const Shape& s) {
    if (s.bits != 4 && s.bits != 8) return fail(DFLASH_ERR_UNSUPPORTED, "bits %d not in {4, 8}", s.bits);
    if (s.group != 32 && s.group != 64 && s.group != 128)
        return fail(DFLASH_ERR_UNSUPPORTED, "group_size %d not in {32, 64, 128}", s.group);
    if (s.M < 1 || s.M > 16) return fail(DFLASH_ERR_UNSUPPORTED, "M=%d outside 1..16", s.M);
    if (s.N < 1 || s.K < 1) return fail(DFLASH_ERR_INVALID_ARGUMENT, "N=%d K=%d must be positive", s.N, s.K);
    if (s.N > kMaxTiles * kRows)
        return fail(DFLASH_ERR_UNSUPPORTED, "N=%d above the supported %d", s.N, kMaxTiles * kRows);
    if (s.K % s.group != 0)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "K=%d is not a multiple of group_size %d", s.K, s.group);
    return DFLASH_OK;
}

}  // namespace qmm
}  // namespace dflash

extern "C" size_t dflash_qmm_workspace_bytes(int M, int N, int K, int group_size, int bits) {
    (void)bits;
    if (N < 1 || K < 1 || M < 1 || M > 16 || (group_size != 32 && group_size != 64 && group_size != 128) ||
        K % group_size != 0)
        return 0;
    return dflash::qmm::workspace_size(M, K, group_size);
}

extern "C" int dflash_qmm_supported(int N, int K, int group_size, int bits) {
    if ((bits != 4 && bits != 8) || (group_size != 32 && group_size != 64 && group_size != 128)) return 0;
    if (N < 1 || K < 1 || K % group_size != 0 || N > dflash::qmm::kMaxTiles * dflash::qmm::kRows) return 0;
    return 1;
}

extern "C" int dflash_qmm(const dflash_bf16* x, const uint32_t* w, const dflash_bf16* scales,
                          const dflash_bf16* biases, dflash_bf16* y, int M, int N, int K, int group_size,
                          int bits, void* workspace, size_t workspace_bytes, dflash_stream_t stream) {
    using namespace dflash;
    qmm::Shape s{M, N, K, group_size, bits};
    if (int st = qmm::validate(s)) return st;
    if (!x || !w || !scales || !biases || !y)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_qmm: null tensor pointer");
    if (!aligned16(x) || !aligned16(w))
        return fail(DFLASH_ERR_MISALIGNED, "dflash_qmm: x and w must be 16-byte aligned");
    const size_t need = dflash_qmm_workspace_bytes(M, N, K, group_size, bits);
    if (!workspace || !aligned16(workspace) || workspace_bytes < need)
        return fail(DFLASH_ERR_WORKSPACE, "dflash_qmm: workspace of %zu bytes required (got %zu)", need,
                    workspace_bytes);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (bits == 4) return qmm::dispatch_group<4>(s, x, w, scales, biases, y, workspace, st);
    return qmm::dispatch_group<8>(s, x, w, scales, biases, y, workspace, st);
}

// ------------------------------------------------------------------ entry point without allocation
//
// For callers that cannot allocate device memory around a call: code running inside a
// CUDA-graph capture they do not own, plugin hosts whose allocator is off limits,
// real-time paths where a cudaMalloc could block or fail.  The scratch that
// dflash_qmm takes as `workspace` lives instead in this file-scope device array, which
// every GPU that loads the library holds until the process exits.
namespace dflash {
namespace qmm {

constexpr size_t kStaticScratchBytes = size_t(8) << 20;  // 8 MiB per device
static __device__ __align__(256) uint8_t g_static_scratch[kStaticScratchBytes];

// Device address of g_static_scratch on the current device, resolved once per device.
int static_scratch(void** out) {
    static std::mutex mu;
    static void* ptr[64] = {nullptr};
    int dev = 0;
    DFLASH_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(DFLASH_ERR_UNSUPPORTED, "device ordinal %d above 63", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess)
            return fail(DFLASH_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
        ptr[dev] = p;
    }
    *out = ptr[dev];
    return DFLASH_OK;
}

}  // namespace qmm
}  // namespace dflash

extern "C" int dflash_qmm_noalloc(const dflash_bf16* x, const uint32_t* w, const dflash_bf16* scales,
                                  const dflash_bf16* biases, dflash_bf16* y, int M, int N, int K, int group_size,
                                  int bits, dflash_stream_t stream) {
    using namespace dflash;
    qmm::Shape s{M, N, K, group_size, bits};
    if (int st = qmm::validate(s)) return st;
    if (!x || !w || !scales || !biases || !y)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_qmm_noalloc: null tensor pointer");
    if (!aligned16(x) || !aligned16(w))
        return fail(DFLASH_ERR_MISALIGNED, "dflash_qmm_noalloc: x and w must be 16-byte aligned");
    const size_t need = dflash_qmm_workspace_bytes(M, N, K, group_size, bits);
    if (need > qmm::kStaticScratchBytes)
        return fail(DFLASH_ERR_UNSUPPORTED,
                    "dflash_qmm_noalloc: M=%d K=%d group %d needs %zu bytes of scratch, above the %zu-byte static "
                    "maximum; use dflash_qmm with a caller-owned workspace",
                    M, K, group_size, need, qmm::kStaticScratchBytes);
    void* scratch = nullptr;
    if (int st = qmm::static_scratch(&scratch)) return st;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (bits == 4) return qmm::dispatch_group<4>(s, x, w, scales, biases, y, scratch, st);
    return qmm::dispatch_group<8>(s, x, w, scales, biases, y, scratch, st);
}
