// Small-M affine-quantized matmul for sm_100a:  y[M,N] = x[M,K] . deq(W)[N,K]^T.
//
// Replaces SmallMQuantizedMatmul.apply (Sources/DFlashKit/SmallMQuantizedMatmul.swift:
// 210-224) and the stock quantizedMatmul it stands in for.  The work is bound by the
// packed weight stream (M <= 16 rows against N*K quantized weights), so everything is
// arranged to move those bytes from HBM once, at full bandwidth, with one weight-stream
// kernel per call:
//
//  * Two kernels per call, chained with programmatic dependent launch (PDL).  A small
//    prep kernel turns x into per-stage "packets": x in fp16, permuted into MMA fragment
//    order, plus per segment of k the sums the epilogue needs.  The main kernel starts
//    streaming weights, scales and biases before its grid dependency resolves (they are
//    not written by the preceding kernels), so back-to-back calls keep HBM busy across
//    kernel boundaries.
//  * The main grid is a set of 2-CTA thread-block clusters, one CTA per SM.  Output
//    features are cut into row tiles of up to 256 rows, one TMA box high; each cluster
//    takes whole tiles, and its two CTAs take the two halves of K.  Inside a CTA, the
//    four k-lanes of consumer warps hold partial sums that are added in a fixed order
//    through shared memory; the two CTAs then push each other the rows the other one
//    writes, with distributed-shared-memory stores.  No CTA waits on a CTA outside its
//    cluster, and results are deterministic.
//  * One producer thread issues, per stage, one TMA box of [tile rows x 128 B] of packed
//    weights (128-byte swizzle, no multicast) and one bulk copy of the x packet into a
//    ring of up to 8 stages; scale and bias boxes of 8 groups go to a second ring.  The
//    ring depth is chosen per launch to fill shared memory.
//  * 16 consumer warps: k-lane (warp & 3) takes one 32-byte column slice of every
//    stage, row quarter (warp >> 2) takes every fourth 16-row block.  The warps of one
//    SM sub-partition share a k-lane, so the four sub-partitions get equal work for any
//    tile height.  A warp first copies everything it needs from a stage into registers
//    and releases the slot, then dequantises and contracts on mma.sync m16n8k16 with the
//    weights as the 16-row A operand and x (<= 8 rows per n-tile) as the n=8 B operand,
//    interleaving its blocks so that the MMA chains overlap.  A weight is read and
//    dequantised once for all M rows.
//
// Dequantisation uses the factored form  sum_k x (q s + b) = s (sum_k x q) + b (sum_k x)
// per group, on fp16 MMA operands.  A code becomes an exact fp16 value by OR-ing its
// nibble into the mantissa of a power of two, one LOP3 per two weights: a nibble in
// bits 0-3 of a 16-bit lane over 1024.0 (0x6400) reads 1024 + q; a nibble in bits 4-7
// over 64.0 (0x5400) reads 64 + q (the mantissa step there is 1/16), so both nibbles of
// a byte unpack without a shift and a packed word costs 4 LOP3 and one shift for 8
// weights.  The MMA accumulator starts at -z, where z = sum_k offset_k x' comes with
// the packet, so the MMA leaves exactly sum_k q x' and the combine is two FMAs per
// output: acc += s tmp + b xs.  For 8-bit codes the high nibble over 1024.0 reads
// 1024 + 16 q_hi, so both MMAs use the same x and z = 2048 sum x'.  x enters fp16 as
// x' = x / f with f a power of two per segment.  f is 1 for a segment whose largest |x|
// lies in [2^-6, 2^15), and only otherwise does the combine multiply by f: larger
// segments are scaled down below fp16's overflow, smaller ones up so that their largest
// value lands in [2^14, 2^15).  bf16's 8-bit significand fits fp16's 11 bits, so a value
// converts exactly when it lies within fp16's normal range (2^-14 upward) after the
// scaling, i.e. within 14 + 6 = 20 binades of its segment's largest value in the worst
// case; values further below become fp16 subnormals and lose low bits (below 2^-24 they
// become zero), which moves the output by far less than its bf16 rounding.  Within a
// lane's words the k order is permuted identically
// for weights and x (a sum does not depend on k order), so weights are consumed exactly
// as MLX packs them.
#include "common.cuh"
#include "dflash_stack.h"
#include "tp_layout.cuh"

#include <cstdlib>

namespace dflash {
namespace qmm {

constexpr int kConsumerWarps = 16;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 128;  // + the producer warpgroup (one thread issues)
constexpr int kLaunchRegs = 96;                   // per thread at launch: 640 x 96 fits one SM
constexpr int kConsumerRegs = 112;                // after setmaxnreg: 512 x 112 + 128 x 32 = 640 x 96
constexpr int kProducerRegs = 32;
static_assert(kConsumerThreads * kConsumerRegs + 128 * kProducerRegs <= kThreads * kLaunchRegs,
              "setmaxnreg split exceeds the registers the block is launched with");
constexpr int kKLanes = 4;                       // consumer warps per row quarter
constexpr int kMaxTileBlocks = 16;               // 16-row blocks per row tile (TMA box <= 256 rows)
constexpr int kRowBytes = 128;                   // packed weight bytes per row per stage
constexpr int kMaxStages = 8;
constexpr int kMaxSbStages = 8;
constexpr int kMaxCluster = 8;  // CTAs of a cluster, each taking a contiguous 1/cs of K
// Shared memory a weight-stream CTA plans for: the 227 KB opt-in maximum less 16 KB, so
// that the small kernels chained around a call — the next call's prep blocks, the verify
// stack's norms and glue — can be resident beside a running CTA instead of waiting for it
// to exit (measured: config 2 17.4 -> 16.5 us per back-to-back call, the TP = 1 verify
// forward 6.96 -> 6.69 ms; 8 KB of headroom gives the former, 16 KB both).
constexpr int kSmemLimit = 232448 - 16384;
constexpr int kBarConsumers = 1;                 // named barrier: all consumer warps
constexpr int kPrepThreads = 32;                 // one warp per prep block: fits beside a running main CTA
constexpr int kMaxN = 1 << 24;
constexpr uint32_t kMag1024 = 0x64006400u;       // fp16x2 (1024, 1024): + nibble in bits 0-3 (4-7: +16q)
constexpr uint32_t kMag64 = 0x54005400u;         // fp16x2 (64, 64): + nibble in bits 4-7
constexpr uint32_t kLoNib = 0x000F000Fu;
constexpr uint32_t kHiNib = 0x00F000F0u;

template <int BITS_, int GROUP_, int NT_, bool STMA_>
struct Cfg {
    static constexpr int BITS = BITS_, GROUP = GROUP_, NT = NT_;
    static constexpr bool STMA = STMA_;                   // scales/biases by TMA (else read from global)
    static constexpr int MR = 8 * NT;                     // x rows in a packet (zero padded past M)
    static constexpr int STAGE_K = kRowBytes * 8 / BITS;  // 256 (4-bit) or 128 (8-bit) k per stage
    static constexpr int UNIT_K = STAGE_K / kKLanes;      // k per k-lane per stage: 64 or 32
    static constexpr int UNIT_B = UNIT_K * 2;             // fp16 bytes of one x row of a unit
    static constexpr int SEG_K = UNIT_K < GROUP ? UNIT_K : GROUP;  // k per combine segment
    static constexpr int SEGS = UNIT_K / SEG_K;           // segments per unit: 2 for 4-bit g32, else 1
    static constexpr int GPS = STAGE_K / GROUP;           // groups per stage
    static constexpr int SBP = 8 / GPS;                   // stages per scale/bias box of 8 groups
    static constexpr int X_BYTES = kKLanes * MR * UNIT_B;
    static constexpr int T_BYTES = kKLanes * SEGS * MR * 16;
    static constexpr int PKT = X_BYTES + T_BYTES;         // packet bytes per stage
    static constexpr int XREGS = UNIT_B / 4 / 4;          // 32-bit B registers per lane per unit: 8 or 4
    // 16-row blocks per consumer warp and tile: 4 (tiles up to 256 rows), 2 with two
    // n-tiles (M > 8), whose doubled x fragments and accumulators would not fit 4
    static constexpr int MAXB = NT == 2 ? 2 : 4;
    static_assert(PKT % 16 == 0, "bulk copies move multiples of 16 bytes");
    static_assert(GPS >= 1 && 8 % GPS == 0, "scale boxes hold 8 groups");
};

// Packet layout (one per stage of STAGE_K columns of x; offsets in bytes):
//   x region  [unit u][row m][UNIT_B]: the fp16 x' of k in [u UNIT_K, (u+1) UNIT_K) of the
//             stage, in 16-byte chunks of 8 k.  Chunk c is stored at c ^ x_swizzle(m) and
//             holds its 8 values in fragment order (4-bit: 0,4,1,5,2,6,3,7; 8-bit:
//             0,2,1,3,4,6,5,7), so a lane's B fragments are two (4-bit) or one (8-bit)
//             conflict-free 16-byte loads.
//   table     [unit u][segment][row m] float4 (-z', xs, f, 0)
template <class C>
__host__ __device__ __forceinline__ constexpr int x_swizzle(int m) {
    return C::BITS == 8 ? 0 : (C::SEGS == 2 ? ((m & 1) << 2) : (m & 1));
}

// ------------------------------------------------------------------ small device helpers

// (v & mask) | mag as one LOP3: the mask is an immediate, the magic a register (left
// to itself the compiler splits this into an AND and an OR with two immediates, which
// doubles the load on the ALU pipe).
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

// Per-warpgroup register budget changes (all 128 threads of a warpgroup execute them).
template <uint32_t N>
__device__ __forceinline__ void regs_raise() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_lower() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// D += A * B, m16n8k16, fp16 operands, fp32 accumulate.
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void tma_load_2d_u32(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

__device__ __forceinline__ void bulk_copy_g2s(uint32_t dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ uint32_t cluster_id() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t nclusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}
// Store into another CTA's shared memory; the bytes complete on that CTA's mbarrier.
__device__ __forceinline__ void st_async_f32x2(uint32_t addr, float a, float b, uint32_t remote_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(addr),
                 "f"(a), "f"(b), "r"(remote_bar)
                 : "memory");
}
// Arrive (release, cluster scope) on an mbarrier of another CTA of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "n"(kSuspendHintNs)
        : "memory");
    return ok != 0;
}
// Bounded wait with cluster-scope acquire, for hand-offs between the CTAs of a cluster.
// Runs to its limit even after an abort elsewhere, so that both CTAs keep taking the
// same steps; a timeout records `errbit` and the abort flag.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t* bar, uint32_t parity, volatile int* abort,
                                                          unsigned errbit) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_cluster(bar, parity)) return true;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(&g_device_error, errbit);
            *abort = 1;
            return false;
        }
    }
}
// Bounded wait that ignores the abort flag: lets copies already in flight land before
// the CTA leaves.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try_wait_sleep(bar, parity)) {
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            atomicOr(&g_device_error, DFLASH_DEVERR_QMM_PIPELINE);
            return;
        }
    }
}
// Split cluster barrier: a relaxed arrive (orders nothing by itself; preceded by
// fence.mbarrier_init it publishes barrier initialisation) and the matching wait.
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory"); }
__device__ __forceinline__ void cluster_sync_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// ------------------------------------------------------------------ prep kernel
//
// One thread per (x row m < MR, run of 8 k): reads 8 bf16 of x (zeros past M or K),
// picks the segment's power-of-two scale, writes the fp16 run in fragment order and,
// from the segment's first lane, the table entry.  Lanes of a segment are adjacent, so
// the segment reductions are xor-shuffles (the same fixed-order sum on every lane).
// Padding (rows past M, k past K) gets x' = 0 and a zero table entry, so the main
// kernel needs no masks along k or m: those columns contribute exactly 0.
// SWIGLU: x is [M, 2K] = [gate | up] and the matmul input is bf16(silu(gate) * up), the
// activation between an MLP's gate/up and down projections, formed here instead of by a
// separate kernel (the same arithmetic, so the result is the same bits).
__device__ __forceinline__ float swiglu_bf16(float g, float u) {
    const float a = g / (1.f + __expf(-g)) * u;
    return bf16_bits_to_float(__bfloat16_as_ushort(__float2bfloat16_rn(a)));
}

template <class C, bool SWIGLU>
__global__ void __launch_bounds__(kPrepThreads) qmm_prep_kernel(const uint16_t* __restrict__ x,
                                                                uint8_t* __restrict__ packets, int M, int K,
                                                                int S, unsigned long long* argmax_keys) {
    pdl_launch_dependents();
    pdl_wait();  // x may be written by the preceding kernel
    if (argmax_keys && blockIdx.x == 0 && threadIdx.x < M) argmax_keys[threadIdx.x] = 0ull;
    constexpr int CPR = C::STAGE_K / 8;  // runs of 8 per stage row
    constexpr int SL = C::SEG_K / 8;     // lanes per segment: 4 or 8
    const long long runs = (long long)S * CPR;
    const long long idx = (long long)blockIdx.x * kPrepThreads + threadIdx.x;
    if (idx >= runs * C::MR) return;  // whole warps only: runs * MR is a multiple of 32
    const int m = (int)(idx / runs);
    const int k0 = (int)(idx % runs) * 8;

    float v[8];
    if (m < M && k0 < K) {
        const uint4 r = __ldg(reinterpret_cast<const uint4*>(x + (size_t)m * (SWIGLU ? 2 * K : K) + k0));
        v[0] = bf16_lo(r.x);
        v[1] = bf16_hi(r.x);
        v[2] = bf16_lo(r.y);
        v[3] = bf16_hi(r.y);
        v[4] = bf16_lo(r.z);
        v[5] = bf16_hi(r.z);
        v[6] = bf16_lo(r.w);
        v[7] = bf16_hi(r.w);
        if constexpr (SWIGLU) {
            const uint4 q = __ldg(reinterpret_cast<const uint4*>(x + (size_t)m * 2 * K + K + k0));
            v[0] = swiglu_bf16(v[0], bf16_lo(q.x));
            v[1] = swiglu_bf16(v[1], bf16_hi(q.x));
            v[2] = swiglu_bf16(v[2], bf16_lo(q.y));
            v[3] = swiglu_bf16(v[3], bf16_hi(q.y));
            v[4] = swiglu_bf16(v[4], bf16_lo(q.z));
            v[5] = swiglu_bf16(v[5], bf16_hi(q.z));
            v[6] = swiglu_bf16(v[6], bf16_lo(q.w));
            v[7] = swiglu_bf16(v[7], bf16_hi(q.w));
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
#pragma unroll
    for (int o = 1; o < SL; o <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    float f = 1.f, inv = 1.f;
    // false for NaN (NaN inputs propagate unscaled), and for segments whose largest value is
    // below 2^-100 (zero, or too small to register in any output: left to flush)
    if (amax >= 32768.f || (amax < 0x1p-6f && amax >= 0x1p-100f)) {
        const int e = ((__float_as_int(amax) >> 23) & 0xff) - 127;  // floor(log2 amax) in [-100, 128]
        const int sh = e - 14;                                      // amax / 2^sh in [2^14, 2^15)
        f = __int_as_float((127 + sh) << 23);
        inv = __int_as_float((127 - sh) << 23);
    }
    // fragment order of the run: 4-bit (0,4)(1,5)(2,6)(3,7); 8-bit (0,2)(1,3)(4,6)(5,7)
    float r[8];
    uint32_t h[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int a = C::BITS == 4 ? i : ((i >> 1) << 2) + (i & 1);
        const int b = C::BITS == 4 ? i + 4 : a + 2;
        h[i] = pack_half2(v[a] * inv, v[b] * inv);
        const __half2 hh = *reinterpret_cast<const __half2*>(&h[i]);
        r[a] = __low2float(hh);
        r[b] = __high2float(hh);
    }
    float z, xs = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    if constexpr (C::BITS == 4) {
        // nibbles 0, 2, 4, 6 of a word read 1024 + q, nibbles 1, 3, 5, 7 read 64 + q
        const float ev = (r[0] + r[2]) + (r[4] + r[6]);
        const float od = (r[1] + r[3]) + (r[5] + r[7]);
        z = fmaf(1024.f, ev, 64.f * od);
    } else {
        z = 2048.f * (((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7])));
    }
#pragma unroll
    for (int o = 1; o < SL; o <<= 1) {
        z += __shfl_xor_sync(0xffffffffu, z, o);
        xs += __shfl_xor_sync(0xffffffffu, xs, o);
    }
    const int s = k0 / C::STAGE_K, kin = k0 % C::STAGE_K;
    const int u = kin / C::UNIT_K, c = (kin % C::UNIT_K) / 8;
    uint8_t* pkt = packets + (size_t)s * C::PKT;
    *reinterpret_cast<uint4*>(pkt + (u * C::MR + m) * C::UNIT_B + ((c ^ x_swizzle<C>(m)) << 4)) =
        make_uint4(h[0], h[1], h[2], h[3]);
    if (kin % C::SEG_K == 0) {
        const int seg = (kin % C::UNIT_K) / C::SEG_K;
        *reinterpret_cast<float4*>(pkt + C::X_BYTES + ((u * C::SEGS + seg) * C::MR + m) * 16) =
            make_float4(-z, xs, f, 0.f);
    }
}

// ------------------------------------------------------------------ main kernel

struct Params {
    const uint8_t* packets;
    const uint16_t* scales;  // read directly only without scale TMA
    const uint16_t* biases;
    uint16_t* y;
    int M, N, K, GT;
    int R, nb;    // tile rows = 16 nb
    int nb0;         // clusters of 2: blocks of a tile written by rank 0 (rank 1 writes the rest)
    int own_stride;  // clusters of 4 or 8: rows of one sender's slot in the receive buffer
    int ntiles;   // ceil(N / R)
    int S;        // stages along K
    int NS, NSB;  // ring depths
    int y_vec;    // y rows 16-byte aligned with N % 8 == 0: write y in 16-byte chunks
    // push: instead of y, write the output into slot `rank` of exchange set `set` of every
    // rank's exchange buffer (tp_layout.cuh) as epoch-tagged words (N % 8 == 0)
    int push, rank, world, set;
    tp::Bases xb;
    // argmax: instead of y, fold each row's (largest bf16 output, lowest index) into
    // argmax_keys[m] with a 64-bit atomic max (zeroed by the prep kernel)
    unsigned long long* argmax_keys;
    int argmax_base;  // added to the output index in the keys (a vocabulary shard's first row)
    uint32_t stage_bytes, sb_bytes, red_off, red_bytes, recv_off, bar_off;
};

// Shared-memory barrier block (at bar_off).
struct Bars {
    uint64_t full[kMaxStages], empty[kMaxStages];
    uint64_t sbfull[kMaxSbStages], sbempty[kMaxSbStages];
    uint64_t xfull, xdone;  // cluster exchange: the other CTAs' rows for us have landed / they have read ours
    int abort;
};

// MMA fragment row g (0..7) of a 16-row block maps to block row phys(g) (+8 for the
// second half): even rows for g < 4, odd rows for g >= 4, so that each half-warp's
// 64-bit weight loads hit 8 different 16-byte chunks of the 128-byte swizzle.
__device__ __forceinline__ int phys_row(int g) { return ((g & 3) << 1) | (g >> 2); }

struct StageCtx {
    uint32_t wb;    // weight box of this stage
    uint32_t pkt;   // packet of this stage
    uint32_t sb;    // scale/bias slot (scale TMA only)
    int sbcol0;     // group index of the slot's first column
    int s;          // stage index along K
    int tile_row0;  // first output row of the tile
};

// Shared-memory offsets of one consumer lane that do not change from stage to stage:
// a warp always handles the same unit (k-lane) and the same blocks of every stage.
// Block i of the warp sits 4 i blocks below block 0, so its offsets are immediates.
struct LaneOfs {
    uint32_t x0, x1;  // packet: this lane's two 16-byte B chunks (n-tile 0)
    uint32_t tab;     // packet: table entry of column 2 tq (segment 0, n-tile 0)
    uint32_t w0, w1;  // weight box: this lane's words of row 16 qd + pr (second word for 4-bit g32)
    uint32_t sb;      // scale slot: row 16 qd + pr
};

template <class C>
__device__ __forceinline__ LaneOfs lane_offsets(int kl, int qd, int g, int tq) {
    LaneOfs o;
    const int pr = phys_row(g);
    const uint32_t xrow = (kl * C::MR + g) * C::UNIT_B;
    if constexpr (C::BITS == 4) {
        // SEGS 1: chunks 2tq, 2tq+1 (the lane's words 2tq, 2tq+1); SEGS 2: chunks tq, tq+4
        const int c0 = C::SEGS == 2 ? tq : 2 * tq;
        const int c1 = C::SEGS == 2 ? tq + 4 : 2 * tq + 1;
        o.x0 = xrow + ((c0 ^ x_swizzle<C>(g)) << 4);
        o.x1 = xrow + ((c1 ^ x_swizzle<C>(g)) << 4);
    } else {
        o.x0 = xrow + (tq << 4);
        o.x1 = o.x0;
    }
    o.tab = C::X_BYTES + (kl * C::SEGS * C::MR + 2 * tq) * 16;
    // the lane's words in a 128-byte row: unit kl is bytes [32 kl, 32 kl + 32);
    // rows 16 b + pr and 16 b + pr + 8 both have (row & 7) == pr
    const uint32_t rowb = (16 * qd + pr) * kRowBytes;
    if constexpr (C::SEGS == 2) {
        o.w0 = rowb + (((2 * kl) ^ pr) << 4) + tq * 4;
        o.w1 = rowb + (((2 * kl + 1) ^ pr) << 4) + tq * 4;
    } else {
        o.w0 = rowb + (((2 * kl + (tq >> 1)) ^ pr) << 4) + (tq & 1) * 8;
        o.w1 = o.w0 + 4;
    }
    o.sb = (16 * qd + pr) * 16;
    return o;
}

// Everything one consumer warp takes from a stage: its x fragments and table entries
// for unit kl, and the weight words of its NB blocks.
template <class C, int NB>
struct StageRegs {
    uint32_t xb[C::NT][C::XREGS];
    float tz[C::SEGS][C::NT][2], txs[C::SEGS][C::NT][2], tf[C::SEGS][C::NT][2];
    bool slow[C::SEGS];
    uint32_t w[NB][2][2];  // block, row half (r0 / r0 + 8), word
};

template <class C, int NB>
__device__ __forceinline__ void load_stage(StageRegs<C, NB>& R, uint32_t wb, uint32_t pkt, const LaneOfs& o) {
#pragma unroll
    for (int nt = 0; nt < C::NT; ++nt) {
        const uint4 v0 = lds128(pkt + o.x0 + nt * 8 * C::UNIT_B);
        R.xb[nt][0] = v0.x;
        R.xb[nt][1] = v0.y;
        R.xb[nt][2] = v0.z;
        R.xb[nt][3] = v0.w;
        if constexpr (C::BITS == 4) {
            const uint4 v1 = lds128(pkt + o.x1 + nt * 8 * C::UNIT_B);
            R.xb[nt][4] = v1.x;
            R.xb[nt][5] = v1.y;
            R.xb[nt][6] = v1.z;
            R.xb[nt][7] = v1.w;
        }
    }
#pragma unroll
    for (int sg = 0; sg < C::SEGS; ++sg) {
        bool any = false;
#pragma unroll
        for (int nt = 0; nt < C::NT; ++nt) {
            const uint32_t a = pkt + o.tab + (sg * C::MR + 8 * nt) * 16;
            const uint4 v0 = lds128(a), v1 = lds128(a + 16);
            R.tz[sg][nt][0] = __uint_as_float(v0.x);
            R.txs[sg][nt][0] = __uint_as_float(v0.y);
            R.tf[sg][nt][0] = __uint_as_float(v0.z);
            R.tz[sg][nt][1] = __uint_as_float(v1.x);
            R.txs[sg][nt][1] = __uint_as_float(v1.y);
            R.tf[sg][nt][1] = __uint_as_float(v1.z);
            any |= (v0.z != 0x3f800000u) | (v1.z != 0x3f800000u);
        }
        R.slow[sg] = __any_sync(0xffffffffu, any);
    }
#pragma unroll
    for (int i = 0; i < NB; ++i) {
        const uint32_t a = wb + 4 * 16 * kRowBytes * i;
        if constexpr (C::SEGS == 2) {
            R.w[i][0][0] = lds32(a + o.w0);
            R.w[i][0][1] = lds32(a + o.w1);
            R.w[i][1][0] = lds32(a + o.w0 + 8 * kRowBytes);
            R.w[i][1][1] = lds32(a + o.w1 + 8 * kRowBytes);
        } else {
            const uint2 u0 = lds64(a + o.w0), u1 = lds64(a + o.w0 + 8 * kRowBytes);
            R.w[i][0][0] = u0.x;
            R.w[i][0][1] = u0.y;
            R.w[i][1][0] = u1.x;
            R.w[i][1][1] = u1.y;
        }
    }
}

// bf16 bits -> fp32 as an integer multiply (FMA pipe) by a register holding 65536,
// which keeps the conversion off the ALU pipe that the unpack loads.
__device__ __forceinline__ float bf16_to_f32_fma(uint32_t b, uint32_t k65536) {
    uint32_t d;
    asm("mul.lo.u32 %0, %1, %2;" : "=r"(d) : "r"(b), "r"(k65536));
    return __uint_as_float(d);
}

// D = A * B + C, m16n8k16, fp16 operands, fp32 accumulate, C from separate registers.
__device__ __forceinline__ void mma_f16_c(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1, float c0, float c1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%10, %11, %10, %11};"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1));
}

// Dequantise and contract one stage from registers.  The blocks' MMA chains are issued
// round-robin so that the latency of one chain hides behind the others; each chain
// starts from the segment's -z.  `release` is the stage's empty barrier: the warp
// arrives on it once its last MMAs have consumed every register loaded from the slot
// (an arrive releases the warp's earlier shared-memory reads, complete by then, so it
// does not stall).  Scales and biases come from the scale/bias ring (released later)
// or, without scale TMA, from global memory.
template <class C, int NB>
__device__ __forceinline__ void compute_stage(const StageRegs<C, NB>& R, const StageCtx& x, const Params& p,
                                              const LaneOfs& o, int kl, int qd, int pr, uint32_t mag1024,
                                              uint32_t mag64, uint32_t k65536, int lane, uint64_t* release,
                                              float (&acc)[C::MAXB][C::NT][4]) {
#pragma unroll
    for (int nt = 0; nt < C::NT; ++nt) {
#pragma unroll
        for (int sg = 0; sg < C::SEGS; ++sg) {
            float d[NB][4];
            const float c0 = R.tz[sg][nt][0], c1 = R.tz[sg][nt][1];
#pragma unroll
            for (int wi = 0; wi < 2; ++wi) {
                if (C::SEGS == 2 && wi != sg) continue;  // 4-bit g32: segment sg is word sg
                const bool first = (C::SEGS == 2) || wi == 0;
                if constexpr (C::BITS == 4) {
                    const uint32_t b0 = R.xb[nt][4 * wi + 0], b1 = R.xb[nt][4 * wi + 1];
                    const uint32_t b2 = R.xb[nt][4 * wi + 2], b3 = R.xb[nt][4 * wi + 3];
#pragma unroll
                    for (int i = 0; i < NB; ++i) {
                        const uint32_t v0 = R.w[i][0][wi], v1 = R.w[i][1][wi];
                        const uint32_t a0 = unpack<kLoNib>(v0, mag1024), a1 = unpack<kLoNib>(v1, mag1024);
                        const uint32_t a2 = unpack<kHiNib>(v0, mag64), a3 = unpack<kHiNib>(v1, mag64);
                        if (first) mma_f16_c(d[i], a0, a1, a2, a3, b0, b1, c0, c1);
                        else mma_f16(d[i], a0, a1, a2, a3, b0, b1);
                    }
#pragma unroll
                    for (int i = 0; i < NB; ++i) {
                        const uint32_t t0 = R.w[i][0][wi] >> 8, t1 = R.w[i][1][wi] >> 8;
                        mma_f16(d[i], unpack<kLoNib>(t0, mag1024), unpack<kLoNib>(t1, mag1024),
                                unpack<kHiNib>(t0, mag64), unpack<kHiNib>(t1, mag64), b2, b3);
                    }
                } else {
                    // bytes (0, 2) in place and (1, 3) shifted: low nibbles 1024 + q_lo,
                    // high nibbles 1024 + 16 q_hi, against the same x
                    const uint32_t b0 = R.xb[nt][2 * wi], b1 = R.xb[nt][2 * wi + 1];
#pragma unroll
                    for (int i = 0; i < NB; ++i) {
                        const uint32_t v0 = R.w[i][0][wi], v1 = R.w[i][1][wi];
                        const uint32_t t0 = v0 >> 8, t1 = v1 >> 8;
                        const uint32_t a0 = unpack<kLoNib>(v0, mag1024), a1 = unpack<kLoNib>(v1, mag1024);
                        const uint32_t a2 = unpack<kLoNib>(t0, mag1024), a3 = unpack<kLoNib>(t1, mag1024);
                        if (first) mma_f16_c(d[i], a0, a1, a2, a3, b0, b1, c0, c1);
                        else mma_f16(d[i], a0, a1, a2, a3, b0, b1);
                    }
#pragma unroll
                    for (int i = 0; i < NB; ++i) {
                        const uint32_t v0 = R.w[i][0][wi], v1 = R.w[i][1][wi];
                        const uint32_t t0 = v0 >> 8, t1 = v1 >> 8;
                        mma_f16(d[i], unpack<kHiNib>(v0, mag1024), unpack<kHiNib>(v1, mag1024),
                                unpack<kHiNib>(t0, mag1024), unpack<kHiNib>(t1, mag1024), b0, b1);
                    }
                }
            }
            if (nt == C::NT - 1 && sg == C::SEGS - 1) {
                __syncwarp();
                if (lane == 0) mbar_arrive(release);
            }
            const int col = (x.s * C::STAGE_K + kl * C::UNIT_K + sg * C::SEG_K) / C::GROUP;
            const uint32_t sa = x.sb + o.sb + 2 * (col - x.sbcol0);
            const uint32_t ba = sa + p.R * 16;
#pragma unroll
            for (int i = 0; i < NB; ++i) {
                float e0 = d[i][0], e1 = d[i][1], e2 = d[i][2], e3 = d[i][3];
                if (R.slow[sg]) {
                    e0 *= R.tf[sg][nt][0];
                    e1 *= R.tf[sg][nt][1];
                    e2 *= R.tf[sg][nt][0];
                    e3 *= R.tf[sg][nt][1];
                }
                float s0, s1, b0, b1;
                if constexpr (C::STMA) {
                    const uint32_t bo = 4 * 16 * 16 * i;  // block i: 64 rows down
                    s0 = bf16_to_f32_fma(lds16(sa + bo), k65536);
                    s1 = bf16_to_f32_fma(lds16(sa + bo + 8 * 16), k65536);
                    b0 = bf16_to_f32_fma(lds16(ba + bo), k65536);
                    b1 = bf16_to_f32_fma(lds16(ba + bo + 8 * 16), k65536);
                } else {
                    const int n0 = x.tile_row0 + 16 * (qd + 4 * i) + pr, n1 = n0 + 8;
                    const bool in_k = col < p.GT;
                    const bool ok0 = n0 < p.N && in_k, ok1 = n1 < p.N && in_k;
                    const size_t i0 = (size_t)n0 * p.GT + col, i1 = (size_t)n1 * p.GT + col;
                    s0 = ok0 ? bf16_bits_to_float(__ldg(p.scales + i0)) : 0.f;
                    b0 = ok0 ? bf16_bits_to_float(__ldg(p.biases + i0)) : 0.f;
                    s1 = ok1 ? bf16_bits_to_float(__ldg(p.scales + i1)) : 0.f;
                    b1 = ok1 ? bf16_bits_to_float(__ldg(p.biases + i1)) : 0.f;
                }
                float* a = acc[i][nt];
                a[0] = fmaf(s0, e0, fmaf(b0, R.txs[sg][nt][0], a[0]));
                a[1] = fmaf(s0, e1, fmaf(b0, R.txs[sg][nt][1], a[1]));
                a[2] = fmaf(s1, e2, fmaf(b1, R.txs[sg][nt][0], a[2]));
                a[3] = fmaf(s1, e3, fmaf(b1, R.txs[sg][nt][1], a[3]));
            }
        }
    }
}

// The stages of one tile for one consumer warp with NB blocks.
template <class C, int NB>
__device__ __forceinline__ void run_tile(const Params& p, Bars* bars, volatile int* abort, uint32_t ring,
                                         uint32_t sbring, const LaneOfs& o, int kl, int qd, int pr, int lane,
                                         int s_beg, int s_end, int tile_row0, uint32_t mag1024, uint32_t mag64,
                                         uint32_t k65536, int& slot, int& ph, int& qslot, int& qph,
                                         float (&acc)[C::MAXB][C::NT][4]) {
    const uint32_t wbytes = (uint32_t)p.R * kRowBytes;
    StageCtx cx;
    cx.tile_row0 = tile_row0;
    cx.sb = sbring;
    cx.sbcol0 = 0;
    for (int s = s_beg; s < s_end; ++s) {
        if (C::STMA && (s == s_beg || s % C::SBP == 0)) {
            mbar_wait_bounded(&bars->sbfull[qslot], qph, abort, DFLASH_DEVERR_QMM_PIPELINE);
            cx.sb = sbring + qslot * p.sb_bytes;
            cx.sbcol0 = (s / C::SBP) * 8;
        }
        const bool ready = mbar_wait_bounded(&bars->full[slot], ph, abort, DFLASH_DEVERR_QMM_PIPELINE);
        if constexpr (NB > 0) {
            if (ready) {
                cx.wb = ring + slot * p.stage_bytes;
                cx.pkt = cx.wb + wbytes;
                cx.s = s;
                StageRegs<C, NB> R;
                load_stage<C, NB>(R, cx.wb, cx.pkt, o);
                compute_stage<C, NB>(R, cx, p, o, kl, qd, pr, mag1024, mag64, k65536, lane, &bars->empty[slot], acc);
            }
        }
        if (NB == 0 || !ready) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->empty[slot]);
        }
        if (++slot == p.NS) {
            slot = 0;
            ph ^= 1;
        }
        if (C::STMA && (s == s_end - 1 || (s + 1) % C::SBP == 0)) {
            __syncwarp();
            if (lane == 0) mbar_arrive(&bars->sbempty[qslot]);
            if (++qslot == p.NSB) {
                qslot = 0;
                qph ^= 1;
            }
        }
    }
}

// Producers.  The j-th stage of a CTA is stage s_beg + j % nstages of tile
// cid + (j / nstages) ncl.  Two threads in different warps (so on different SM
// sub-partitions) share the work, because each TMA issue holds its thread for a while:
// one issues the weight boxes, the other the x packets and the scale/bias boxes.  A
// stage's full barrier takes one arrival from each.  Scale/bias slots open at the CTA's
// first stage of a tile and at every multiple of SBP.  Both return false when a bounded
// wait gave up.
template <class C>
__device__ __forceinline__ bool issue_weights(int j, Bars* bars, volatile int* abort, const CUtensorMap& tm_w,
                                              const Params& p, uint32_t ring, int cid, int ncl, int s_beg, int nstages,
                                              uint32_t wbytes) {
    const int t = cid + (j / nstages) * ncl, s = s_beg + j % nstages;
    const int slot = j % p.NS;
    if (!mbar_wait_bounded(&bars->empty[slot], ((j / p.NS) & 1) ^ 1, abort, DFLASH_DEVERR_QMM_PIPELINE))
        return false;
    mbar_arrive_expect_tx(&bars->full[slot], wbytes);
    tma_load_2d_u32(ring + slot * p.stage_bytes, &tm_w, &bars->full[slot], s * (kRowBytes / 4), t * p.R);
    return true;
}

template <class C>
__device__ __forceinline__ bool issue_aux(int j, int& pq, Bars* bars, volatile int* abort, const CUtensorMap& tm_s,
                                          const CUtensorMap& tm_b, const Params& p, uint32_t ring, uint32_t sbring,
                                          int cid, int ncl, int s_beg, int nstages, uint32_t wbytes) {
    const int t = cid + (j / nstages) * ncl, s = s_beg + j % nstages;
    if (C::STMA && (s == s_beg || s % C::SBP == 0)) {
        const int q = pq % p.NSB;
        if (!mbar_wait_bounded(&bars->sbempty[q], ((pq / p.NSB) & 1) ^ 1, abort, DFLASH_DEVERR_QMM_PIPELINE))
            return false;
        mbar_arrive_expect_tx(&bars->sbfull[q], 2u * p.R * 16);
        const uint32_t dst = sbring + q * p.sb_bytes;
        tma_load_2d_u32(dst, &tm_s, &bars->sbfull[q], (s / C::SBP) * 8, t * p.R);
        tma_load_2d_u32(dst + p.R * 16, &tm_b, &bars->sbfull[q], (s / C::SBP) * 8, t * p.R);
        ++pq;
    }
    if (j == 0) pdl_wait();  // the packets come from the prep kernel
    const int slot = j % p.NS;
    if (!mbar_wait_bounded(&bars->empty[slot], ((j / p.NS) & 1) ^ 1, abort, DFLASH_DEVERR_QMM_PIPELINE))
        return false;
    mbar_arrive_expect_tx(&bars->full[slot], C::PKT);
    bulk_copy_g2s(ring + slot * p.stage_bytes + wbytes, p.packets + (size_t)s * C::PKT, C::PKT, &bars->full[slot]);
    return true;
}

// CS: CTAs per cluster (1, 2, 4 or 8), fixed at compile time so that the exchange of
// partials between them compiles to straight-line code.
template <class C, int CS>
__global__ void __launch_bounds__(kThreads, 1)
    qmm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_s,
               const __grid_constant__ CUtensorMap tm_b, const Params p) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Bars* bars = reinterpret_cast<Bars*>(smem + p.bar_off);
    volatile int* abort = &bars->abort;
    const uint32_t ring = smem_u32(smem);
    const uint32_t sbring = ring + p.NS * p.stage_bytes;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr uint32_t cs = CS;
    const uint32_t rank = CS > 1 ? cluster_rank() : 0u;
    const int cid = (int)cluster_id(), ncl = (int)nclusters_x();
    const int s_beg = (int)((long long)p.S * rank / cs), s_end = (int)((long long)p.S * (rank + 1) / cs);
    const int nstages = s_end - s_beg;
    const int my_tiles = (nstages > 0 && cid < p.ntiles) ? (p.ntiles - 1 - cid) / ncl + 1 : 0;
    const int total = my_tiles * nstages;
    const int first_batch = total < p.NS ? total : p.NS;
    const uint32_t wbytes = (uint32_t)p.R * kRowBytes;

    pdl_launch_dependents();

    constexpr int kAuxThread = kConsumerThreads + 32;  // lane 0 of the second producer warp
    int issued = 0;  // weight boxes issued (first producer thread)
    if (tid == kConsumerThreads) {
        prefetch_tensormap(&tm_w);
        for (int i = 0; i < p.NS; ++i) {
            mbar_init(&bars->full[i], 2);  // weight thread + packet thread
            mbar_init(&bars->empty[i], kConsumerWarps);
        }
        for (int i = 0; i < p.NSB; ++i) {
            mbar_init(&bars->sbfull[i], 1);
            mbar_init(&bars->sbempty[i], kConsumerWarps);
        }
        mbar_init(&bars->xfull, 1);
        mbar_init(&bars->xdone, CS > 1 ? CS - 1 : 1);
        bars->abort = 0;
        fence_barrier_init();
    }
    // publishes the exchange barriers to the peer; its wait comes after the first loads
    __syncwarp();
    cluster_arrive_relaxed();
    if (tid == kConsumerThreads) {
        // The first ring's worth of weight boxes goes out before anything else: fresh
        // slots, so these never wait.
        for (; issued < first_batch; ++issued)
            issue_weights<C>(issued, bars, abort, tm_w, p, ring, cid, ncl, s_beg, nstages, wbytes);
    }
    __syncthreads();
    cluster_wait();

    if (warp >= kConsumerWarps) {
        // ---------------------------------------------------------------- producers
        regs_lower<kProducerRegs>();
        if (tid == kConsumerThreads && total > 0) {
            while (issued < total &&
                   issue_weights<C>(issued, bars, abort, tm_w, p, ring, cid, ncl, s_beg, nstages, wbytes))
                ++issued;
            if (*abort) {
                // let every copy already issued land before shared memory is released
                const int lo = issued > p.NS ? issued - p.NS : 0;
                for (int j = lo; j < issued; ++j) mbar_drain(&bars->full[j % p.NS], (j / p.NS) & 1);
            }
        } else if (tid == kAuxThread && total > 0) {
            if constexpr (C::STMA) {
                prefetch_tensormap(&tm_s);
                prefetch_tensormap(&tm_b);
            }
            int j = 0, pq = 0;
            while (j < total && issue_aux<C>(j, pq, bars, abort, tm_s, tm_b, p, ring, sbring, cid, ncl, s_beg, nstages,
                                             wbytes))
                ++j;
            if (*abort) {
                const int qlo = pq > p.NSB ? pq - p.NSB : 0;
                for (int q = qlo; q < pq; ++q) mbar_drain(&bars->sbfull[q % p.NSB], (q / p.NSB) & 1);
            }
        }
    } else {
        // ---------------------------------------------------------------- consumers
        regs_raise<kConsumerRegs>();
        if (total == 0) goto done;
        const int kl = warp & (kKLanes - 1), qd = warp / kKLanes;
        const int g = lane >> 2, tq = lane & 3;
        const int nblk = p.nb > qd ? (p.nb - qd + 3) / 4 : 0;  // blocks qd, qd + 4, ... below nb
        const int pr = phys_row(g);
        const uint32_t mag1024 = pinned<kMag1024>(), mag64 = pinned<kMag64>(), k65536 = pinned<65536u>();
        const LaneOfs lo = lane_offsets<C>(kl, qd, g, tq);
        float* bufa = reinterpret_cast<float*>(smem + p.red_off);
        float* bufb = reinterpret_cast<float*>(smem + p.red_off + p.red_bytes);
        float* recv = reinterpret_cast<float*>(smem + p.recv_off);
        constexpr int MR = C::MR;
        pdl_wait();  // y may still be read or written by the preceding kernel
        uint32_t push_epoch = 0;
        if (p.push) {  // this exchange's epoch; CTA 0 records it for this rank's consumer
            tp::Header* own = reinterpret_cast<tp::Header*>(p.xb.b[p.rank]);
            push_epoch = own->seq[p.set] + 1u;
            if (blockIdx.x == 0 && tid == 0) own->next[p.set] = push_epoch;
        }
        int slot = 0, ph = 0, qslot = 0, qph = 0, tt = 0;
        for (int t = cid; t < p.ntiles; t += ncl, ++tt) {
            float acc[C::MAXB][C::NT][4];
#pragma unroll
            for (int i = 0; i < C::MAXB; ++i)
#pragma unroll
                for (int nt = 0; nt < C::NT; ++nt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc[i][nt][e] = 0.f;
            switch (nblk) {
                case 4:
                    if constexpr (C::MAXB >= 4)
                        run_tile<C, 4>(p, bars, abort, ring, sbring, lo, kl, qd, pr, lane, s_beg, s_end, t * p.R,
                                       mag1024, mag64, k65536, slot, ph, qslot, qph, acc);
                    break;
                case 3:
                    if constexpr (C::MAXB >= 3)
                        run_tile<C, 3>(p, bars, abort, ring, sbring, lo, kl, qd, pr, lane, s_beg, s_end, t * p.R,
                                       mag1024, mag64, k65536, slot, ph, qslot, qph, acc);
                    break;
                case 2:
                    run_tile<C, 2>(p, bars, abort, ring, sbring, lo, kl, qd, pr, lane, s_beg, s_end, t * p.R, mag1024,
                                   mag64, k65536, slot, ph, qslot, qph, acc);
                    break;
                case 1:
                    run_tile<C, 1>(p, bars, abort, ring, sbring, lo, kl, qd, pr, lane, s_beg, s_end, t * p.R, mag1024,
                                   mag64, k65536, slot, ph, qslot, qph, acc);
                    break;
                default:  // no block of this tile: keep the ring moving
                    run_tile<C, 0>(p, bars, abort, ring, sbring, lo, kl, qd, pr, lane, s_beg, s_end, t * p.R, mag1024,
                                   mag64, k65536, slot, ph, qslot, qph, acc);
            }

            // ---- tile epilogue.  Within the CTA: ((k-lane 0 + 1) + (k-lane 2 + 3)) through
            // bufa/bufb; then the k-lane 0 warps hold the CTA's sum of their blocks and push
            // the blocks the peer writes into the peer's recv buffer.
            if (tt > 0) named_bar_sync(kBarConsumers, kConsumerThreads);  // last tile's bufa/bufb readers are done
            if (kl & 1) {
                float* buf = kl == 1 ? bufa : bufb;
#pragma unroll
                for (int i = 0; i < C::MAXB; ++i) {
                    if (i >= nblk) break;
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int nt = 0; nt < C::NT; ++nt)
                            *reinterpret_cast<float2*>(buf + (16 * (qd + 4 * i) + pr + 8 * h) * MR + 8 * nt + 2 * tq) =
                                make_float2(acc[i][nt][2 * h], acc[i][nt][2 * h + 1]);
                }
            }
            named_bar_sync(kBarConsumers, kConsumerThreads);
            if (!(kl & 1)) {
                float* buf = kl == 0 ? bufa : bufb;
#pragma unroll
                for (int i = 0; i < C::MAXB; ++i) {
                    if (i >= nblk) break;
#pragma unroll
                    for (int h = 0; h < 2; ++h)
#pragma unroll
                        for (int nt = 0; nt < C::NT; ++nt) {
                            float2* q = reinterpret_cast<float2*>(buf + (16 * (qd + 4 * i) + pr + 8 * h) * MR + 8 * nt +
                                                                  2 * tq);
                            const float2 o = *q;
                            acc[i][nt][2 * h] += o.x;
                            acc[i][nt][2 * h + 1] += o.y;
                            if (kl == 2) *q = make_float2(acc[i][nt][2 * h], acc[i][nt][2 * h + 1]);
                        }
                }
            }
            named_bar_sync(kBarConsumers, kConsumerThreads);
            int own0, own1, own_rows;
            uint16_t* stg;
            if constexpr (CS <= 2) {
                own0 = cs > 1 ? (rank == 0 ? 0 : p.nb0) : 0;
                own1 = cs > 1 ? (rank == 0 ? p.nb0 : p.nb) : p.nb;
                own_rows = 16 * (own1 - own0);
                stg = reinterpret_cast<uint16_t*>(bufa);  // bf16 y of the owned rows, [m][row]
                if (kl == 0) {
                    const int peer0 = rank == 0 ? p.nb0 : 0;  // first block the peer writes
#pragma unroll
                    for (int i = 0; i < C::MAXB; ++i) {
                        if (i >= nblk) break;
#pragma unroll
                        for (int h = 0; h < 2; ++h)
#pragma unroll
                            for (int nt = 0; nt < C::NT; ++nt) {
                                const float2 o = *reinterpret_cast<const float2*>(
                                    bufb + (16 * (qd + 4 * i) + pr + 8 * h) * MR + 8 * nt + 2 * tq);
                                acc[i][nt][2 * h] += o.x;
                                acc[i][nt][2 * h + 1] += o.y;
                            }
                    }
                    if (cs > 1) {
                        if (tt > 0)  // the peer has read what we sent for the previous tile
                            mbar_wait_cluster_bounded(&bars->xdone, (tt - 1) & 1, abort, DFLASH_DEVERR_QMM_REDUCE);
                        if (tid == 0) mbar_arrive_expect_tx(&bars->xfull, (uint32_t)own_rows * MR * 4u);
                        const uint32_t peer = rank ^ 1u;
                        const uint32_t peer_recv = map_to_rank(smem_u32(recv), peer);
                        const uint32_t peer_bar = map_to_rank(smem_u32(&bars->xfull), peer);
#pragma unroll
                        for (int i = 0; i < C::MAXB; ++i) {
                            if (i >= nblk) break;
                            const int b = qd + 4 * i;
                            if (b >= own0 && b < own1) continue;
#pragma unroll
                            for (int h = 0; h < 2; ++h)
#pragma unroll
                                for (int nt = 0; nt < C::NT; ++nt)
                                    st_async_f32x2(
                                        peer_recv + (uint32_t)((16 * (b - peer0) + pr + 8 * h) * MR + 8 * nt + 2 * tq) * 4u,
                                        acc[i][nt][2 * h], acc[i][nt][2 * h + 1], peer_bar);
                        }
                        mbar_wait_cluster_bounded(&bars->xfull, tt & 1, abort, DFLASH_DEVERR_QMM_REDUCE);
                    }
                    // the owned rows: rank 0's partial first, then rank 1's, rounded once to bf16
#pragma unroll
                    for (int i = 0; i < C::MAXB; ++i) {
                        if (i >= nblk) break;
                        const int b = qd + 4 * i;
                        if (b < own0 || b >= own1) continue;
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const int rowl = 16 * (b - own0) + pr + 8 * h;
#pragma unroll
                            for (int nt = 0; nt < C::NT; ++nt)
#pragma unroll
                                for (int e = 0; e < 2; ++e) {
                                    const int m = 8 * nt + 2 * tq + e;
                                    float v = acc[i][nt][2 * h + e];
                                    if (cs > 1) {
                                        const float o = recv[rowl * MR + m];
                                        v = rank == 0 ? v + o : o + v;
                                    }
                                    const __nv_bfloat16 o = __float2bfloat16_rn(v);
                                    stg[m * own_rows + rowl] = *reinterpret_cast<const uint16_t*>(&o);
                                }
                        }
                    }
                }
                named_bar_sync(kBarConsumers, kConsumerThreads);
                // the peer may refill recv once we are past reading it (only if it has another tile)
                if (cs > 1 && tid == 0 && t + ncl < p.ntiles)
                    mbar_arrive_remote(map_to_rank(smem_u32(&bars->xdone), rank ^ 1u));
            } else {
                // Cluster rank r owns (reduces and writes) blocks [nb r / cs, nb (r + 1) / cs) of
                // the tile.  The k-lane 0 warps park the CTA's partial of every block in bufa;
                // then all consumer threads push the rows other ranks own into their receive
                // buffers (slot = sender rank, skipping the owner), wait for their own rows
                // from the other ranks, and sum them in rank order into the bf16 staging
                // buffer (bufb).
                own0 = (int)((uint32_t)p.nb * rank / cs);
                own1 = (int)((uint32_t)p.nb * (rank + 1) / cs);
                own_rows = 16 * (own1 - own0);
                stg = reinterpret_cast<uint16_t*>(bufb);
                if (kl == 0) {
#pragma unroll
                    for (int i = 0; i < C::MAXB; ++i) {
                        if (i >= nblk) break;
#pragma unroll
                        for (int h = 0; h < 2; ++h)
#pragma unroll
                            for (int nt = 0; nt < C::NT; ++nt) {
                                float2* q = reinterpret_cast<float2*>(bufa + (16 * (qd + 4 * i) + pr + 8 * h) * MR +
                                                                      8 * nt + 2 * tq);
                                const float2 o = *reinterpret_cast<const float2*>(
                                    bufb + (16 * (qd + 4 * i) + pr + 8 * h) * MR + 8 * nt + 2 * tq);
                                *q = make_float2(acc[i][nt][2 * h] + o.x, acc[i][nt][2 * h + 1] + o.y);
                            }
                    }
                }
                named_bar_sync(kBarConsumers, kConsumerThreads);
                if (tt > 0)  // every receiver has read what we sent for the previous tile
                    mbar_wait_cluster_bounded(&bars->xdone, (tt - 1) & 1, abort, DFLASH_DEVERR_QMM_REDUCE);
                if (tid == 0) mbar_arrive_expect_tx(&bars->xfull, (cs - 1) * (uint32_t)own_rows * MR * 4u);
                const uint32_t recv_base = smem_u32(recv), xfull_base = smem_u32(&bars->xfull);
                const uint32_t recv_cap = (cs - 1) * (uint32_t)p.own_stride * MR * 4u;
                constexpr int P2 = MR / 2;  // float2 per row
                for (int e = tid; e < p.nb * 16 * P2; e += kConsumerThreads) {
                    const int row = e / P2, c2 = e - row * P2, b = row >> 4;
                    if (b >= own0 && b < own1) continue;
                    uint32_t o = 0;  // owner of block b
                    while (o + 1 < cs && (int)((uint32_t)p.nb * (o + 1) / cs) <= b) ++o;
                    const int o0 = (int)((uint32_t)p.nb * o / cs);
                    const uint32_t slot = rank < o ? rank : rank - 1;
                    const uint32_t off = ((slot * (uint32_t)p.own_stride + (uint32_t)(row - 16 * o0)) * MR + 2 * c2) * 4u;
                    if (off + 8u > recv_cap) {  // cannot happen for a consistent plan; never write past the buffer
                        atomicOr(&g_device_error, DFLASH_DEVERR_QMM_REDUCE);
                        continue;
                    }
                    const float2 v = *reinterpret_cast<const float2*>(bufa + row * MR + 2 * c2);
                    st_async_f32x2(map_to_rank(recv_base, o) + off, v.x, v.y, map_to_rank(xfull_base, o));
                }
                mbar_wait_cluster_bounded(&bars->xfull, tt & 1, abort, DFLASH_DEVERR_QMM_REDUCE);
                for (int e = tid; e < own_rows * MR; e += kConsumerThreads) {
                    const int rowl = e / MR, m = e - rowl * MR;
                    float v = 0.f;
#pragma unroll
                    for (uint32_t r = 0; r < cs; ++r) {
                        if (r == rank) {
                            v += bufa[(16 * own0 + rowl) * MR + m];
                        } else {
                            const uint32_t sl = r < rank ? r : r - 1;
                            v += recv[(sl * p.own_stride + rowl) * MR + m];
                        }
                    }
                    const __nv_bfloat16 o = __float2bfloat16_rn(v);
                    stg[m * own_rows + rowl] = *reinterpret_cast<const uint16_t*>(&o);
                }
                named_bar_sync(kBarConsumers, kConsumerThreads);
                // the senders may refill recv once we are past reading it (only if they have another tile)
                if (tid == 0 && t + ncl < p.ntiles) {
#pragma unroll
                    for (uint32_t r = 0; r < cs; ++r)
                        if (r != rank) mbar_arrive_remote(map_to_rank(smem_u32(&bars->xdone), r));
                }
            }
            // y rows of the owned blocks, from the staging buffer
            const int n0 = t * p.R + 16 * own0;
            if (p.argmax_keys) {
                // warp m scans row m of the owned outputs; lanes keep their best key, the
                // warp reduces, lane 0 folds it into the row's global key
                for (int m = warp; m < p.M; m += kConsumerWarps) {
                    unsigned long long best = 0ull;
                    for (int r = lane; r < own_rows; r += 32) {
                        const int n = n0 + r;
                        if (n >= p.N) break;
                        const uint32_t u = static_cast<uint32_t>(stg[m * own_rows + r]) << 16;
                        const uint32_t ord = (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // order of the float
                        const unsigned long long key =
                            (static_cast<unsigned long long>(ord) << 32) | (~static_cast<uint32_t>(n + p.argmax_base));
                        best = key > best ? key : best;
                    }
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
                        best = other > best ? other : best;
                    }
                    if (lane == 0 && best) atomicMax(p.argmax_keys + m, best);
                }
            } else if (p.push) {
                const int chunks = own_rows / 8;
                const uint64_t hi = (uint64_t)push_epoch << 32;
                for (int e = tid; e < p.M * chunks; e += kConsumerThreads) {
                    const int m = e / chunks, c = e - m * chunks;
                    const int n = n0 + 8 * c;
                    if (n < p.N) {
                        const uint4 v = *reinterpret_cast<const uint4*>(stg + m * own_rows + 8 * c);
                        const size_t w0 = ((size_t)m * p.N + n) / 2;
                        for (int r = 0; r < p.world; ++r) {
                            uint64_t* d = tp::slot_ptr(p.xb.b[r], p.world, p.M, p.N, p.set, p.rank) + w0;
                            tp::st_relaxed_sys_u64(d, hi | v.x);
                            tp::st_relaxed_sys_u64(d + 1, hi | v.y);
                            tp::st_relaxed_sys_u64(d + 2, hi | v.z);
                            tp::st_relaxed_sys_u64(d + 3, hi | v.w);
                        }
                    }
                }
            } else if (p.y_vec) {
                const int chunks = own_rows / 8;
                for (int e = tid; e < p.M * chunks; e += kConsumerThreads) {
                    const int m = e / chunks, c = e - m * chunks;
                    const int n = n0 + 8 * c;
                    if (n < p.N)
                        *reinterpret_cast<uint4*>(p.y + (size_t)m * p.N + n) =
                            *reinterpret_cast<const uint4*>(stg + m * own_rows + 8 * c);
                }
            } else {
                for (int e = tid; e < p.M * own_rows; e += kConsumerThreads) {
                    const int m = e / own_rows, r = e - m * own_rows;
                    if (n0 + r < p.N) p.y[(size_t)m * p.N + n0 + r] = stg[m * own_rows + r];
                }
            }
        }
    }
done:
    // No CTA leaves while its peer may still touch its shared memory.  On the normal path
    // the exchange barriers already guarantee that; this covers the error paths, where a
    // bounded wait gave up.  Relaxed: it orders no memory, so it does not wait for y.
    __syncwarp();
    cluster_sync_relaxed();
}

// ------------------------------------------------------------------ host side

struct Shape {
    int M, N, K, group, bits;
};

// Input transform and output destination of one call (dflash_qmm_ex).
struct Options {
    bool swiglu = false;  // x is [M, 2K] = [gate | up]; the input is bf16(silu(gate) * up)
    bool push = false;    // y goes to the peer exchange instead of memory
    int rank = 0, world = 1, set = 0;
    tp::Bases xb = {};
    unsigned long long* argmax_keys = nullptr;  // y is reduced to per-row argmax keys instead
    int argmax_base = 0;
};

struct Plan {
    int cs, nclusters, R, nb, nb0, own_stride, ntiles, S, NS, NSB;
    uint32_t stage_bytes, sb_bytes, red_off, red_bytes, recv_off, bar_off;
    size_t smem;
};

template <class C>
inline int stages_along_k(int K) {
    return (K + C::STAGE_K - 1) / C::STAGE_K;
}

inline uint32_t round_up_u32(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// Scale/bias slots the producer opens within its first `ns` stage issues (the only
// issues made before any consumer runs, so the ring must hold them all).
template <class C>
int first_batch_sb_slots(int S, int cs, int ns) {
    int worst = 0;
    for (int rank = 0; rank < cs; ++rank) {
        const int s_beg = (int)((long long)S * rank / cs), s_end = (int)((long long)S * (rank + 1) / cs);
        const int nst = s_end - s_beg;
        if (nst <= 0) continue;
        int slots = 0;
        for (int j = 0; j < ns; ++j) {
            const int s = s_beg + j % nst;
            if (s == s_beg || s % C::SBP == 0) ++slots;
        }
        worst = slots > worst ? slots : worst;
    }
    return worst;
}

// Cost model of one CTA's work, used to choose the cluster size and tile height: a stage
// costs a fixed issue/hand-off time plus its bytes at one SM's share of the HBM stream,
// and every tile ends in an epilogue that grows with the ranks exchanging partials.
constexpr double kStageFixedUs = 0.25;
constexpr double kSmBytesPerUs = 44000.0;
constexpr double kEpilogueUs = 1.0, kEpiloguePerRankUs = 0.3;

// Tile height and grid: clusters of cs CTAs (one per SM) split K into cs contiguous
// ranges; tiles of at most 256 rows, sized so that every cluster gets the same number of
// tiles (to within one) and the tiles the same height.  Among cs in {1, 2, 4, 8} and the
// tiles-per-cluster counts, the plan with the lowest modelled time wins; then the deepest
// ring that fits.  max_clusters[i] is how many clusters of 2^i CTAs fit on the device.
template <class C>
Plan make_plan(const Shape& s, const int* cmax_by_lg) {
    Plan pl;
    pl.S = stages_along_k<C>(s.K);
    const int NB = (s.N + 15) / 16;
    double best = 1e30;
    pl.cs = 1;
    pl.nb = 1;
    for (int lg = 0, cs = 1; cs <= kMaxCluster; ++lg, cs *= 2) {
        if (cs > 1 && pl.S < cs) break;  // every CTA takes at least one stage
        const int cmax = cmax_by_lg[lg];
        if (cmax < 1) continue;
        const int sp = (pl.S + cs - 1) / cs;
        for (int T = 1; T <= 8; ++T) {
            int nb = (NB + cmax * T - 1) / (cmax * T);
            if (nb > kMaxTileBlocks / 4 * C::MAXB) nb = kMaxTileBlocks / 4 * C::MAXB;
            if (nb < 1) nb = 1;
            const int ntiles = (s.N + 16 * nb - 1) / (16 * nb);
            const int ncl = ntiles < cmax ? ntiles : cmax;
            const int teff = (ntiles + ncl - 1) / ncl;
            const double cost = teff * (sp * (kStageFixedUs + 16.0 * nb * kRowBytes / kSmBytesPerUs) + kEpilogueUs +
                                        kEpiloguePerRankUs * (cs - 1));
            if (cost < best - 1e-9) {
                best = cost;
                pl.cs = cs;
                pl.nb = nb;
            }
        }
    }
    pl.R = 16 * pl.nb;
    pl.ntiles = (s.N + pl.R - 1) / pl.R;
    const int cmax = cmax_by_lg[pl.cs == 1 ? 0 : pl.cs == 2 ? 1 : pl.cs == 4 ? 2 : 3];
    pl.nclusters = pl.ntiles < cmax ? pl.ntiles : cmax;
    pl.nb0 = (pl.nb + 1) / 2;
    pl.own_stride = 16 * ((pl.nb + pl.cs - 1) / pl.cs);
    pl.stage_bytes = round_up_u32((uint32_t)pl.R * kRowBytes + C::PKT, 1024);
    pl.sb_bytes = C::STMA ? round_up_u32(2u * pl.R * 16, 128) : 0;
    pl.red_bytes = round_up_u32((uint32_t)pl.R * C::MR * 4, 128);
    const uint32_t recv_bytes =
        pl.cs <= 2 ? round_up_u32((uint32_t)pl.nb0 * 16 * C::MR * 4, 128)
                   : round_up_u32((uint32_t)(pl.cs - 1) * pl.own_stride * C::MR * 4, 128);
    const uint32_t bar_bytes = round_up_u32(sizeof(Bars), 128);
    pl.NS = 0;
    pl.NSB = 1;
    for (int ns = kMaxStages; ns >= 2; --ns) {
        int nsb = 1;
        if (C::STMA) {
            nsb = (ns + C::SBP - 1) / C::SBP + 1;
            const int need = first_batch_sb_slots<C>(pl.S, pl.cs, ns);
            if (nsb < need) nsb = need;
            if (nsb > kMaxSbStages) continue;
        }
        const size_t total = 1024 + (size_t)ns * pl.stage_bytes + (C::STMA ? (size_t)nsb * pl.sb_bytes : 0) +
                             2 * (size_t)pl.red_bytes + recv_bytes + bar_bytes;
        if (total <= (size_t)kSmemLimit) {
            pl.NS = ns;
            pl.NSB = nsb;
            break;
        }
    }
    pl.red_off = pl.NS * pl.stage_bytes + (C::STMA ? pl.NSB * pl.sb_bytes : 0);
    pl.recv_off = pl.red_off + 2 * pl.red_bytes;
    pl.bar_off = pl.recv_off + recv_bytes;
    pl.smem = 1024 + (size_t)pl.bar_off + bar_bytes;
    return pl;
}

template <class C>
using QmmKernel = void (*)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const Params);

template <class C>
QmmKernel<C> kernel_for(int cs) {
    switch (cs) {
        case 1: return qmm_kernel<C, 1>;
        case 2: return qmm_kernel<C, 2>;
        case 4: return qmm_kernel<C, 4>;
        default: return qmm_kernel<C, 8>;
    }
}

// How many clusters of 1, 2, 4 and 8 CTAs of qmm_kernel<C, cs> (full shared memory) fit on
// `dev` at once; queried once per device (falls back to SMs / cs).
template <class C>
const int* max_clusters(int dev) {
    static std::mutex mu;
    static int cache[64][4];
    static bool done[64] = {false};
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!done[dev]) {
        const int sms = sm_count(dev);
        for (int lg = 0, cs = 1; lg < 4; ++lg, cs *= 2) {
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)cs);
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = kSmemLimit;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = cs;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, kernel_for<C>(cs), &cfg) != cudaSuccess || n < 1) {
                (void)cudaGetLastError();
                n = sms / cs;
            }
            cache[dev][lg] = n;
        }
        done[dev] = true;
    }
    return cache[dev];
}

template <class C>
int launch(const Shape& s, const dflash_bf16* x, const uint32_t* w, const dflash_bf16* scales,
           const dflash_bf16* biases, dflash_bf16* y, void* ws, cudaStream_t stream, const Options& o) {
    static std::once_flag once;
    static cudaError_t attr_err = cudaSuccess;
    static int launch_regs = 0;
    std::call_once(once, [] {
        launch_regs = 1 << 30;
        for (int cs = 1; cs <= kMaxCluster && attr_err == cudaSuccess; cs *= 2) {
            attr_err = cudaFuncSetAttribute(kernel_for<C>(cs), cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
            cudaFuncAttributes fa;
            if (attr_err == cudaSuccess) attr_err = cudaFuncGetAttributes(&fa, kernel_for<C>(cs));
            if (attr_err == cudaSuccess && fa.numRegs < launch_regs) launch_regs = fa.numRegs;
        }
    });
    if (attr_err != cudaSuccess)
        return fail(DFLASH_ERR_CUDA, "cudaFuncSetAttribute(qmm): %s", cudaGetErrorString(attr_err));
    // the warpgroups' setmaxnreg shares must fit the registers the block is launched with
    if (launch_regs * kThreads < kConsumerThreads * kConsumerRegs + 128 * kProducerRegs)
        return fail(DFLASH_ERR_UNSUPPORTED, "qmm kernel built with %d registers per thread, %d needed", launch_regs,
                    kLaunchRegs);

    int dev = 0;
    DFLASH_CUDA_TRY(cudaGetDevice(&dev));
    // The plan and the three tensor maps depend only on the device, the shape and the
    // weight / scale / bias addresses: a small direct-mapped cache keeps them, so a call
    // on weights seen before costs no planning and no tensor-map encoding on the host.
    struct Entry {
        bool valid;
        int dev, N, K;
        const void *w, *s, *b;
        Plan pl;
        CUtensorMap tm_w, tm_s, tm_b;
    };
    constexpr int kEntries = 512;
    static std::mutex cache_mu;
    static Entry cache[kEntries];
    const size_t h = (reinterpret_cast<uintptr_t>(w) >> 8) ^ ((size_t)s.N * 2654435761u) ^ ((size_t)s.K * 40503u) ^
                     ((size_t)dev << 7);
    Entry& slot = cache[h % kEntries];
    Plan pl;
    CUtensorMap tm_w, tm_s, tm_b;
    bool hit = false;
    {
        std::lock_guard<std::mutex> lock(cache_mu);
        if (slot.valid && slot.dev == dev && slot.N == s.N && slot.K == s.K && slot.w == w && slot.s == scales &&
            slot.b == biases) {
            pl = slot.pl;
            tm_w = slot.tm_w;
            tm_s = slot.tm_s;
            tm_b = slot.tm_b;
            hit = true;
        }
    }
    const int* cmax = max_clusters<C>(dev);
    if (!hit) pl = make_plan<C>(s, cmax);
    static const bool log_plan = getenv("DFLASH_QMM_LOG_PLAN") != nullptr;
    if (log_plan)  // diagnostics: the plan of every launch on stderr
        fprintf(stderr,
                "dflash_qmm plan: M=%d N=%d K=%d g=%d b=%d -> cs=%d R=%d tiles=%d clusters=%d S=%d NS=%d NSB=%d "
                "smem=%zu (fit: %d %d %d %d clusters of 1 2 4 8)\n",
                s.M, s.N, s.K, s.group, s.bits, pl.cs, pl.R, pl.ntiles, pl.nclusters, pl.S, pl.NS, pl.NSB, pl.smem,
                cmax[0], cmax[1], cmax[2], cmax[3]);
    if (pl.NS < 2) return fail(DFLASH_ERR_UNSUPPORTED, "qmm: no shared-memory plan for N=%d K=%d", s.N, s.K);
    const int GT = s.K / s.group;

    if (!hit) {
        int st;
        const uint64_t words = (uint64_t)s.K * s.bits / 32;
        st = encode_tensor_map_2d(&tm_w, CU_TENSOR_MAP_DATA_TYPE_UINT32, w, words, (uint64_t)s.N, words * 4,
                                  kRowBytes / 4, pl.R, CU_TENSOR_MAP_SWIZZLE_128B);
        if (st) return st;
        if constexpr (C::STMA) {
            st = encode_tensor_map_2d(&tm_s, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, scales, (uint64_t)GT, (uint64_t)s.N,
                                      (uint64_t)GT * 2, 8, pl.R, CU_TENSOR_MAP_SWIZZLE_NONE);
            if (st) return st;
            st = encode_tensor_map_2d(&tm_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, biases, (uint64_t)GT, (uint64_t)s.N,
                                      (uint64_t)GT * 2, 8, pl.R, CU_TENSOR_MAP_SWIZZLE_NONE);
            if (st) return st;
        } else {
            tm_s = tm_w;
            tm_b = tm_w;
        }
        std::lock_guard<std::mutex> lock(cache_mu);
        slot.valid = true;
        slot.dev = dev;
        slot.N = s.N;
        slot.K = s.K;
        slot.w = w;
        slot.s = scales;
        slot.b = biases;
        slot.pl = pl;
        slot.tm_w = tm_w;
        slot.tm_s = tm_s;
        slot.tm_b = tm_b;
    }

    Params p;
    p.packets = reinterpret_cast<const uint8_t*>(ws);
    p.scales = scales;
    p.biases = biases;
    p.y = y;
    p.M = s.M;
    p.N = s.N;
    p.K = s.K;
    p.GT = GT;
    p.R = pl.R;
    p.nb = pl.nb;
    p.nb0 = pl.nb0;
    p.own_stride = pl.own_stride;
    p.ntiles = pl.ntiles;
    p.S = pl.S;
    p.NS = pl.NS;
    p.NSB = pl.NSB;
    p.y_vec = (s.N % 8 == 0) && aligned16(y);
    p.push = o.push ? 1 : 0;
    p.rank = o.rank;
    p.world = o.world;
    p.set = o.set;
    p.xb = o.xb;
    p.argmax_keys = o.argmax_keys;
    p.argmax_base = o.argmax_base;
    p.stage_bytes = pl.stage_bytes;
    p.sb_bytes = pl.sb_bytes;
    p.red_off = pl.red_off;
    p.red_bytes = pl.red_bytes;
    p.recv_off = pl.recv_off;
    p.bar_off = pl.bar_off;

    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = pl.cs;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    {
        // prep: one thread per (x row, run of 8 k) of every stage
        const long long threads = (long long)C::MR * pl.S * (C::STAGE_K / 8);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)((threads + kPrepThreads - 1) / kPrepThreads));
        cfg.blockDim = dim3(kPrepThreads);
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        DFLASH_CUDA_TRY(cudaLaunchKernelEx(&cfg, o.swiglu ? qmm_prep_kernel<C, true> : qmm_prep_kernel<C, false>,
                                           reinterpret_cast<const uint16_t*>(x), reinterpret_cast<uint8_t*>(ws), s.M,
                                           s.K, pl.S, o.argmax_keys));
    }
    {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(pl.nclusters * pl.cs));
        cfg.blockDim = dim3(kThreads);
        cfg.dynamicSmemBytes = pl.smem;
        cfg.stream = stream;
        cfg.attrs = attr;
        cfg.numAttrs = 2;
        DFLASH_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel_for<C>(pl.cs), tm_w, tm_s, tm_b, p));
    }
    return DFLASH_OK;
}

template <int BITS, int GROUP, int NT>
int dispatch_stma(const Shape& s, const dflash_bf16* x, const uint32_t* w, const dflash_bf16* sc,
                  const dflash_bf16* bi, dflash_bf16* y, void* ws, cudaStream_t st, const Options& o) {
    const bool stma = ((s.K / s.group) % 8 == 0) && aligned16(sc) && aligned16(bi);
    if (stma) return launch<Cfg<BITS, GROUP, NT, true>>(s, x, w, sc, bi, y, ws, st, o);
    return launch<Cfg<BITS, GROUP, NT, false>>(s, x, w, sc, bi, y, ws, st, o);
}

template <int BITS, int GROUP>
int dispatch_nt(const Shape& s, const dflash_bf16* x, const uint32_t* w, const dflash_bf16* sc,
                const dflash_bf16* bi, dflash_bf16* y, void* ws, cudaStream_t st, const Options& o) {
    if (s.M <= 8) return dispatch_stma<BITS, GROUP, 1>(s, x, w, sc, bi, y, ws, st, o);
    return dispatch_stma<BITS, GROUP, 2>(s, x, w, sc, bi, y, ws, st, o);
}

template <int BITS>
int dispatch_group(const Shape& s, const dflash_bf16* x, const uint32_t* w, const dflash_bf16* sc,
                   const dflash_bf16* bi, dflash_bf16* y, void* ws, cudaStream_t st, const Options& o = Options()) {
    switch (s.group) {
        case 32: return dispatch_nt<BITS, 32>(s, x, w, sc, bi, y, ws, st, o);
        case 64: return dispatch_nt<BITS, 64>(s, x, w, sc, bi, y, ws, st, o);
        case 128: return dispatch_nt<BITS, 128>(s, x, w, sc, bi, y, ws, st, o);
    }
    return fail(DFLASH_ERR_UNSUPPORTED, "group_size %d not in {32, 64, 128}", s.group);
}

// The workspace holds the x packets of every stage along K: its size depends on bits,
// group (segments per unit), M (x rows per packet) and K, not on N.
template <int BITS, int GROUP>
size_t packets_for(int M, int K) {
    if (M <= 8) return (size_t)stages_along_k<Cfg<BITS, GROUP, 1, true>>(K) * Cfg<BITS, GROUP, 1, true>::PKT;
    return (size_t)stages_along_k<Cfg<BITS, GROUP, 2, true>>(K) * Cfg<BITS, GROUP, 2, true>::PKT;
}

inline size_t workspace_size(int M, int K, int group, int bits) {
    size_t b = 0;
    if (bits == 4)
        b = group == 32 ? packets_for<4, 32>(M, K) : group == 64 ? packets_for<4, 64>(M, K) : packets_for<4, 128>(M, K);
    else
        b = group == 32 ? packets_for<8, 32>(M, K) : group == 64 ? packets_for<8, 64>(M, K) : packets_for<8, 128>(M, K);
    return (b + 255) / 256 * 256;
}

int validate(const Shape& s) {
    if (s.bits != 4 && s.bits != 8) return fail(DFLASH_ERR_UNSUPPORTED, "bits %d not in {4, 8}", s.bits);
    if (s.group != 32 && s.group != 64 && s.group != 128)
        return fail(DFLASH_ERR_UNSUPPORTED, "group_size %d not in {32, 64, 128}", s.group);
    if (s.M < 1 || s.M > 16) return fail(DFLASH_ERR_UNSUPPORTED, "M=%d outside 1..16", s.M);
    if (s.N < 1 || s.K < 1) return fail(DFLASH_ERR_INVALID_ARGUMENT, "N=%d K=%d must be positive", s.N, s.K);
    if (s.N > kMaxN) return fail(DFLASH_ERR_UNSUPPORTED, "N=%d above the supported %d", s.N, kMaxN);
    if (s.K % s.group != 0)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "K=%d is not a multiple of group_size %d", s.K, s.group);
    return DFLASH_OK;
}

}  // namespace qmm
}  // namespace dflash

extern "C" size_t dflash_qmm_workspace_bytes(int M, int N, int K, int group_size, int bits) {
    if (N < 1 || K < 1 || M < 1 || M > 16 || (group_size != 32 && group_size != 64 && group_size != 128) ||
        K % group_size != 0 || (bits != 4 && bits != 8))
        return 0;
    return dflash::qmm::workspace_size(M, K, group_size, bits);
}

extern "C" int dflash_qmm_supported(int N, int K, int group_size, int bits) {
    if ((bits != 4 && bits != 8) || (group_size != 32 && group_size != 64 && group_size != 128)) return 0;
    if (N < 1 || K < 1 || K % group_size != 0 || N > dflash::qmm::kMaxN) return 0;
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
    const size_t need = qmm::workspace_size(M, K, group_size, bits);
    if (!workspace || workspace_bytes < need || !aligned16(workspace))
        return fail(DFLASH_ERR_WORKSPACE, "dflash_qmm: a 16-byte aligned workspace of %zu bytes is required (got %zu)",
                    need, workspace_bytes);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (bits == 4) return qmm::dispatch_group<4>(s, x, w, scales, biases, y, workspace, st);
    return qmm::dispatch_group<8>(s, x, w, scales, biases, y, workspace, st);
}

// ------------------------------------------------------------------ entry point on host buffers
//
// dflash_qmm for x and y in host memory: the workspace also holds the device copies of
// x and y, and the call queues the copy in, the two kernels and the copy out on the
// stream, so a host issues one library call per matmul instead of three.
namespace dflash {
namespace qmm {

inline size_t round256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace qmm
}  // namespace dflash

extern "C" size_t dflash_qmm_host_workspace_bytes(int M, int N, int K, int group_size, int bits) {
    const size_t packets = dflash_qmm_workspace_bytes(M, N, K, group_size, bits);
    if (!packets) return 0;
    return packets + dflash::qmm::round256((size_t)2 * M * K) + dflash::qmm::round256((size_t)2 * M * N);
}

extern "C" int dflash_qmm_host(const dflash_bf16* x_host, const uint32_t* w, const dflash_bf16* scales,
                               const dflash_bf16* biases, dflash_bf16* y_host, int M, int N, int K, int group_size,
                               int bits, void* workspace, size_t workspace_bytes, dflash_stream_t stream) {
    using namespace dflash;
    qmm::Shape s{M, N, K, group_size, bits};
    if (int st = qmm::validate(s)) return st;
    if (!x_host || !w || !scales || !biases || !y_host)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_qmm_host: null pointer");
    if (!aligned16(w)) return fail(DFLASH_ERR_MISALIGNED, "dflash_qmm_host: w must be 16-byte aligned");
    const size_t need = dflash_qmm_host_workspace_bytes(M, N, K, group_size, bits);
    if (!workspace || workspace_bytes < need || !aligned16(workspace))
        return fail(DFLASH_ERR_WORKSPACE,
                    "dflash_qmm_host: a 16-byte aligned workspace of %zu bytes is required (got %zu)", need,
                    workspace_bytes);
    const size_t packets = qmm::workspace_size(M, K, group_size, bits);
    uint8_t* base = static_cast<uint8_t*>(workspace);
    dflash_bf16* x_dev = reinterpret_cast<dflash_bf16*>(base + packets);
    dflash_bf16* y_dev = reinterpret_cast<dflash_bf16*>(base + packets + qmm::round256((size_t)2 * M * K));
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    DFLASH_CUDA_TRY(cudaMemcpyAsync(x_dev, x_host, (size_t)2 * M * K, cudaMemcpyDefault, st));
    const int r = bits == 4 ? qmm::dispatch_group<4>(s, x_dev, w, scales, biases, y_dev, workspace, st)
                            : qmm::dispatch_group<8>(s, x_dev, w, scales, biases, y_dev, workspace, st);
    if (r) return r;
    DFLASH_CUDA_TRY(cudaMemcpyAsync(y_host, y_dev, (size_t)2 * M * N, cudaMemcpyDefault, st));
    return DFLASH_OK;
}

extern "C" int dflash_qmm_ex(const dflash_bf16* x, const uint32_t* w, const dflash_bf16* scales,
                             const dflash_bf16* biases, dflash_bf16* y, int M, int N, int K, int group_size, int bits,
                             void* workspace, size_t workspace_bytes, const dflash_qmm_options* opts,
                             dflash_stream_t stream) {
    using namespace dflash;
    qmm::Shape s{M, N, K, group_size, bits};
    if (int st = qmm::validate(s)) return st;
    qmm::Options o;
    if (opts) {
        o.swiglu = opts->x_swiglu != 0;
        o.push = opts->push != 0;
        o.argmax_keys = reinterpret_cast<unsigned long long*>(opts->argmax_keys);
        o.argmax_base = opts->argmax_index_base;
        if (opts->argmax_index_base < 0)
            return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_qmm_ex: negative argmax_index_base");
    }
    if (o.push && o.argmax_keys)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_qmm_ex: push and argmax are exclusive");
    if (o.argmax_keys && (reinterpret_cast<uintptr_t>(o.argmax_keys) & 7u))
        return fail(DFLASH_ERR_MISALIGNED, "dflash_qmm_ex: argmax_keys must be 8-byte aligned");
    if (!x || !w || !scales || !biases || (!y && !o.push && !o.argmax_keys))
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_qmm_ex: null tensor pointer");
    if (!aligned16(x) || !aligned16(w))
        return fail(DFLASH_ERR_MISALIGNED, "dflash_qmm_ex: x and w must be 16-byte aligned");
    if (o.swiglu && K % 8)
        return fail(DFLASH_ERR_MISALIGNED, "dflash_qmm_ex: the up half of [gate | up] must start 16-byte aligned");
    if (o.push) {
        if (opts->world < 1 || opts->world > tp::kMaxRanks || opts->rank < 0 || opts->rank >= opts->world ||
            (opts->set != 0 && opts->set != 1) || !opts->bases)
            return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_qmm_ex: bad push rank/world/set/bases");
        if (N % 8) return fail(DFLASH_ERR_UNSUPPORTED, "dflash_qmm_ex: pushing needs N %% 8 == 0 (N=%d)", N);
        o.rank = opts->rank;
        o.world = opts->world;
        o.set = opts->set;
        for (int r = 0; r < o.world; ++r) {
            if (!opts->bases[r] || !aligned16(opts->bases[r]))
                return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_qmm_ex: bad exchange base %d", r);
            o.xb.b[r] = opts->bases[r];
        }
    }
    const size_t need = qmm::workspace_size(M, K, group_size, bits);
    if (!workspace || workspace_bytes < need || !aligned16(workspace))
        return fail(DFLASH_ERR_WORKSPACE,
                    "dflash_qmm_ex: a 16-byte aligned workspace of %zu bytes is required (got %zu)", need,
                    workspace_bytes);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (bits == 4) return qmm::dispatch_group<4>(s, x, w, scales, biases, y, workspace, st, o);
    return qmm::dispatch_group<8>(s, x, w, scales, biases, y, workspace, st, o);
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

// The calling thread's current CUDA context (driver API, resolved at run time like the
// tensor-map encoder), or null when none is current yet.
void* current_context() {
    using CtxGetCurrentFn = CUresult (*)(CUcontext*);
    static CtxGetCurrentFn fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        const cudaError_t e = cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q);
        return (e == cudaSuccess && q == cudaDriverEntryPointSuccess) ? reinterpret_cast<CtxGetCurrentFn>(f)
                                                                      : nullptr;
    }();
    CUcontext c = nullptr;
    if (!fn || fn(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}

// Device address of g_static_scratch on the current device.  Resolved on a device's first
// call and cached together with the context it was resolved in; a different context on
// that device (after cudaDeviceReset, the module is loaded again at a new address)
// resolves it again, so a cached address never outlives its context.
int static_scratch(void** out) {
    static std::mutex mu;
    static void* ptr[64] = {nullptr};
    static void* ctx[64] = {nullptr};
    int dev = 0;
    DFLASH_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(DFLASH_ERR_UNSUPPORTED, "device ordinal %d above 63", dev);
    std::lock_guard<std::mutex> lock(mu);
    void* now = current_context();
    if (!ptr[dev] || !now || now != ctx[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess)
            return fail(DFLASH_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
        ptr[dev] = p;
        ctx[dev] = current_context();  // current now: the lookup above made the device's context current
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
