// Gated-delta recurrence on sm_100a: the verify-time step (whose inputs are the
// capture) and the rollback replay from the pre-round snapshot.
//
// Reference contract: rollbackGatedDeltaRound / rollbackGatedDeltaTree, called at
// Sources/DFlashKit/DFlashSpeculativeGenerator.swift:455-460, must leave the state a
// committed forward over the kept positions would have left
// (Tests/DFlashKitTests/GatedDeltaRollbackTests.swift:84-111).  The step, the tree
// step and the replay are one kernel template run in three modes, and all run the
// per-position update through the same device function, so a replay of `keep` positions
// performs exactly the arithmetic a committed step over those positions does.
//
// Per head the fp32 state S is [dv, dk], dk contiguous.  Rows of S are independent:
//     u_i   = v_i - alpha * sum_j S_ij k_j
//     S_ij <- alpha * S_ij + (beta * u_i) * k_j
// which is  S <- alpha S;  S <- S + beta (v - S k) k^T  with the decay applied first.
// The work is bound by reading the snapshot and writing the new state once
// (2 * 4 * dv * dk bytes per head).  Each row is held in registers by 8 threads (16 floats
// each for dk = 128) for all positions, with 128-byte coalesced row access.  On large grids
// each thread holds four rows (g, g + 8, g + 16, g + 24 of its block's 32): one
// shared-memory read of k_t serves all four, one transposed shuffle reduction sums their
// dot products, and the four rows' recurrences are independent chains the scheduler
// interleaves.  Grids too small to fill the SMs that way (a single layer's step at a
// verify block's 8 positions) hold one row per thread in blocks of 8 rows instead: four
// times the blocks and a quarter of the per-position chain.  The sums of a row use the
// same lane tree either way, so both layouts produce the same bits.  The arithmetic is
// packed fp32 (two lanes per FMA).  k (and q), the block's v, alpha and beta of the
// positions are staged in shared memory while the state loads are in flight, so the
// position loop reads no global memory.
#include "common.cuh"

namespace dflash {
namespace gdn {

constexpr int kRowThreads = 8;                             // threads per state row
constexpr int kRowGroups = 8;                              // row groups per block
constexpr int kBlockThreads = kRowThreads * kRowGroups;    // 64
constexpr int kRowsPerBlock = 32;                          // rows of S per block, four rows per thread
constexpr int kMaxPositions = 64;
constexpr int kStageBatch = 4;                             // global loads per thread per staging round
static_assert(kMaxPositions <= kBlockThreads, "alpha and beta are staged one position per thread");

struct RowList {
    int32_t r[kMaxPositions];
};

// Widens 4 consecutive bf16 (one 8-byte word) to fp32.
__device__ __forceinline__ float4 widen_bf16x4(const uint2 v) {
    return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xffff0000u),
                       __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xffff0000u));
}

// v of a row group's R rows at one position (one shared-memory read).
template <int R>
struct alignas(4 * R) RowVals {
    float x[R];
};

// Totals, over the 8 threads of a row group (lanes 8g' .. 8g'+7 of a warp), of the
// partial dot products a[j] of the group's R rows; every lane gets all of them.  Each
// total is ((a0 + a4) + (a2 + a6)) + ((a1 + a5) + (a3 + a7)) over the group's lanes, for
// one row or four.  Four rows: a transposed reduction, where each of three exchange steps
// halves the values a lane carries (after the last, lanes 2j and 2j+1 of the group hold
// the total of row j), then three exchanges hand every lane the other rows' totals.
// Every lane ends with the same bits.
template <int R>
__device__ __forceinline__ void group_sum(float (&a)[R]) {
    const unsigned kAll = 0xffffffffu;
    if constexpr (R == 1) {
        a[0] += __shfl_xor_sync(kAll, a[0], 4);
        a[0] += __shfl_xor_sync(kAll, a[0], 2);
        a[0] += __shfl_xor_sync(kAll, a[0], 1);
        return;
    } else {
        static_assert(R == 4, "one or four rows per thread");
        const bool b2 = threadIdx.x & 4, b1 = threadIdx.x & 2;
        float k0 = b2 ? a[2] : a[0], k1 = b2 ? a[3] : a[1];  // rows kept: {0, 1} or {2, 3}
        k0 += __shfl_xor_sync(kAll, b2 ? a[0] : a[2], 4);
        k1 += __shfl_xor_sync(kAll, b2 ? a[1] : a[3], 4);
        float t = b1 ? k1 : k0;  // row 2 b2 + b1
        t += __shfl_xor_sync(kAll, b1 ? k0 : k1, 2);
        t += __shfl_xor_sync(kAll, t, 1);
        const float x2 = __shfl_xor_sync(kAll, t, 2);  // row 2 b2 + !b1
        const float x4 = __shfl_xor_sync(kAll, t, 4);  // row 2 !b2 + b1
        const float x6 = __shfl_xor_sync(kAll, t, 6);  // row 2 !b2 + !b1
        const float lo = b1 ? x2 : t, hi = b1 ? t : x2, olo = b1 ? x6 : x4, ohi = b1 ? x4 : x6;
        a[0] = b2 ? olo : lo;
        a[1] = b2 ? ohi : hi;
        a[2] = b2 ? lo : olo;
        a[3] = b2 ? hi : ohi;
    }
}

// Packed fp32 arithmetic (two lanes per instruction, sm_100): a float4 chunk of a row is
// handled as two float2 halves.
__device__ __forceinline__ float2 lo2(const float4& v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(const float4& v) { return make_float2(v.z, v.w); }
__device__ __forceinline__ float4 cat4(const float2& a, const float2& b) { return make_float4(a.x, a.y, b.x, b.y); }

// Dot products of the thread's R row slices with CH chunks of a vector, summed over the
// row group, into d.
template <int CH, int R>
__device__ __forceinline__ void rows_dot(const float4 (&s)[R][CH], const float4 (&x)[CH], float (&d)[R]) {
    float2 acc[R];
#pragma unroll
    for (int j = 0; j < R; ++j) acc[j] = make_float2(0.f, 0.f);
#pragma unroll
    for (int c = 0; c < CH; ++c) {
#pragma unroll
        for (int j = 0; j < R; ++j) acc[j] = __ffma2_rn(lo2(s[j][c]), lo2(x[c]), acc[j]);
#pragma unroll
        for (int j = 0; j < R; ++j) acc[j] = __ffma2_rn(hi2(s[j][c]), hi2(x[c]), acc[j]);
    }
#pragma unroll
    for (int j = 0; j < R; ++j) d[j] = acc[j].x + acc[j].y;
    group_sum<R>(d);
}

// One position of the recurrence for the R row slices a thread holds: s the rows' CH
// float4 chunks, k the matching chunks of k_t (fp32), v the rows' v_t.
template <int CH, int R>
__device__ __forceinline__ void rows_step(float4 (&s)[R][CH], const float4 (&k)[CH], const RowVals<R>& v,
                                          float alpha, float beta) {
    float dot[R];
    rows_dot<CH, R>(s, k, dot);
    const float2 aa = make_float2(alpha, alpha);
#pragma unroll
    for (int j = 0; j < R; ++j) {
        const float bu = beta * (v.x[j] - alpha * dot[j]);
        const float2 bb = make_float2(bu, bu);
#pragma unroll
        for (int c = 0; c < CH; ++c)
            s[j][c] = cat4(__ffma2_rn(bb, lo2(k[c]), __fmul2_rn(aa, lo2(s[j][c]))),
                           __ffma2_rn(bb, hi2(k[c]), __fmul2_rn(aa, hi2(s[j][c]))));
    }
}

struct ReplayParams {
    const float* snapshot;
    float* state_out;
    const dflash_bf16* k;
    const dflash_bf16* v;
    const float* alpha;
    const float* beta;
    const dflash_bf16* q;     // step kernel only (may be null)
    dflash_bf16* out;         // step kernel only (may be null)
    float q_scale;
    int keep, width, heads, dk, dv;
    RowList rows;
    const int32_t* parents;   // tree step only: the block's parent list (device, width entries)
    int k_heads;              // heads of q and k (0: = heads); value head h reads key head h / (heads / k_heads)
};

// grid: (dv / (8 R), heads, layers) — (dv / (8 R), heads, width) for a tree step, block z
// taking the z-th leaf of the tree in row order; block: 64 threads = 8 row groups x 8
// threads, group g holding rows g, g + 8, ..., g + 8 (R - 1) of the block's 8 R (R = 4 or
// 1).  Thread q of a group holds float4 chunks q, q+8, q+16, ... of its rows (dk = 32 * CH).
//
// Tree step (TREE): the recurrence of a tree row is that of its root-to-row path, so
// each block runs the chain of one leaf's path from the same pre-round state and writes
// the outputs of the path's rows that no earlier leaf's path holds (every row is written
// by exactly one block; a row shared by several paths gets the same arithmetic on each).
// No state is written: after the round, dflash_gdn_replay rebuilds it from the snapshot
// over the accepted path.
// Dynamic shared memory of a block over n positions: k (and q times q_scale) widened to
// fp32 [n][dk], the block's rpb values of v per position (fp32, stored as the R-tuples a
// row group reads), alpha and beta.  Staged once, so the position loop touches no global
// memory and the snapshot loads are the only long waits.
__host__ __device__ inline size_t smem_bytes(int n, int dk, bool with_q, int rpb) {
    return (size_t)n * dk * 4 * (with_q ? 2 : 1) + (size_t)n * rpb * 4 + (size_t)n * 8;
}

// What a launch computes: the rollback replay (state only), the chain step (outputs and
// state) or the tree step (outputs only).
enum Mode { kReplay = 0, kStep = 1, kTree = 2 };

template <int CH, int MODE, int R>
__global__ void __launch_bounds__(kBlockThreads) gdn_kernel(const __grid_constant__ ReplayParams p) {
    constexpr int DK = 32 * CH;
    constexpr int RPB = kRowGroups * R;  // rows of S per block
    constexpr bool TREE = MODE == kTree;
    constexpr bool want_out = MODE != kReplay;
    const int n = TREE ? p.width : p.keep;  // positions staged
    extern __shared__ __align__(16) uint8_t dyn[];
    float(*ks)[DK] = reinterpret_cast<float(*)[DK]>(dyn);
    float(*qs_sh)[DK] = reinterpret_cast<float(*)[DK]>(dyn + (size_t)n * DK * 4);
    // vs[r][g] = v of rows g, g + 8, ..., g + 8 (R - 1) at position r
    RowVals<R>(*vs)[kRowGroups] =
        reinterpret_cast<RowVals<R>(*)[kRowGroups]>(dyn + (size_t)n * DK * 4 * (want_out ? 2 : 1));
    float2* ab = reinterpret_cast<float2*>(reinterpret_cast<uint8_t*>(vs) + (size_t)n * RPB * 4);
    __shared__ int32_t path_rows[TREE ? kMaxTreeRows : 1];
    __shared__ uint32_t path_info[2];  // tree: rows on this block's path, rows it writes

    const int layer = TREE ? 0 : blockIdx.z, h = blockIdx.y;
    const int row0 = blockIdx.x * RPB;
    const int tid = threadIdx.x;
    const int g = tid / kRowThreads, qd = tid % kRowThreads;
    const int row = row0 + g;  // and row + 8, ..., row + 8 (R - 1)

    int keep = p.keep;
    if constexpr (TREE) {
        if (tid < 32) {  // warp 0, lane = block row (width <= 32)
            const int lane = tid;
            const int par = lane < p.width ? tree_parent(p.parents, lane) : -1;
            const uint32_t path = lane < p.width ? tree_walk(p.parents, lane).path : 0u;
            const uint32_t has_child = __reduce_or_sync(0xffffffffu, par >= 0 ? 1u << par : 0u);
            const uint32_t leaves = __ballot_sync(0xffffffffu, lane < p.width && !((has_child >> lane) & 1u));
            uint32_t m = leaves;  // drop the blockIdx.z lowest leaves
            for (int i = 0; i < (int)blockIdx.z && m; ++i) m &= m - 1;
            const int leaf = m ? __ffs(m) - 1 : -1;  // the same on every lane
            const uint32_t mine = leaf >= 0 ? __shfl_sync(0xffffffffu, path, leaf) : 0u;
            const uint32_t earlier = leaf >= 0 ? leaves & ((1u << leaf) - 1u) : 0u;
            const uint32_t taken = __reduce_or_sync(0xffffffffu, (earlier >> lane) & 1u ? path : 0u);
            if (lane == 0) {
                path_info[0] = mine;
                path_info[1] = mine & ~taken;
            }
            if ((mine >> lane) & 1u) path_rows[__popc(mine & ((1u << lane) - 1u))] = lane;
        }
        __syncthreads();
        keep = __popc(path_info[0]);
        if (keep == 0) return;  // fewer leaves than blocks along z (uniform over the block)
    }
    auto row_at = [&](int r) -> int {
        if constexpr (TREE) return path_rows[r];
        else return p.rows.r[r];
    };

    // This thread's slices of its state rows: requested first, so that the staging below
    // runs while they are in flight.
    const size_t head_base = (((size_t)layer * p.heads + h) * p.dv + row) * DK;
    const float4* src = reinterpret_cast<const float4*>(p.snapshot + head_base) + qd;
    constexpr int kNext = kRowGroups * DK / 4;  // float4 offset of the group's next row
    float4 s[R][CH];
#pragma unroll
    for (int j = 0; j < R; ++j)
#pragma unroll
        for (int c = 0; c < CH; ++c)  // every leaf's block of a tree step reads the same state: keep it in L2 there
            s[j][c] = TREE ? __ldg(src + j * kNext + c * kRowThreads) : __ldcs(src + j * kNext + c * kRowThreads);

    // Stage k (and q), v, alpha and beta of the replayed positions, in rounds of up to
    // kStageBatch loads of each kind per thread.  A round issues all its global loads before
    // its shared-memory stores, so it costs one memory latency, and the first overlaps the
    // state loads above (a verify block of 8 positions takes one round).  q and k have
    // k_heads heads, each shared by heads / k_heads consecutive value heads; alpha and beta
    // are [width, heads] per layer.
    const int kh = p.k_heads > 0 ? p.k_heads : p.heads;
    const int hk = h / (p.heads / kh);
    const int nk = keep * (DK / 4), nv = keep * RPB;
    const uint16_t* kbits = reinterpret_cast<const uint16_t*>(p.k);
    const uint16_t* qbits = reinterpret_cast<const uint16_t*>(p.q);
    const uint16_t* vbits = reinterpret_cast<const uint16_t*>(p.v);
    for (int i0 = 0; i0 < nk || i0 < nv; i0 += kStageBatch * kBlockThreads) {
        uint2 kr[kStageBatch], qr[kStageBatch];
        uint32_t vr[kStageBatch];
#pragma unroll
        for (int u = 0; u < kStageBatch; ++u) {
            const int idx = i0 + u * kBlockThreads + tid;
            if (idx < nk) {
                const int r = idx / (DK / 4), c4 = (idx % (DK / 4)) * 4;
                const size_t base = (((size_t)layer * p.width + row_at(r)) * kh + hk) * DK + c4;
                kr[u] = __ldg(reinterpret_cast<const uint2*>(kbits + base));
                if (want_out) qr[u] = __ldg(reinterpret_cast<const uint2*>(qbits + base));
            }
            if (idx < nv) {
                const int r = idx / RPB, j = idx % RPB;
                vr[u] = __ldg(vbits + (((size_t)layer * p.width + row_at(r)) * p.heads + h) * p.dv + row0 + j);
            }
        }
        const bool with_ab = i0 == 0 && tid < keep;
        float a = 0.f, b = 0.f;
        if (with_ab) {
            const size_t ai = ((size_t)layer * p.width + row_at(tid)) * p.heads + h;
            a = __ldg(p.alpha + ai);
            b = __ldg(p.beta + ai);
        }
#pragma unroll
        for (int u = 0; u < kStageBatch; ++u) {
            const int idx = i0 + u * kBlockThreads + tid;
            if (idx < nk) {
                const int r = idx / (DK / 4), c4 = (idx % (DK / 4)) * 4;
                *reinterpret_cast<float4*>(&ks[r][c4]) = widen_bf16x4(kr[u]);
                if (want_out) {
                    const float4 qv = widen_bf16x4(qr[u]);
                    *reinterpret_cast<float4*>(&qs_sh[r][c4]) =
                        make_float4(qv.x * p.q_scale, qv.y * p.q_scale, qv.z * p.q_scale, qv.w * p.q_scale);
                }
            }
            if (idx < nv) {
                const int r = idx / RPB, j = idx % RPB;
                vs[r][j % kRowGroups].x[j / kRowGroups] = __uint_as_float(vr[u] << 16);
            }
        }
        if (with_ab) ab[tid] = make_float2(a, b);
    }

    __syncthreads();

#pragma unroll 2
    for (int r = 0; r < keep; ++r) {
        float4 k[CH];
#pragma unroll
        for (int c = 0; c < CH; ++c) k[c] = *reinterpret_cast<const float4*>(&ks[r][4 * (qd + c * kRowThreads)]);
        const float2 a_b = ab[r];
        rows_step<CH, R>(s, k, vs[r][g], a_b.x, a_b.y);
        if (want_out) {
            float4 qv[CH];
#pragma unroll
            for (int c = 0; c < CH; ++c) qv[c] = *reinterpret_cast<const float4*>(&qs_sh[r][4 * (qd + c * kRowThreads)]);
            float o[R];
            rows_dot<CH, R>(s, qv, o);
            const int t = row_at(r);
            bool write = qd < R;  // lane j of the group writes row g + 8 j
            if constexpr (TREE) write = write && ((path_info[1] >> t) & 1u);
            if (write) {
                float oj = o[0];
#pragma unroll
                for (int j = 1; j < R; ++j) oj = qd == j ? o[j] : oj;
                __nv_bfloat16 ob = __float2bfloat16_rn(oj);
                p.out[(((size_t)layer * p.width + t) * p.heads + h) * p.dv + row + qd * kRowGroups] =
                    *reinterpret_cast<uint16_t*>(&ob);
            }
        }
    }
    if constexpr (!TREE) {
        float4* dst = reinterpret_cast<float4*>(p.state_out + head_base) + qd;
#pragma unroll
        for (int j = 0; j < R; ++j)
#pragma unroll
            for (int c = 0; c < CH; ++c) __stcs(dst + j * kNext + c * kRowThreads, s[j][c]);
    }
}

// The kernels of one rows-per-thread layout, by [dk / 32 -> 0, 1, 2][mode].
template <int R>
const void* kernel_for(int dk, int mode) {
    static const void* const table[3][3] = {
        {(const void*)gdn_kernel<1, kReplay, R>, (const void*)gdn_kernel<1, kStep, R>,
         (const void*)gdn_kernel<1, kTree, R>},
        {(const void*)gdn_kernel<2, kReplay, R>, (const void*)gdn_kernel<2, kStep, R>,
         (const void*)gdn_kernel<2, kTree, R>},
        {(const void*)gdn_kernel<4, kReplay, R>, (const void*)gdn_kernel<4, kStep, R>,
         (const void*)gdn_kernel<4, kTree, R>}};
    return table[dk == 32 ? 0 : dk == 64 ? 1 : 2][mode];
}

int launch(const ReplayParams& p, int layers, cudaStream_t stream) {
    const bool tree = p.parents != nullptr;  // tree step: one layer, one block per leaf slot
    const bool with_q = p.out != nullptr && p.q != nullptr;
    const int mode = tree ? kTree : with_q ? kStep : kReplay;
    static std::once_flag once;
    static cudaError_t attr = cudaSuccess;
    std::call_once(once, [] {  // up to 64 positions of fp32 k and q: past the 48 KB default
        const int bytes = (int)smem_bytes(kMaxPositions, 128, true, kRowsPerBlock);
        for (int dk : {32, 64, 128})
            for (int m : {kReplay, kStep, kTree})
                for (const void* f : {kernel_for<4>(dk, m), kernel_for<1>(dk, m)})
                    if (attr == cudaSuccess)
                        attr = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    });
    if (attr != cudaSuccess) return fail(DFLASH_ERR_CUDA, "cudaFuncSetAttribute(gdn): %s", cudaGetErrorString(attr));
    if (p.dk != 32 && p.dk != 64 && p.dk != 128) return fail(DFLASH_ERR_UNSUPPORTED, "dk=%d not in {32, 64, 128}", p.dk);

    // Four rows per thread unless that leaves the grid under two blocks per SM; then one
    // row per thread, in four times the blocks.
    const int depth = tree ? p.width : layers;
    int dev = 0;
    DFLASH_CUDA_TRY(cudaGetDevice(&dev));
    const bool one_row = (long long)(p.dv / kRowsPerBlock) * p.heads * depth <= 2LL * sm_count(dev);
    const int rpb = one_row ? kRowGroups : kRowsPerBlock;
    const dim3 grid(p.dv / rpb, p.heads, depth);
    const size_t sm = smem_bytes(tree ? p.width : p.keep, p.dk, with_q, rpb);
    const void* fn = one_row ? kernel_for<1>(p.dk, mode) : kernel_for<4>(p.dk, mode);
    void* args[] = {const_cast<ReplayParams*>(&p)};
    DFLASH_CUDA_TRY(cudaLaunchKernel(fn, grid, dim3(kBlockThreads), args, sm, stream));
    return DFLASH_OK;
}

int check_dims(int heads, int dk, int dv) {
    if (heads < 1) return fail(DFLASH_ERR_INVALID_ARGUMENT, "heads=%d must be positive", heads);
    if (dk != 32 && dk != 64 && dk != 128) return fail(DFLASH_ERR_UNSUPPORTED, "dk=%d not in {32, 64, 128}", dk);
    if (dv < kRowsPerBlock || dv % kRowsPerBlock != 0)
        return fail(DFLASH_ERR_UNSUPPORTED, "dv=%d must be a positive multiple of %d", dv, kRowsPerBlock);
    return DFLASH_OK;
}

// conv window gather: out[l][r][:] = r+keep < kc1 ? window[l][r+keep][:] : conv_in[l][rows[r+keep-kc1]][:]
__global__ void conv_rollback_kernel(const dflash_bf16* window, dflash_bf16* out, const dflash_bf16* conv_in,
                                     RowList rows, int keep, int width, int kc1, int channels, int vec8) {
    const int l = blockIdx.y, r = blockIdx.x;
    const int pos = keep + r;
    const dflash_bf16* src = (pos < kc1) ? window + ((size_t)l * kc1 + pos) * channels
                                         : conv_in + ((size_t)l * width + rows.r[pos - kc1]) * channels;
    dflash_bf16* dst = out + ((size_t)l * kc1 + r) * channels;
    if (vec8) {
        for (int c = threadIdx.x; c < channels / 8; c += blockDim.x)
            reinterpret_cast<uint4*>(dst)[c] = reinterpret_cast<const uint4*>(src)[c];
    } else {
        for (int c = threadIdx.x; c < channels; c += blockDim.x) dst[c] = src[c];
    }
}

// Test hook: an mbarrier nothing ever arrives on, waited on with a bound.
__global__ void bounded_wait_kernel(unsigned long long limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(&bar, 0)) {
            if (globaltimer_ns() - t0 > limit_ns) {
                atomicOr(&g_device_error, DFLASH_DEVERR_TEST_WAIT);
                break;
            }
        }
    }
}

int fill_rows(RowList& rl, const int32_t* rows, int keep, int width) {
    for (int i = 0; i < keep; ++i) {
        const int r = rows ? rows[i] : i;
        if (r < 0 || r >= width)
            return fail(DFLASH_ERR_INVALID_ARGUMENT, "rows[%d]=%d outside [0, %d)", i, r, width);
        rl.r[i] = r;
    }
    return DFLASH_OK;
}

}  // namespace gdn
}  // namespace dflash

namespace dflash {
namespace gdn {

// heads value heads share k_heads key heads (q and k): k_heads divides heads.
int check_key_heads(int heads, int k_heads) {
    if (k_heads < 1 || heads % k_heads != 0)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "k_heads=%d must divide heads=%d", k_heads, heads);
    return DFLASH_OK;
}

}  // namespace gdn
}  // namespace dflash

static int gdn_step_impl(const float* state_in, float* state_out, const dflash_bf16* q, const dflash_bf16* k,
                         const dflash_bf16* v, const float* alpha, const float* beta, dflash_bf16* out, int T,
                         int heads, int k_heads, int dk, int dv, float q_scale, dflash_stream_t stream) {
    using namespace dflash;
    if (int st = gdn::check_dims(heads, dk, dv)) return st;
    if (int st = gdn::check_key_heads(heads, k_heads)) return st;
    if (T < 1 || T > gdn::kMaxPositions)
        return fail(DFLASH_ERR_UNSUPPORTED, "T=%d outside 1..%d", T, gdn::kMaxPositions);
    if (!state_in || !state_out || !k || !v || !alpha || !beta || (out && !q))
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_gdn_step: null tensor pointer");
    if (state_in == state_out)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_gdn_step: state_in and state_out must differ");
    if (!aligned16(state_in) || !aligned16(state_out) || (reinterpret_cast<uintptr_t>(k) & 7) ||
        (q && (reinterpret_cast<uintptr_t>(q) & 7)))
        return fail(DFLASH_ERR_MISALIGNED, "dflash_gdn_step: state 16-byte, q/k 8-byte alignment required");
    gdn::ReplayParams p{};
    p.snapshot = state_in;
    p.state_out = state_out;
    p.k = k;
    p.v = v;
    p.alpha = alpha;
    p.beta = beta;
    p.q = q;
    p.out = out;
    p.q_scale = q_scale;
    p.keep = T;
    p.width = T;
    p.heads = heads;
    p.k_heads = k_heads;
    p.dk = dk;
    p.dv = dv;
    if (int st = gdn::fill_rows(p.rows, nullptr, T, T)) return st;
    return gdn::launch(p, 1, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int dflash_gdn_step(const float* state_in, float* state_out, const dflash_bf16* q,
                               const dflash_bf16* k, const dflash_bf16* v, const float* alpha,
                               const float* beta, dflash_bf16* out, int T, int heads, int dk, int dv,
                               float q_scale, dflash_stream_t stream) {
    return gdn_step_impl(state_in, state_out, q, k, v, alpha, beta, out, T, heads, heads, dk, dv, q_scale, stream);
}

extern "C" int dflash_gdn_step_grouped(const float* state_in, float* state_out, const dflash_bf16* q,
                                       const dflash_bf16* k, const dflash_bf16* v, const float* alpha,
                                       const float* beta, dflash_bf16* out, int T, int heads, int k_heads, int dk,
                                       int dv, float q_scale, dflash_stream_t stream) {
    return gdn_step_impl(state_in, state_out, q, k, v, alpha, beta, out, T, heads, k_heads, dk, dv, q_scale,
                         stream);
}

static int gdn_step_tree_impl(const float* state_in, const dflash_bf16* q, const dflash_bf16* k,
                              const dflash_bf16* v, const float* alpha, const float* beta, const int32_t* parents,
                              dflash_bf16* out, int T, int heads, int k_heads, int dk, int dv, float q_scale,
                              dflash_stream_t stream) {
    using namespace dflash;
    if (int st = gdn::check_dims(heads, dk, dv)) return st;
    if (int st = gdn::check_key_heads(heads, k_heads)) return st;
    if (T < 1 || T > kMaxTreeRows) return fail(DFLASH_ERR_UNSUPPORTED, "T=%d outside 1..%d", T, kMaxTreeRows);
    if (!state_in || !q || !k || !v || !alpha || !beta || !parents || !out)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_gdn_step_tree: null pointer");
    if (!aligned16(state_in) || (reinterpret_cast<uintptr_t>(k) & 7) || (reinterpret_cast<uintptr_t>(q) & 7))
        return fail(DFLASH_ERR_MISALIGNED, "dflash_gdn_step_tree: state 16-byte, q/k 8-byte alignment required");
    gdn::ReplayParams p{};
    p.snapshot = state_in;
    p.k = k;
    p.v = v;
    p.alpha = alpha;
    p.beta = beta;
    p.q = q;
    p.out = out;
    p.q_scale = q_scale;
    p.keep = T;
    p.width = T;
    p.heads = heads;
    p.k_heads = k_heads;
    p.dk = dk;
    p.dv = dv;
    p.parents = parents;
    return gdn::launch(p, 1, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int dflash_gdn_step_tree(const float* state_in, const dflash_bf16* q, const dflash_bf16* k,
                                    const dflash_bf16* v, const float* alpha, const float* beta,
                                    const int32_t* parents, dflash_bf16* out, int T, int heads, int dk, int dv,
                                    float q_scale, dflash_stream_t stream) {
    return gdn_step_tree_impl(state_in, q, k, v, alpha, beta, parents, out, T, heads, heads, dk, dv, q_scale,
                              stream);
}

extern "C" int dflash_gdn_step_tree_grouped(const float* state_in, const dflash_bf16* q, const dflash_bf16* k,
                                            const dflash_bf16* v, const float* alpha, const float* beta,
                                            const int32_t* parents, dflash_bf16* out, int T, int heads,
                                            int k_heads, int dk, int dv, float q_scale, dflash_stream_t stream) {
    return gdn_step_tree_impl(state_in, q, k, v, alpha, beta, parents, out, T, heads, k_heads, dk, dv, q_scale,
                              stream);
}

static int gdn_replay_impl(const float* snapshot, float* state_out, const dflash_bf16* k, const dflash_bf16* v,
                           const float* alpha, const float* beta, const int32_t* rows, int keep, int width,
                           int layers, int heads, int k_heads, int dk, int dv, dflash_stream_t stream) {
    using namespace dflash;
    if (int st = gdn::check_dims(heads, dk, dv)) return st;
    if (int st = gdn::check_key_heads(heads, k_heads)) return st;
    if (layers < 1) return fail(DFLASH_ERR_INVALID_ARGUMENT, "layers=%d must be positive", layers);
    if (width < 1 || width > gdn::kMaxPositions || keep < 1 || keep > width)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "need 1 <= keep (%d) <= width (%d) <= %d", keep, width,
                    gdn::kMaxPositions);
    if (!snapshot || !state_out || !k || !v || !alpha || !beta)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_gdn_replay: null tensor pointer");
    if (snapshot == state_out)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_gdn_replay: snapshot and state_out must differ");
    if (!aligned16(snapshot) || !aligned16(state_out) || (reinterpret_cast<uintptr_t>(k) & 7))
        return fail(DFLASH_ERR_MISALIGNED, "dflash_gdn_replay: state 16-byte, k 8-byte alignment required");
    gdn::ReplayParams p{};
    p.snapshot = snapshot;
    p.state_out = state_out;
    p.k = k;
    p.v = v;
    p.alpha = alpha;
    p.beta = beta;
    p.keep = keep;
    p.width = width;
    p.heads = heads;
    p.k_heads = k_heads;
    p.dk = dk;
    p.dv = dv;
    if (int st = gdn::fill_rows(p.rows, rows, keep, width)) return st;
    return gdn::launch(p, layers, reinterpret_cast<cudaStream_t>(stream));
}

extern "C" int dflash_gdn_replay(const float* snapshot, float* state_out, const dflash_bf16* k,
                                 const dflash_bf16* v, const float* alpha, const float* beta,
                                 const int32_t* rows, int keep, int width, int layers, int heads, int dk,
                                 int dv, dflash_stream_t stream) {
    return gdn_replay_impl(snapshot, state_out, k, v, alpha, beta, rows, keep, width, layers, heads, heads, dk, dv,
                           stream);
}

extern "C" int dflash_gdn_replay_grouped(const float* snapshot, float* state_out, const dflash_bf16* k,
                                         const dflash_bf16* v, const float* alpha, const float* beta,
                                         const int32_t* rows, int keep, int width, int layers, int heads,
                                         int k_heads, int dk, int dv, dflash_stream_t stream) {
    return gdn_replay_impl(snapshot, state_out, k, v, alpha, beta, rows, keep, width, layers, heads, k_heads, dk, dv,
                           stream);
}

extern "C" int dflash_gdn_conv_rollback(const dflash_bf16* window, dflash_bf16* window_out,
                                        const dflash_bf16* conv_in, const int32_t* rows, int keep, int width,
                                        int layers, int kc1, int channels, dflash_stream_t stream) {
    using namespace dflash;
    if (layers < 1 || kc1 < 1 || channels < 1)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "layers, kc1 and channels must be positive");
    if (width < 1 || width > gdn::kMaxPositions || keep < 1 || keep > width)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "need 1 <= keep (%d) <= width (%d) <= %d", keep, width,
                    gdn::kMaxPositions);
    if (!window || !window_out || !conv_in)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_gdn_conv_rollback: null tensor pointer");
    if (window == window_out)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "dflash_gdn_conv_rollback: window_out must not alias window");
    gdn::RowList rl{};
    if (int st = gdn::fill_rows(rl, rows, keep, width)) return st;
    const int vec8 = (channels % 8 == 0) && aligned16(window) && aligned16(window_out) && aligned16(conv_in);
    dim3 grid(kc1, layers);
    gdn::conv_rollback_kernel<<<grid, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        window, window_out, conv_in, rl, keep, width, kc1, channels, vec8);
    DFLASH_CUDA_TRY(cudaGetLastError());
    return DFLASH_OK;
}

extern "C" int dflash_test_bounded_wait(uint64_t limit_ns, dflash_stream_t stream) {
    using namespace dflash;
    if (limit_ns == 0 || limit_ns > kWaitLimitNs)
        return fail(DFLASH_ERR_INVALID_ARGUMENT, "limit_ns must be in 1..%llu", kWaitLimitNs);
    gdn::bounded_wait_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_ns);
    DFLASH_CUDA_TRY(cudaGetLastError());
    return DFLASH_OK;
}
